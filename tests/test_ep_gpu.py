"""Expert parallelism on 2+ GPUs (NCCL): every rank's output must equal the
single-GPU MLPBlock output for the same tokens, bit for bit (the same kernels
run on the same rows; only the rows' placement differs)."""
import os
import socket

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 GPUs", allow_module_level=True)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, E, M, q):
    import datetime
    import importlib
    import sys

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
        mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
        ep = importlib.import_module("gpt-oss-tvm_b200.ep")
        cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=E)
        p = synth.moe_params(E, seed=5)
        El = E // world
        local = {k: (v[rank * El:(rank + 1) * El] if k.startswith("mlp") else v) for k, v in p.items()}
        blk = mlp.MLPBlock(cfg, device=dev, expert_offset=rank * El, num_local_experts=El).load_state(local)
        full = mlp.MLPBlock(cfg, device=dev).load_state(p)
        x = synth.activations(M, seed=100 + rank)
        xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
        runner = ep.ExpertParallelMoE(blk, M)
        out = runner.forward(xd)
        ref = full.forward(xd)
        torch.cuda.synchronize()
        same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
        maxdiff = float((out.float() - ref.float()).abs().max())
        q.put((rank, same, maxdiff, runner.last_splits))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 300])
def test_expert_parallel_matches_single_gpu(M):
    world = 2
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 16, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same, maxdiff, splits in res:
        assert same, f"rank {rank}: EP output differs from single-GPU (max |diff| {maxdiff})"
