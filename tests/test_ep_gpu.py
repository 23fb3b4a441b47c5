"""Expert parallelism on 2+ GPUs, both ways of moving the rows: NCCL
all-to-all-v (peer=False) and stores into the other ranks' IPC-shared
buffers (peer=True, the default).  With the fp32 return path every rank's
output equals the single-GPU MLPBlock output for the same tokens, bit for bit
(the same kernels run on the same rows; only the rows' placement differs).
With the default bf16 return path (expert outputs rounded to bf16 before the
weighted combine) the output is within the block's tolerance of the
single-GPU one: max |diff| / max |ref| <= 2e-2, cosine >= 0.9995; and the two
ways of moving the rows give the same bits.  Every run does two steps (the
second reuses every buffer)."""
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


def _worker(rank, world, port, E, M, exact, peer, q):
    import datetime
    import importlib
    import sys

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    # one GEMM kernel for every row placement: the decode GEMV (<= 64 routed
    # rows) adds in a different order than the tensor-core kernel, and only
    # the latter has the peer-return epilogue, so bit-equality across the
    # placements is a property of the tensor-core kernel alone
    os.environ["GPTOSS_MOE_GEMV"] = "0"
    os.environ["GPTOSS_MOE_MX"] = "0"
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
        runner = ep.ExpertParallelMoE(blk, M, exact_return=exact, peer=peer)
        other = ep.ExpertParallelMoE(blk, M, exact_return=exact, peer=not peer)
        for step in range(2):
            if step:
                x = synth.activations(M, seed=200 + rank)
                xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
            out = runner.forward(xd).clone()
            out_other = other.forward(xd)
        ref = full.forward(xd)
        torch.cuda.synchronize()
        same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
        same_paths = bool(torch.equal(out.view(torch.int16), out_other.view(torch.int16)))
        # compare the MoE part (output minus the residual input)
        d, r = (out.float() - xd.float()).flatten(), (ref.float() - xd.float()).flatten()
        rel = float((d - r).abs().max() / r.abs().max().clamp_min(1e-30))
        cos = float(torch.dot(d, r) / (d.norm() * r.norm()).clamp_min(1e-30))
        q.put((rank, same, rel, cos, same_paths))
        dist.barrier()
        runner.close()
        other.close()
    finally:
        dist.destroy_process_group()


def _run(M, exact, peer=True):
    world = 2
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 16, M, exact, peer, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("peer", [True, False], ids=["peer", "nccl"])
@pytest.mark.parametrize("M", [1, 300])
def test_expert_parallel_exact_return_matches_single_gpu(M, peer):
    for rank, same, rel, cos, same_paths in _run(M, True, peer):
        assert same, f"rank {rank}: EP output differs from single-GPU (rel {rel}, cos {cos})"
        assert same_paths, f"rank {rank}: peer and NCCL paths differ"


@pytest.mark.parametrize("M", [1, 300])
def test_expert_parallel_bf16_return_within_tolerance(M):
    for rank, same, rel, cos, same_paths in _run(M, False, True):
        assert rel <= 2e-2 and cos >= 0.9995, f"rank {rank}: rel {rel:.3e}, cos {cos:.6f}"
        assert same_paths, f"rank {rank}: peer and NCCL paths differ"
