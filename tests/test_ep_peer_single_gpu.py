"""The peer-memory expert-parallel kernels on one GPU (a one-rank group):
IPC allocation, the device-side row layout, the dispatch kernel and the
down-projection epilogue that stores rows into the owner's return buffer all
run, addressed to the rank itself.  With the fp32 return path the output is
bit-equal to MLPBlock.forward (both on the tensor-core GEMM kernel); with the bf16 return path it is within the
block's tolerance (max |diff| / max |ref| <= 2e-2, cosine >= 0.9995).  Two
steps each (the second reuses every buffer)."""
import os
import socket

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(port, E, M, exact, q):
    import datetime
    import importlib
    import sys

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    # one GEMM kernel for every row placement: the decode GEMV (<= 64 routed
    # rows) adds in a different order than the tensor-core kernel, and only
    # the latter has the peer-return epilogue, so bit-equality across the
    # placements is a property of the tensor-core kernel alone
    os.environ["GPTOSS_MOE_GEMV"] = "0"
    os.environ["GPTOSS_MOE_MX"] = "0"
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
        mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
        ep = importlib.import_module("gpt-oss-tvm_b200.ep")
        cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=E)
        p = synth.moe_params(E, seed=5)
        blk = mlp.MLPBlock(cfg, device=dev).load_state(p)
        runner = ep.ExpertParallelMoE(blk, M, exact_return=exact, peer=True)
        res = []
        for step in range(2):
            x = synth.activations(M, seed=300 + step)
            xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
            out = runner.forward(xd).clone()
            ref = blk.forward(xd)
            torch.cuda.synchronize()
            same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
            d, r = (out.float() - xd.float()).flatten(), (ref.float() - xd.float()).flatten()
            rel = float((d - r).abs().max() / r.abs().max().clamp_min(1e-30))
            cos = float(torch.dot(d, r) / (d.norm() * r.norm()).clamp_min(1e-30))
            res.append((same, rel, cos))
        err = blk.device_error() | runner.backend.device_error()
        runner.close()
        q.put((res, err, runner.last_splits))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exact", [True, False], ids=["fp32-return", "bf16-return"])
@pytest.mark.parametrize("M", [3, 300])
def test_peer_path_one_rank_matches_block(M, exact):
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    proc = ctx.Process(target=_worker, args=(_free_port(), 16, M, exact, q))
    proc.start()
    res, err, splits = q.get(timeout=300)
    proc.join(timeout=120)
    assert proc.exitcode == 0
    assert err == 0
    assert splits == ([M * 4], [M * 4])
    for same, rel, cos in res:
        if exact:
            assert same, f"peer path differs from MLPBlock.forward (rel {rel}, cos {cos})"
        else:
            assert rel <= 2e-2 and cos >= 0.9995, f"rel {rel:.3e}, cos {cos:.6f}"
