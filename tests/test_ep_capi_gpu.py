"""Expert parallelism through the C boundary (gptoss_ep_init / dispatch /
combine / forward): each rank holds its expert shard, the ranks meet through
NCCL (an id created with gptoss_ep_unique_id and handed to every rank) and
CUDA IPC buffers.  With the fp32 return path (exact_return) every rank's
output equals the single-GPU MLPBlock.forward for the same tokens bit for bit;
with the bf16 return path it is within the block's tolerance (max |diff| /
max |ref| <= 2e-2, cosine >= 0.9995).  One rank runs on one GPU; two ranks
when two GPUs are present.  Two steps each (the second reuses every buffer)."""
import ctypes
import os

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _worker(rank, world, uid, E, M, exact, q):
    import importlib
    import sys
    sys.path.insert(0, REPO)
    # one GEMM kernel for every row placement (see test_ep_gpu.py)
    os.environ["GPTOSS_MOE_GEMV"] = "0"
    os.environ["GPTOSS_MOE_MX"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    L = importlib.import_module("gpt-oss-tvm_b200._lib")
    synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=E)
    lib = L.load()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    S = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = synth.moe_params(E, seed=5)
    El = E // world
    local = {k: (v[rank * El:(rank + 1) * El] if k.startswith("mlp") else v) for k, v in p.items()}
    blk = mlp.MLPBlock(cfg, device=dev, expert_offset=rank * El, num_local_experts=El).load_state(local)
    full = mlp.MLPBlock(cfg, device=dev).load_state(p)
    blk.flags = full.flags  # the ranks agree on the GEMM operand path
    w = blk.c_weights()
    idb = (ctypes.c_ubyte * 128).from_buffer_copy(uid)
    ep = lib.gptoss_ep_init(idb, rank, world, M, E, 4, 2880, 2880, int(exact), S)
    assert ep, lib.gptoss_last_error().decode()
    try:
        # the wrong shard and a combine without a dispatch are refused
        wrong = full.c_weights()
        errs = [lib.gptoss_ep_forward(ep, None, 0, ctypes.byref(wrong), None, S) != 0 if world > 1 else True,
                lib.gptoss_ep_combine(ep, None, 0, ctypes.byref(w), None, S) != 0]
        for step in range(2):
            x = synth.activations(M, seed=100 * (step + 1) + rank)
            xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
            out = torch.empty_like(xd)
            rc = lib.gptoss_ep_forward(ep, P(xd), M, ctypes.byref(w), P(out), S)
            assert rc == 0, lib.gptoss_last_error().decode()
        ref = full.forward(xd)
        torch.cuda.synchronize()
        err = lib.gptoss_ep_error(ep)
        same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
        d, r = (out.float() - xd.float()).flatten(), (ref.float() - xd.float()).flatten()
        rel = float((d - r).abs().max() / r.abs().max().clamp_min(1e-30))
        cos = float(torch.dot(d, r) / (d.norm() * r.norm()).clamp_min(1e-30))
        q.put((rank, same, rel, cos, int(err), errs))
    finally:
        torch.cuda.synchronize()
        lib.gptoss_ep_destroy(ep)


def _run(world, M, exact, E=16):
    import importlib
    L = importlib.import_module("gpt-oss-tvm_b200._lib")
    uid = (ctypes.c_ubyte * 128)()
    assert L.load().gptoss_ep_unique_id(uid) == 0
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, bytes(uid), E, M, exact, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _worlds():
    return [1] + ([2] if torch.cuda.device_count() >= 2 else [])


@pytest.mark.parametrize("world", _worlds())
@pytest.mark.parametrize("M", [1, 300])
def test_ep_capi_exact_return_matches_single_gpu(world, M):
    for rank, same, rel, cos, err, errs in _run(world, M, True):
        assert err == 0 and all(errs)
        assert same, f"rank {rank}: output differs from one GPU (rel {rel}, cos {cos})"


@pytest.mark.parametrize("world", _worlds())
def test_ep_capi_bf16_return_within_tolerance(world):
    for rank, same, rel, cos, err, errs in _run(world, 300, False):
        assert err == 0
        assert rel <= 2e-2 and cos >= 0.9995, f"rank {rank}: rel {rel:.3e}, cos {cos:.6f}"
