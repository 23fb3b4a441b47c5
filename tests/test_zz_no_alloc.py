"""gptoss_moe_forward_noalloc: the MoE block without any device allocation.

Some callers cannot allocate device memory while the block runs (a serving
loop whose memory is planned before the first request, code that must not
call cudaMalloc because it synchronises the device, a host with no CUDA
allocator).  This entry point keeps its scratch in a fixed array inside the
library.  Both entry points launch the same kernels on the same rows, so the
output must equal gptoss_moe_forward's (the entry point with a
library-allocated workspace) bit for bit; it is also held to the bf16
tolerance of the other tests against it, so a failure says how far off it is.

The calls run in a sequence that reuses the array the previous call left:
64 tokens, then 7 and 1 with different inputs, so a smaller call follows a
larger one (stale expert offsets, token tiles or rows in the array would show
up), over 32 and 128 experts and both GEMM operand paths (f16 and bf16).
The device error word in the array must stay clear.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one; it also passes alone in a fresh process.
"""
import ctypes
import importlib

import numpy as np
import pytest

from conftest import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402


@pytest.fixture(scope="module", params=[32, 128], ids=["E32", "E128"])
def block(request):
    E = request.param
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=E)
    blk = mlp.MLPBlock(cfg).load_state(synth().moe_params(E, seed=E))
    assert blk.f16_path, "the synthetic scale codes allow the f16 path"
    yield blk
    blk.free_workspace()


@pytest.mark.parametrize("f16", [True, False], ids=["f16", "bf16"])
def test_noalloc_matches_workspace_entry_point_bit_for_bit(block, f16):
    lib = G._lib.load()
    assert lib.gptoss_moe_noalloc_error() == 0
    w = block.c_weights()
    if not f16:
        w.flags = 0  # exact bf16 weight decode and bf16 activations
    for M in (64, 7, 1, 64):
        x = G.dev(synth().activations(M, seed=1000 * M + block.num_experts + (0 if f16 else 1)))
        ref = torch.empty_like(x)
        G.call("gptoss_moe_forward", G.P(x), M, ctypes.byref(w), block.workspace(64), G.P(ref), G.S())
        out = torch.full_like(x, float("nan"))
        rc = lib.gptoss_moe_forward_noalloc(G.P(x), M, ctypes.byref(w), G.P(out), G.S())
        assert rc == 0, lib.gptoss_last_error().decode()
        torch.cuda.synchronize()
        got, exp = G.host(out), G.host(ref)
        G.tol_check(G.f32(got), G.f32(exp), what=f"noalloc M={M}")
        assert np.array_equal(got, exp), f"noalloc M={M}: {int((got != exp).sum())} elements differ"
        assert lib.gptoss_moe_noalloc_error() == 0, "device error word set"
    assert block.device_error() == 0


def test_noalloc_twice_in_a_row_on_the_same_input(block):
    lib = G._lib.load()
    M = 16
    x = G.dev(synth().activations(M, seed=77))
    ref = torch.empty_like(x)
    w = block.c_weights()
    G.call("gptoss_moe_forward", G.P(x), M, ctypes.byref(w), block.workspace(64), G.P(ref), G.S())
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        rc = lib.gptoss_moe_forward_noalloc(G.P(x), M, ctypes.byref(w), G.P(out), G.S())
        assert rc == 0, lib.gptoss_last_error().decode()
        torch.cuda.synchronize()
        assert np.array_equal(G.host(out), G.host(ref)), f"call {call + 1} differs"
    assert lib.gptoss_moe_noalloc_error() == 0


def test_noalloc_rejects_sizes_beyond_the_scratch(block):
    lib = G._lib.load()
    x = torch.zeros(65, 2880, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    w = block.c_weights()
    rc = lib.gptoss_moe_forward_noalloc(G.P(x), 65, ctypes.byref(w), G.P(out), G.S())
    assert rc != 0
    assert "64 tokens" in lib.gptoss_last_error().decode()
    w.num_experts = w.num_local_experts = 256
    rc = lib.gptoss_moe_forward_noalloc(G.P(x), 1, ctypes.byref(w), G.P(out), G.S())
    assert rc != 0
    assert "128 experts" in lib.gptoss_last_error().decode()
