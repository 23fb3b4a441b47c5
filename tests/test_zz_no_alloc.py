"""gptoss_moe_forward_noalloc: the MoE block without any device allocation.

Some callers cannot allocate device memory while the block runs (a serving
loop whose memory is planned before the first request, code that must not
call cudaMalloc because it synchronises the device, a host with no CUDA
allocator).  This entry point keeps its scratch in a fixed array inside the
library.  Its output must agree with gptoss_moe_forward (the entry point with
a library-allocated workspace) within the bf16 tolerance of the other tests,
on two calls in a row (the second one reuses the array the first one left).

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


@pytest.fixture(scope="module")
def block():
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=32)
    blk = mlp.MLPBlock(cfg).load_state(synth().moe_params(32, seed=0))
    yield blk
    blk.free_workspace()


@pytest.mark.parametrize("M", [1, 7, 64])
def test_noalloc_matches_workspace_entry_point_twice(block, M):
    lib = G._lib.load()
    x = G.dev(synth().activations(M, seed=40 + M))
    ref = torch.empty_like(x)
    G.call("gptoss_moe_forward", G.P(x), M, ctypes.byref(block.c_weights()), block.workspace(M), G.P(ref), G.S())
    w = block.c_weights()
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        rc = lib.gptoss_moe_forward_noalloc(G.P(x), M, ctypes.byref(w), G.P(out), G.S())
        assert rc == 0, lib.gptoss_last_error().decode()
        torch.cuda.synchronize()
        got, exp = G.f32(G.host(out)), G.f32(G.host(ref))
        G.tol_check(got, exp, what=f"noalloc call {call + 1}, M={M}")
        G.tol_check(got - G.f32(G.host(x)), exp - G.f32(G.host(x)), what=f"noalloc MoE part, call {call + 1}")


def test_noalloc_rejects_sizes_beyond_the_scratch(block):
    lib = G._lib.load()
    x = torch.zeros(65, 2880, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    w = block.c_weights()
    rc = lib.gptoss_moe_forward_noalloc(G.P(x), 65, ctypes.byref(w), G.P(out), G.S())
    assert rc != 0
    assert "64 tokens" in lib.gptoss_last_error().decode()
