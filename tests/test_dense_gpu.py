"""The tensor-core dense projections (gptoss_dense_gemm) against a plain
PyTorch fp32 reference of nn.Linear (model/attention.py:85-92, :254; the
unembedding of model/transformer.py:99-104, without bias).

Tolerance: every output within one bf16 rounding of the fp32 product,
|out - ref| <= 2^-8 |ref| + 2^-8 max|ref| * 2^-7 (the fp32 sums are the
same numbers in another order; the extra absolute term covers outputs that
cancel to near zero).  Results are deterministic: two calls give the same
bits, including the split-K cluster path at decode sizes."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402


def _case(T, N, K, bias=True, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 7 * T + N)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g, device="cuda") * 0.02).to(torch.bfloat16) if bias else None
    return x, w, b


def _run(x, w, b, err=None):
    T, K = x.shape
    N = w.shape[0]
    out = torch.full((T, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    G.call("gptoss_dense_gemm", G.P(x), T, G.P(w), G.P(b), N, K, G.P(out), G.P(err), G.S())
    return out


def _check(out, x, w, b, what):
    ref = x.float() @ w.float().t()
    if b is not None:
        ref = ref + b.float()
    o = out.float()
    assert torch.isfinite(o).all(), f"{what}: unwritten or non-finite outputs"
    tol = ref.abs() * 2.0 ** -8 + ref.abs().max() * 2.0 ** -15
    bad = (o - ref).abs() > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} outputs off by more than a bf16 rounding " \
                          f"(max {float((o - ref).abs().max()):.3e})"


@pytest.mark.parametrize("T", [1, 3, 16, 17, 64, 65, 200, 256])
@pytest.mark.parametrize("N,K", [(5120, 2880), (2880, 4096)], ids=["qkv", "out"])
def test_decode_sizes_match_fp32(T, N, K):
    x, w, b = _case(T, N, K)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = _run(x, w, b, err)
    out2 = _run(x, w, b, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    _check(out, x, w, b, f"T={T} N={N} K={K}")
    assert torch.equal(out, out2), "two calls differ"


@pytest.mark.parametrize("T", [257, 300, 1000, 4096])
@pytest.mark.parametrize("N,K", [(5120, 2880), (2880, 4096)], ids=["qkv", "out"])
def test_prefill_sizes_match_fp32(T, N, K):
    x, w, b = _case(T, N, K)
    out = _run(x, w, b)
    torch.cuda.synchronize()
    _check(out, x, w, b, f"T={T} N={N} K={K}")


@pytest.mark.parametrize("T", [1, 8, 64])
def test_unembedding_shape(T):
    """201088 x 2880 without bias (the vocabulary projection of the last tokens)."""
    x, w, _ = _case(T, 201088, 2880, bias=False)
    out = _run(x, w, None)
    torch.cuda.synchronize()
    _check(out, x, w, None, f"unembedding T={T}")
    # the greedy token is the same as from the fp32 product
    ref = x.float() @ w.float().t()
    agree = (out.float().argmax(1) == ref.argmax(1)).float().mean()
    assert agree >= 0.99


@pytest.mark.parametrize("T,N,K", [(5, 1000, 1000), (300, 1000, 520), (40, 136, 64), (2, 8, 8)])
def test_ragged_sizes(T, N, K):
    """N not a multiple of the 128/256 tiles, K not a multiple of 64 (the TMA
    zero-fills the tail), a single K chunk."""
    x, w, b = _case(T, N, K)
    out = _run(x, w, b)
    torch.cuda.synchronize()
    _check(out, x, w, b, f"T={T} N={N} K={K}")


def test_empty_and_bad_arguments():
    lib = G._lib.load()
    x, w, b = _case(4, 64, 64)
    out = torch.empty(4, 64, dtype=torch.bfloat16, device="cuda")
    assert lib.gptoss_dense_gemm(G.P(x), 0, G.P(w), G.P(b), 64, 64, G.P(out), None, G.S()) == 0
    assert lib.gptoss_dense_gemm(G.P(x), 4, G.P(w), G.P(b), 64, 60, G.P(out), None, G.S()) == -1
    assert b"multiple of 8" in lib.gptoss_last_error()
    xo = torch.empty(4 * 64 + 1, dtype=torch.bfloat16, device="cuda")[1:].view(4, 64)
    assert lib.gptoss_dense_gemm(ctypes.c_void_p(xo.data_ptr()), 4, G.P(w), G.P(b), 64, 64, G.P(out), None,
                                 G.S()) == -1
    assert b"16-byte aligned" in lib.gptoss_last_error()
    torch.cuda.synchronize()
