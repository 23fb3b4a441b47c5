"""GPU parity of the block-scaled decode GEMMs (tcgen05.mma kind::mxf8f6f4).

The activation quantizer is checked bit for bit against a numpy restatement
(e4m3 rounding to nearest even from ml_dtypes) and against its error bound;
the two grouped GEMMs and the whole block against the CPU oracle within the
bf16 tolerance of the other expert tests (max|gpu - ref| / max|ref| <= 2e-2,
cosine >= 0.9995), at decode sizes: gpt-oss-20b (32 experts) and
gpt-oss-120b (128 experts, the configs[4] 256-token batch), skewed routing
that splits an expert over several token tiles and leaves experts empty, and
scale codes outside the range of the f16 path.
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

from test_moe_gpu import _check_experts, _check_permutation, _check_routing  # noqa: E402


def quantize_ref(x: np.ndarray):
    """numpy restatement of quantize_mx_kernel: x [rows, K] float32 ->
    hi, lo [rows, K] e4m3 bytes and the exponents [rows, K/32] of each."""
    import ml_dtypes
    rows, K = x.shape
    g = x.reshape(rows, K // 32, 32).astype(np.float32)
    amax = np.abs(g).max(axis=2)
    E = ((amax.view(np.uint32) >> 23) & 0xFF).astype(np.int32) - 127
    e_hi = np.where(amax > 0, np.clip(E - 7, -127, 120), 0)
    e_lo = np.maximum(-127, e_hi - 5)
    a = (g * np.ldexp(np.float32(1), -e_hi)[..., None]).astype(np.float32)
    hi = a.astype(ml_dtypes.float8_e4m3fn)
    r = ((a - hi.astype(np.float32)) * np.ldexp(np.float32(1), e_hi - e_lo)[..., None]).astype(np.float32)
    lo = r.astype(ml_dtypes.float8_e4m3fn)
    return (hi.view(np.uint8).reshape(rows, K), lo.view(np.uint8).reshape(rows, K),
            (e_hi + 127).astype(np.uint8), (e_lo + 127).astype(np.uint8))


@pytest.mark.parametrize("src_f16", [False, True], ids=["bf16-src", "f16-src"])
def test_quantize_mx_bits_and_error_bound(src_f16):
    import ml_dtypes
    rng = np.random.default_rng(3 + src_f16)
    rows, K = 37, 2880
    x = rng.standard_normal((rows, K)).astype(np.float32)
    x[0, :32] = 0.0                                         # an all-zero group
    x[1, 32:64] = 0.0
    x[1, 40] = -3.5                                         # one non-zero value
    x[2] *= 1e4                                             # large and
    x[3] *= 1e-5                                            # small magnitudes
    x[4, ::7] = 0.0
    if src_f16:
        src = torch.from_numpy(x).to(torch.float16)
    else:
        src = torch.from_numpy(x).to(torch.bfloat16)
    xs = src.float().numpy()
    perm = rng.permutation(rows).astype(np.int32)
    d_src, d_idx = src.cuda(), G.dev(perm)
    q = torch.empty(rows, 2 * K, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(rows, 192, dtype=torch.uint8, device="cuda")
    G.call("gptoss_moe_quantize_mx", G.P(d_src), int(src_f16), G.P(d_idx), rows, K, G.P(q), G.P(sc), G.S())
    torch.cuda.synchronize()
    qh, sch = G.host(q), G.host(sc)
    hi, lo, eh, el = quantize_ref(xs[perm])
    np.testing.assert_array_equal(qh[:, :K], hi)
    np.testing.assert_array_equal(qh[:, K:], lo)
    np.testing.assert_array_equal(sch[:, :K // 32], eh)
    np.testing.assert_array_equal(sch[:, 96:96 + K // 32], el)
    # value: 2^e_hi hi + 2^e_lo lo is within 2^-8 |x| (+ the lo subnormal floor)
    fh = qh[:, :K].view(ml_dtypes.float8_e4m3fn).astype(np.float64)
    fl = qh[:, K:].view(ml_dtypes.float8_e4m3fn).astype(np.float64)
    sh = np.repeat(np.ldexp(1.0, eh.astype(np.int32) - 127), 32, axis=1)
    sl = np.repeat(np.ldexp(1.0, el.astype(np.int32) - 127), 32, axis=1)
    got = fh * sh + fl * sl
    ref = xs[perm].astype(np.float64)
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + sl * 2.0 ** -9 + 1e-30)


def _block_case(oracle, E, M, seed, scale_lo=118, scale_hi=124, routing=None, sample=None):
    p = synth().moe_params(E, seed=seed, scale_lo=scale_lo, scale_hi=scale_hi)
    x = synth().activations(M, seed=seed + 1)
    mask = None
    if sample is not None:
        mask = np.zeros(M, np.uint8)
        mask[sample] = 1
    if routing is not None:
        ref = _oracle_with_routing(oracle, x, p, routing, mask)
    else:
        ref = oracle.moe_forward(x, p, rows_mask=mask, return_all=True)
    ref["x"] = x
    r = G.MoEPieces(p, mx=True).run(x, routing=routing)
    return p, x, ref, r


def _oracle_with_routing(oracle, x, p, routing, mask):
    """The oracle block with the router's choice replaced by `routing`."""
    w, idx = routing
    t = oracle.rms_norm(x, p["norm_weight"])
    h1 = oracle.moe_einsum(t, idx, p["mlp1_weight_blocks"], p["mlp1_weight_scales"], p["mlp1_bias"], mask)
    y = oracle.swiglu(h1)
    h2 = oracle.moe_einsum(y, idx, p["mlp2_weight_blocks"], p["mlp2_weight_scales"], p["mlp2_bias"], mask)
    gated, out = oracle.gating_residual(h2, w, x)
    return dict(t=t, weights=w, indices=idx, y=y, h2=h2, gated=gated, out=out)


@pytest.mark.parametrize("E,M", [(32, 17), (32, 64)])
def test_mx_block_gpt_oss_20b_decode(oracle, E, M):
    _, _, ref, r = _block_case(oracle, E, M, seed=200 + M)
    _check_routing(r, ref, M, E)
    _check_permutation(oracle, r, E)
    _check_experts(oracle, r, ref)


def test_mx_block_gpt_oss_120b_decode_256_tokens(oracle):
    """configs[4] decode batch: 256 tokens over 128 experts (1024 routed rows)."""
    M = 256
    sample = np.sort(np.random.default_rng(5).choice(M, 24, replace=False))
    _, _, ref, r = _block_case(oracle, 128, M, seed=300, sample=sample)
    _check_routing(r, ref, M, 128)
    _check_experts(oracle, r, ref, sample)


def test_mx_block_skewed_routing_splits_tiles_and_leaves_experts_empty(oracle):
    """60 tokens all routed to experts 0-3 of 32: each of those experts has 60
    rows (two token tiles of <= 32), the other 28 experts none."""
    M, E = 60, 32
    S = synth()
    idx = np.tile(np.array([[3, 0, 2, 1]], np.int32), (M, 1))
    w = S.bf16_bits(np.tile(np.array([[0.4, 0.3, 0.2, 0.1]], np.float32), (M, 1)))
    _, _, ref, r = _block_case(oracle, E, M, seed=400, routing=(w, idx))
    assert int(r["tile_rows"][0]) <= 32 and int(r["tile_ptr"][1]) == 2
    _check_experts(oracle, r, ref)


def test_mx_block_scale_codes_outside_the_f16_range(oracle):
    """Scale codes 100..150 rule out the f16 path; the block-scaled MMA takes
    the E8M0 exponents as they are."""
    M, E = 40, 32
    p, x, ref, r = _block_case(oracle, E, M, seed=500, scale_lo=100, scale_hi=150)
    assert not G.MoEPieces(p).f16
    _check_experts(oracle, r, ref)


def test_moe_forward_takes_the_block_scaled_path(oracle, monkeypatch):
    """gptoss_moe_forward and the no-allocation forward at a decode size with
    GPTOSS_MOE_MX=1: bit-equal to the step-by-step block-scaled path, and to
    each other."""
    M, E = 64, 32
    p = synth().moe_params(E, seed=600)
    x = synth().activations(M, seed=601)
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=E)
    blk = mlp.MLPBlock(cfg).load_state(p)
    monkeypatch.setenv("GPTOSS_MOE_MX", "1")
    out = G.host(blk.forward(G.dev(x).reshape(1, M, 2880))).reshape(M, 2880)
    r = G.MoEPieces(p, mx=True).run(x)
    np.testing.assert_array_equal(out, r["out"])
    lib = G._lib.load()
    xd = G.dev(x)
    o2 = torch.empty_like(xd)
    w = blk.c_weights()
    assert lib.gptoss_moe_forward_noalloc(G.P(xd), M, ctypes.byref(w), G.P(o2), G.S()) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(G.host(o2), out)
    assert blk.device_error() == 0 and lib.gptoss_moe_noalloc_error() == 0
    ref = oracle.moe_forward(x, p)
    G.tol_check(G.f32(out), G.f32(ref), what="block output (block-scaled path)")
    blk.free_workspace()
