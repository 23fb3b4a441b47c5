"""GPU parity of the MoE block (C ABI) against the CPU oracle.

Bit-exact: RMSNorm, router logits, top-k indices and softmax weights, the
expert-major permutation and the MXFP4 decode.  Tolerance (bf16): the
expert GEMM outputs and the block output, with
max|gpu - ref| / max|ref| <= 2e-2 and cosine >= 0.9995.
"""
import ctypes

import numpy as np
import pytest

from conftest import golden, synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402


@pytest.fixture(scope="module")
def params_e8():
    return synth().moe_params(8, seed=10)


def _check_routing(r, ref, M, E, k=4):
    np.testing.assert_array_equal(r["t"], ref["t"])
    np.testing.assert_array_equal(r["logits"], ref["logits"])
    np.testing.assert_array_equal(r["indices"], ref["indices"])
    np.testing.assert_array_equal(r["weights"], ref["weights"])


def _check_permutation(oracle, r, E, k=4):
    indptr, tok, rev, exp_ = oracle.moe_permute(r["indices"], E)
    np.testing.assert_array_equal(r["indptr"], indptr)
    np.testing.assert_array_equal(r["token_of_row"], tok)
    np.testing.assert_array_equal(r["row_of_pair"], rev)
    np.testing.assert_array_equal(r["expert_of_row"], exp_)


def _check_experts(oracle, r, ref, rows=None):
    """y and h2 of the sampled tokens (permuted rows) against the oracle."""
    M, k = r["indices"].shape
    rows = np.arange(M) if rows is None else rows
    rev = r["row_of_pair"].reshape(M, k)
    y_gpu = r["y"][rev[rows].ravel()]
    y_ref = ref["y"][rows].reshape(-1, ref["y"].shape[-1])
    G.tol_check(y_gpu, y_ref, what="mlp1+swiglu")
    h2_gpu = r["h2"][rev[rows].ravel()]
    h2_ref = ref["h2"][rows].reshape(-1, ref["h2"].shape[-1])
    G.tol_check(h2_gpu, h2_ref, what="mlp2")
    G.tol_check(G.f32(r["out"][rows]) - G.f32(ref["x"][rows]), G.f32(ref["gated"][rows]), what="gated sum")
    G.tol_check(G.f32(r["out"][rows]), G.f32(ref["out"][rows]), what="block output")


@pytest.mark.parametrize("f16", [True, False], ids=["f16-path", "bf16-path"])
@pytest.mark.parametrize("M", [1, 5, 37, 300])
def test_moe_block_e8(oracle, params_e8, M, f16):
    x = synth().activations(M, seed=100 + M)
    rows = None if M <= 40 else np.sort(np.random.default_rng(M).choice(M, 24, replace=False))
    mask = None
    if rows is not None:
        mask = np.zeros(M, np.uint8)
        mask[rows] = 1
    ref = oracle.moe_forward(x, params_e8, rows_mask=mask, return_all=True)
    ref["x"] = x
    pieces = G.MoEPieces(params_e8, f16=f16)
    assert pieces.f16 == f16, "the synthetic weights (scale codes 118..124) must allow the f16 path"
    r = pieces.run(x)
    _check_routing(r, ref, M, 8)
    _check_permutation(oracle, r, 8)
    _check_experts(oracle, r, ref, rows)


def test_moe_forward_entry_point_matches_pieces(params_e8):
    """gptoss_moe_forward (one call, library workspace) == the step-by-step path."""
    import importlib
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=8)
    blk = mlp.MLPBlock(cfg).load_state(params_e8)
    x = synth().activations(64, seed=7)
    out = blk.forward(G.dev(x).reshape(1, 64, 2880))
    r = G.MoEPieces(params_e8, mx=None).run(x)
    np.testing.assert_array_equal(G.host(out).reshape(64, 2880), r["out"])
    assert blk.device_error() == 0


def test_golden_moe_e8_reference_outputs():
    """Against the reference's own outputs (TVM C target), no oracle involved."""
    f = golden("moe_e8.npz")
    p = synth().moe_params(8, seed=10)
    pieces = G.MoEPieces(p)
    for M in (1, 5, 16):
        x = synth().activations(M, seed=int(f[f"m{M}_xseed"]))
        r = pieces.run(x)
        np.testing.assert_array_equal(r["logits"], f[f"m{M}_logits"])
        np.testing.assert_array_equal(r["indices"], f[f"m{M}_indices"])
        np.testing.assert_array_equal(r["weights"], f[f"m{M}_weights"])
        G.tol_check(G.f32(r["out"]), G.f32(f[f"m{M}_out"]), what=f"block output M={M}")
        G.tol_check(G.f32(r["out"]) - G.f32(x), G.f32(f[f"m{M}_gated"].reshape(M, -1)), what=f"gated M={M}")


def test_golden_config0_reference_outputs():
    """gpt-oss-20b MoE block (config 0): 1 decode token and 128 prefill tokens."""
    f = golden("moe_cfg0.npz")
    p = synth().moe_params(32, seed=0)
    pieces = G.MoEPieces(p)
    x1 = synth().activations(1, seed=1)
    r = pieces.run(x1)
    for key in ("t", "logits", "indices", "weights"):
        np.testing.assert_array_equal(r[key], f["m1_" + key])
    G.tol_check(G.f32(r["out"]), G.f32(f["m1_out"]), what="config0 decode")
    x = synth().activations(128, seed=1)
    r = pieces.run(x)
    np.testing.assert_array_equal(r["logits"], f["m128_logits"])
    np.testing.assert_array_equal(r["indices"], f["m128_indices"])
    np.testing.assert_array_equal(r["weights"], f["m128_weights"])
    G.tol_check(G.f32(r["out"]), G.f32(f["m128_out"]), what="config0 prefill")
    G.tol_check(G.f32(r["out"]) - G.f32(x), G.f32(f["m128_out"]) - G.f32(x), what="config0 prefill moe part")


def test_config3_scale_routing_bit_exact_and_sampled_experts(oracle):
    """gpt-oss-120b MoE layer at full prefill size (8192 tokens, 128 experts):
    routing and permutation bit-exact for every token, expert outputs on a
    sample of tokens."""
    S = synth()
    p = S.moe_params(128, seed=0)
    M = 8192
    x = S.activations(M, seed=1)
    r = G.MoEPieces(p).run(x)
    t = oracle.rms_norm(x, p["norm_weight"])
    np.testing.assert_array_equal(r["t"], t)
    g = oracle.router(t, p["gate_weight"], p["gate_bias"])
    np.testing.assert_array_equal(r["logits"], g)
    w, idx, _ = oracle.topk_softmax(g, 4)
    np.testing.assert_array_equal(r["indices"], idx)
    np.testing.assert_array_equal(r["weights"], w)
    _check_permutation(oracle, r, 128)
    counts = np.diff(r["indptr"])
    assert counts.max() > 160, "expected some expert with more than one token tile"
    rows = np.sort(np.random.default_rng(3).choice(M, 12, replace=False))
    # include a token of the most loaded expert
    e_max = int(np.argmax(counts))
    rows = np.unique(np.concatenate([rows, [int(r["token_of_row"][r["indptr"][e_max + 1] - 1])]]))
    mask = np.zeros(M, np.uint8)
    mask[rows] = 1
    ref = oracle.moe_forward(x, p, rows_mask=mask, return_all=True)
    ref["x"] = x
    _check_experts(oracle, r, ref, rows)


@pytest.mark.parametrize("f16", [True, False], ids=["f16-path", "bf16-path"])
def test_forced_routing_multi_tile_and_empty_experts(oracle, params_e8, f16):
    """Every token routed to experts 0..3 (600 rows each -> 4 token tiles of
    150 rows per expert, 4 empty experts)."""
    M = 600
    x = synth().activations(M, seed=9)
    idx = np.tile(np.array([[2, 0, 3, 1]], np.int32), (M, 1))
    wts = synth().bf16_bits(np.tile(np.array([[0.4, 0.3, 0.2, 0.1]], np.float32), (M, 1)))
    r = G.MoEPieces(params_e8, f16=f16).run(x, routing=(wts, idx))
    indptr, tok, rev, _ = oracle.moe_permute(idx, 8)
    np.testing.assert_array_equal(r["indptr"], indptr)
    nt = -(-M // 160)  # token tiles of at most 160 rows per expert
    np.testing.assert_array_equal(r["tile_ptr"], [0, nt, 2 * nt, 3 * nt] + [4 * nt] * 5)
    rows = np.array([0, 1, 255, 256, 257, 511, 512, 599])
    t = oracle.rms_norm(x, params_e8["norm_weight"])
    h1 = oracle.moe_einsum(t[rows], idx[rows], params_e8["mlp1_weight_blocks"], params_e8["mlp1_weight_scales"],
                           params_e8["mlp1_bias"])
    y = oracle.swiglu(h1)
    h2 = oracle.moe_einsum(y, idx[rows], params_e8["mlp2_weight_blocks"], params_e8["mlp2_weight_scales"],
                           params_e8["mlp2_bias"])
    revm = r["row_of_pair"].reshape(M, 4)
    G.tol_check(r["y"][revm[rows].ravel()], y.reshape(-1, 2880), what="forced mlp1")
    G.tol_check(r["h2"][revm[rows].ravel()], h2.reshape(-1, 2880), what="forced mlp2")
    _, out = oracle.gating_residual(h2, wts[rows], x[rows])
    G.tol_check(G.f32(r["out"][rows]), G.f32(out), what="forced output")


@pytest.mark.parametrize("f16", [True, False], ids=["f16-path", "bf16-path"])
@pytest.mark.parametrize("case", ["forced", "router"])
def test_cta_pair_kernel_matches_single_cta_kernel(params_e8, f16, case, monkeypatch):
    """Large token tiles run on CTA pairs (tcgen05.mma.cta_group::2: 256
    weight rows per MMA, each SM staging half of the token rows).  The
    single-CTA kernel (GPTOSS_MOE_PAIR=0) adds the same products in the same
    K order, so both give the same bits.  Covers N = 5760 (22.5 pairs of
    128-row tiles: the last pair's second CTA has no rows) and N = 2880 (the
    last pair's first CTA has 64 rows), token tiles of 150 rows (MMA N 160,
    halves of 80 rows), of 17 rows (N 32, halves of 16) and the router's
    mix of sizes."""
    M = 600 if case == "forced" else 300
    x = synth().activations(M, seed=21)
    routing = None
    if case == "forced":
        idx = np.tile(np.array([[2, 0, 3, 1]], np.int32), (M, 1))
        idx[:17] = [[4, 5, 6, 7]]
        wts = synth().bf16_bits(np.tile(np.array([[0.4, 0.3, 0.2, 0.1]], np.float32), (M, 1)))
        routing = (wts, idx)
    monkeypatch.setenv("GPTOSS_MOE_PAIR", "1")
    a = G.MoEPieces(params_e8, f16=f16).run(x, routing=routing)
    monkeypatch.setenv("GPTOSS_MOE_PAIR", "0")
    b = G.MoEPieces(params_e8, f16=f16).run(x, routing=routing)
    np.testing.assert_array_equal(a["y"], b["y"])
    np.testing.assert_array_equal(a["h2"], b["h2"])
    np.testing.assert_array_equal(a["out"], b["out"])


@pytest.mark.parametrize("f16", [True, False], ids=["f16-path", "bf16-path"])
def test_forced_routing_small_tiles(oracle, f16):
    """Decode-sized batch (M*k <= 8E rows) runs the GEMM's small-tile variant:
    256 tokens all routed to experts 0..3 of 128 -> 8 token tiles of 32 rows
    per expert, 124 empty experts."""
    S = synth()
    p = S.moe_params(128, seed=0)
    M = 256
    x = S.activations(M, seed=11)
    idx = np.tile(np.array([[1, 3, 0, 2]], np.int32), (M, 1))
    wts = S.bf16_bits(np.tile(np.array([[0.5, 0.25, 0.125, 0.125]], np.float32), (M, 1)))
    r = G.MoEPieces(p, f16=f16).run(x, routing=(wts, idx))
    indptr, _, _, _ = oracle.moe_permute(idx, 128)
    np.testing.assert_array_equal(r["indptr"], indptr)
    np.testing.assert_array_equal(r["tile_ptr"], [0, 8, 16, 24] + [32] * 125)
    np.testing.assert_array_equal(r["tile_rows"][:4], [32] * 4)
    rows = np.array([0, 1, 31, 32, 33, 127, 200, 255])
    t = oracle.rms_norm(x, p["norm_weight"])
    h1 = oracle.moe_einsum(t[rows], idx[rows], p["mlp1_weight_blocks"], p["mlp1_weight_scales"], p["mlp1_bias"])
    y = oracle.swiglu(h1)
    h2 = oracle.moe_einsum(y, idx[rows], p["mlp2_weight_blocks"], p["mlp2_weight_scales"], p["mlp2_bias"])
    revm = r["row_of_pair"].reshape(M, 4)
    G.tol_check(r["y"][revm[rows].ravel()], y.reshape(-1, 2880), what="small-tile mlp1")
    G.tol_check(r["h2"][revm[rows].ravel()], h2.reshape(-1, 2880), what="small-tile mlp2")
    _, out = oracle.gating_residual(h2, wts[rows], x[rows])
    G.tol_check(G.f32(r["out"][rows]), G.f32(out), what="small-tile output")


@pytest.mark.parametrize("case", ["e32-m1", "e32-m8", "e32-m16", "e128-m2", "forced-9-7"])
def test_decode_gemv_matches_tensor_core_kernel(oracle, case, monkeypatch):
    """Small decode batches (<= 64 routed rows) on the f16 path run the MXFP4
    GEMV kernel (registers -> mma.sync, split-K over four warps);
    GPTOSS_MOE_GEMV=0 runs the tensor-core small-tile kernel on the same
    rows.  Both multiply the same exactly decoded f16 weights and f16
    activations with fp32 accumulation, in different orders: the outputs agree
    to fp32 rounding (h2 within 5e-3 of max|h2|; y within 2^-10 relative plus
    1e-4 of max|y|) and are within the bf16 tolerance of the oracle.
    "forced-9-7": experts with 9 rows (a second 8-row pass) and 7 rows."""
    S = synth()
    E, M = {"e32-m1": (32, 1), "e32-m8": (32, 8), "e32-m16": (32, 16), "e128-m2": (128, 2),
            "forced-9-7": (32, 16)}[case]
    p = S.moe_params(E, seed=4)
    x = S.activations(M, seed=5)
    routing = None
    if case == "forced-9-7":
        idx = np.zeros((M, 4), np.int32)
        idx[:9] = [0, 1, 2, 3]
        idx[9:] = [4, 5, 6, 7]
        wts = S.bf16_bits(np.tile(np.array([[0.4, 0.3, 0.2, 0.1]], np.float32), (M, 1)))
        routing = (wts, idx)
    monkeypatch.setenv("GPTOSS_MOE_GEMV", "1")
    pieces = G.MoEPieces(p, f16=True)
    assert pieces.f16
    a = pieces.run(x, routing=routing)
    monkeypatch.setenv("GPTOSS_MOE_GEMV", "0")
    b = pieces.run(x, routing=routing)
    assert np.max(np.abs(a["h2"] - b["h2"])) <= 5e-3 * np.max(np.abs(b["h2"])), "h2: GEMV vs tensor-core kernel"
    ya, yb = a["y"].astype(np.float64), b["y"].astype(np.float64)
    assert np.all(np.abs(ya - yb) <= 2.0 ** -10 * np.abs(yb) + 1e-4 * np.abs(yb).max()), "y: GEMV vs tensor core"
    G.tol_check(G.f32(a["out"]), G.f32(b["out"]), what="block output GEMV vs tensor core")
    if routing is None:
        ref = oracle.moe_forward(x, p, return_all=True)
        G.tol_check(a["h2"][a["row_of_pair"].reshape(M, 4)].reshape(-1, 2880),
                    ref["h2"].reshape(-1, 2880), what="GEMV mlp2 vs oracle")
        G.tol_check(G.f32(a["out"]) - G.f32(x), G.f32(ref["gated"]), what="GEMV gated sum vs oracle")


def test_f16_path_disabled_for_out_of_range_scales():
    """A scale code outside 104..140 makes gptoss_moe_weights_prepare clear the
    f16 flag; the exact bf16 path then matches the oracle."""
    p = dict(synth().moe_params(8, seed=10))
    p["mlp2_weight_scales"] = p["mlp2_weight_scales"].copy()
    p["mlp2_weight_scales"][3, 5, 7] = 141
    assert not G.MoEPieces(p).f16
    p["mlp2_weight_scales"][3, 5, 7] = 103
    assert not G.MoEPieces(p).f16
    p["mlp2_weight_scales"][3, 5, 7] = 104
    assert G.MoEPieces(p).f16


def test_topk_ties_golden():
    f = golden("topk_ties.npz")
    logits = G.dev(f["logits"])
    M, E = f["logits"].shape
    w = torch.empty(M, 4, dtype=torch.bfloat16, device="cuda")
    idx = torch.empty(M, 4, dtype=torch.int32, device="cuda")
    G.call("gptoss_moe_topk_softmax", G.P(logits), M, E, 4, G.P(w), G.P(idx), None, G.S())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(G.host(idx), f["indices"])
    np.testing.assert_array_equal(G.host(w), f["weights"])


def test_mxfp4_dequant_bit_exact_all_scale_codes(oracle):
    rng = np.random.default_rng(11)
    rows, Gr = 300, 90
    blocks = rng.integers(0, 256, size=(rows, Gr, 16), dtype=np.uint8)
    scales = (np.arange(rows * Gr) % 255).astype(np.uint8).reshape(rows, Gr)  # every code 0..254
    out = torch.empty(rows, Gr * 32, dtype=torch.bfloat16, device="cuda")
    bd, sd = G.dev(blocks), G.dev(scales)
    G.call("gptoss_mxfp4_dequant", G.P(bd), G.P(sd), rows, Gr, G.P(out), G.S())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(G.host(out), oracle.mxfp4_dequant(blocks, scales))


def test_mxfp4_dequant_golden_reference():
    f = golden("mxfp4_decode.npz")
    rng = np.random.default_rng(5)
    blocks = rng.integers(0, 256, size=(2, 5760, 90, 16), dtype=np.uint8)
    scales = rng.integers(100, 150, size=(2, 5760, 90), dtype=np.uint8)
    scales[0, :8, :] = np.arange(8 * 90).reshape(8, 90) % 256
    scales[0, :8, :][scales[0, :8, :] == 255] = 254
    b = np.ascontiguousarray(blocks[:, :64])
    s = np.ascontiguousarray(scales[:, :64])
    out = torch.empty(2 * 64, 2880, dtype=torch.bfloat16, device="cuda")
    bd, sd = G.dev(b), G.dev(s)
    G.call("gptoss_mxfp4_dequant", G.P(bd), G.P(sd), 128, 90, G.P(out), G.S())
    torch.cuda.synchronize()
    dec = G.f32(G.host(out)).reshape(2, 64, 2880)
    kpos, ref = f["kpos"], f["out_rows"]
    for si in range(64):
        for rr, e in enumerate((0, 1, 0, 1)):
            np.testing.assert_array_equal(dec[e, :, kpos[si]] + np.float32(0), ref[si, rr] + np.float32(0))


def test_rmsnorm_bit_exact_odd_sizes(oracle):
    """The streaming kernel (rows in 256-value chunks through a 4-slot ring)
    at decode and prefill token counts, row lengths with a short last chunk
    (520) or fewer values than one chunk (64), and the whole-row kernel it
    falls back to when the weight or output is not 16-byte aligned."""
    rng = np.random.default_rng(12)
    for M, H in ((1, 2880), (33, 2880), (257, 2880), (5000, 2880), (8192, 2880), (300, 520), (70, 64),
                 (9, 4096)):
        x = synth().bf16_bits(rng.standard_normal((M, H)).astype(np.float32) * 3)
        w = synth().bf16_bits(rng.standard_normal(H).astype(np.float32))
        ref = oracle.rms_norm(x, w)
        xd, wd = G.dev(x), G.dev(w)  # keep the device copies alive until the kernel has run
        out = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
        G.call("gptoss_rms_norm", G.P(xd), G.P(wd), M, H, G.ctypes.c_float(1e-5), G.P(out), G.S())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(G.host(out), ref, err_msg=f"M={M} H={H}")
        if M <= 257:  # unaligned output: the whole-row kernel
            buf = torch.empty(M * H + 4, dtype=torch.bfloat16, device="cuda")
            out2 = buf[4:].view(M, H)
            G.call("gptoss_rms_norm", G.P(xd), G.P(wd), M, H, G.ctypes.c_float(1e-5), G.P(out2), G.S())
            torch.cuda.synchronize()
            np.testing.assert_array_equal(G.host(out2.contiguous()), ref, err_msg=f"M={M} H={H} unaligned")


@pytest.mark.parametrize("E", [8, 32, 128])
@pytest.mark.parametrize("fma", ["bf16", "fp32"])
def test_router_bit_exact_both_kernels(oracle, E, fma, monkeypatch):
    """Router logits at token counts served by the per-chain kernel (<= 512
    tokens) and by the register-tiled kernel (> 512), bit-exact; both on the
    bf16 FMA pipe (the default) and on fp32 FMA + conversion
    (GPTOSS_ROUTER_BF16=0)."""
    monkeypatch.setenv("GPTOSS_ROUTER_BF16", "1" if fma == "bf16" else "0")
    rng = np.random.default_rng(40 + E)
    S = synth()
    Wg = S.bf16_bits(rng.standard_normal((E, 2880)).astype(np.float32) * 0.02)
    bg = S.bf16_bits(rng.standard_normal(E).astype(np.float32) * 0.1)
    for M in (1, 17, 512, 513):
        t = S.bf16_bits(rng.standard_normal((M, 2880)).astype(np.float32))
        td, wd, bd = G.dev(t), G.dev(Wg), G.dev(bg)
        logits = torch.empty(M, E, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(M, 4, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(M, 4, dtype=torch.int32, device="cuda")
        G.call("gptoss_moe_router", G.P(td), G.P(wd), G.P(bd), M, E, 2880, 4, G.P(logits), G.P(w), G.P(idx), None,
               G.S())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(G.host(logits), oracle.router(t, Wg, bg), err_msg=f"M={M} E={E}")


def test_empty_inputs_and_oversized_calls(params_e8):
    """Zero tokens is a valid call everywhere on the path (nothing launched,
    return code 0, empty outputs); more tokens than a workspace holds is an
    error with a message, not a launch."""
    import ctypes
    import importlib
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=8)
    blk = mlp.MLPBlock(cfg).load_state(params_e8)
    x0 = torch.empty(1, 0, 2880, dtype=torch.bfloat16, device="cuda")
    y0 = blk.forward(x0)
    torch.cuda.synchronize()
    assert tuple(y0.shape) == (1, 0, 2880) and blk.device_error() == 0
    lib = G._lib.load()
    z = torch.zeros(64, dtype=torch.int32, device="cuda")
    S = G.S()
    assert lib.gptoss_attn_prefill(G.P(z), G.P(z), G.P(z), None, 0, 0, 64, 8, 64, 0, ctypes.c_float(0.125),
                                   G.P(z), None, S) == 0
    assert lib.gptoss_attn_decode(G.P(z), G.P(z), G.P(z), G.P(z), 0, 16, 64, 8, 64, 0, ctypes.c_float(0.125), None,
                                  G.P(z), 0, G.P(z), None, S) == 0
    w = torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda")
    assert lib.gptoss_dense_gemv(G.P(z), 0, G.P(w), None, 8, 64, G.P(z), S) == 0
    # a workspace sized for 4 tokens refuses 5
    ws = lib.gptoss_moe_workspace_create(4, 8, 4, 2880, 2880)
    assert ws
    try:
        wts = blk.c_weights()
        x5 = torch.zeros(5, 2880, dtype=torch.bfloat16, device="cuda")
        o5 = torch.empty_like(x5)
        assert lib.gptoss_moe_forward(G.P(x5), 5, ctypes.byref(wts), ws, G.P(o5), S) != 0
        assert b"max_tokens" in lib.gptoss_last_error()
    finally:
        lib.gptoss_moe_workspace_destroy(ws)
        blk.free_workspace()
    torch.cuda.synchronize()


@pytest.mark.parametrize("E", [8, 32, 128])
def test_fused_decode_routing_equals_separate_kernels(E):
    """gptoss_moe_route (one launch after the logits at decode sizes) gives
    the same logits, top-k, weights, permutation and tile plan as
    gptoss_moe_router + gptoss_moe_permute, at sizes on both sides of its
    256-pair limit, with ties in the logits (a coarse router weight)."""
    import importlib
    L = importlib.import_module("gpt-oss-tvm_b200._lib")
    rng = np.random.default_rng(90 + E)
    S = synth()
    H, K = 2880, 4
    Wg = S.bf16_bits(np.round(rng.standard_normal((E, H)) * 4) / 256)  # few distinct values: ties
    bg = S.bf16_bits(rng.standard_normal(E).astype(np.float32) * 0.1)
    w = L.gptoss_moe_weights()
    w.num_experts = w.num_local_experts = E
    w.hidden, w.intermediate, w.top_k = H, H, K
    wd, bd = G.dev(Wg), G.dev(bg)
    w.gate_weight, w.gate_bias = wd.data_ptr(), bd.data_ptr()
    for M in (1, 5, 63, 64, 65, 256):
        t = G.dev(S.bf16_bits(rng.standard_normal((M, H)).astype(np.float32)))
        i32 = dict(dtype=torch.int32, device="cuda")
        outs = []
        for fused in (True, False):
            o = dict(logits=torch.empty(M, E, dtype=torch.bfloat16, device="cuda"),
                     w=torch.empty(M, K, dtype=torch.bfloat16, device="cuda"), idx=torch.empty(M, K, **i32),
                     indptr=torch.empty(E + 1, **i32), tok=torch.empty(M * K, **i32), rev=torch.empty(M * K, **i32),
                     exr=torch.empty(M * K, **i32), tp=torch.empty(E + 1, **i32), tr=torch.empty(E, **i32))
            err = torch.zeros(1, **i32)
            if fused:
                G.call("gptoss_moe_route", G.P(t), M, ctypes.byref(w), G.P(o["logits"]), G.P(o["w"]), G.P(o["idx"]),
                       G.P(o["indptr"]), G.P(o["tok"]), G.P(o["rev"]), G.P(o["exr"]), G.P(o["tp"]), G.P(o["tr"]),
                       G.P(err), G.S())
            else:
                G.call("gptoss_moe_router", G.P(t), G.P(wd), G.P(bd), M, E, H, K, G.P(o["logits"]), G.P(o["w"]),
                       G.P(o["idx"]), G.P(err), G.S())
                G.call("gptoss_moe_permute", G.P(o["idx"]), M, K, E, G.P(o["indptr"]), G.P(o["tok"]), G.P(o["rev"]),
                       G.P(o["exr"]), G.P(o["tp"]), G.P(o["tr"]), G.P(err), G.S())
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            outs.append(o)
        for k in outs[0]:
            assert torch.equal(outs[0][k], outs[1][k]), f"{k} differs at M={M} E={E}"


def _tile_plan(indptr, pairs, E):
    """The tile plan gptoss_moe_permute documents: at most 32 rows a tile when
    pairs <= 8 E, else 160; an expert's rows split evenly over its tiles,
    rounded up to 16."""
    c = np.diff(indptr.astype(np.int64))
    tmax = 32 if pairs <= 8 * E else 160
    nt = (c + tmax - 1) // tmax
    per = np.where(nt > 0, ((-(-c // np.maximum(nt, 1))) + 15) // 16 * 16, 0)
    return np.concatenate([[0], np.cumsum(nt)]).astype(np.int32), per.astype(np.int32)


@pytest.mark.parametrize("E", [8, 32, 128, 256, 300])
def test_permutation_matches_oracle_at_all_sizes(oracle, E):
    """gptoss_moe_permute against the oracle's stable sort of the pairs by
    expert, from no tokens to 20000 (80000 pairs), with uniform, skewed (one
    expert holding every pair) and sparse (few experts used) routings; E = 300
    takes the two-kernel path for more than 256 experts."""
    rng = np.random.default_rng(E)
    K = 4
    for M in (0, 1, 7, 33, 257, 1000, 8192, 20000):
        for kind in ("uniform", "one", "sparse"):
            if kind == "uniform":
                idx = rng.integers(0, E, (M, K))
            elif kind == "one":
                idx = np.full((M, K), E - 1)
            else:
                idx = rng.choice(np.array([0, E // 2, E - 1]), (M, K))
            idx = idx.astype(np.int32)
            i32 = dict(dtype=torch.int32, device="cuda")
            n = M * K
            d = dict(indptr=torch.full((E + 1,), -7, **i32), tok=torch.full((max(n, 1),), -7, **i32),
                     rev=torch.full((max(n, 1),), -7, **i32), exr=torch.full((max(n, 1),), -7, **i32),
                     tp=torch.full((E + 1,), -7, **i32), tr=torch.full((E,), -7, **i32))
            err = torch.zeros(1, **i32)
            idx_d = G.dev(idx) if n else torch.empty(1, **i32)
            G.call("gptoss_moe_permute", G.P(idx_d), M, K, E, G.P(d["indptr"]), G.P(d["tok"]), G.P(d["rev"]),
                   G.P(d["exr"]), G.P(d["tp"]), G.P(d["tr"]), G.P(err), G.S())
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            h = {k: v.cpu().numpy() for k, v in d.items()}
            indptr, tok, rev, exr = oracle.moe_permute(idx.reshape(M, K), E)
            what = f"E={E} M={M} {kind}"
            np.testing.assert_array_equal(h["indptr"], indptr, err_msg=what)
            np.testing.assert_array_equal(h["tok"][:n], tok, err_msg=what)
            np.testing.assert_array_equal(h["rev"][:n], rev, err_msg=what)
            np.testing.assert_array_equal(h["exr"][:n], exr, err_msg=what)
            tp, tr = _tile_plan(indptr, n, E)
            np.testing.assert_array_equal(h["tp"], tp, err_msg=what)
            np.testing.assert_array_equal(h["tr"], tr, err_msg=what)


@pytest.mark.parametrize("E", [32, 300])
def test_permutation_flags_expert_indices_out_of_range(E):
    """An expert index outside [0, E) sets the routing error bit; the valid
    pairs are still placed."""
    i32 = dict(dtype=torch.int32, device="cuda")
    M, K = 50, 4
    idx = np.random.default_rng(3).integers(0, E, (M, K)).astype(np.int32)
    idx[7, 2] = E
    idx[40, 0] = -1
    n = M * K
    d = [torch.zeros(E + 1, **i32), torch.zeros(n, **i32), torch.zeros(n, **i32), torch.zeros(n, **i32),
         torch.zeros(E + 1, **i32), torch.zeros(E, **i32)]
    err = torch.zeros(1, **i32)
    G.call("gptoss_moe_permute", G.P(G.dev(idx)), M, K, E, *[G.P(x) for x in d], G.P(err), G.S())
    torch.cuda.synchronize()
    assert int(err.item()) & (1 << 3)
    assert int(d[0][E].item()) == n - 2
