"""GPU parity of the attention path (C ABI) against the CPU oracle.

RoPE is compared with the reference's own outputs (tests/golden/rope.npz);
attention, merge and sink rescale with the outputs of TVM's own attention
kernels run with the reference's patch and of the reference's sink code
(tests/golden/attention.npz), and at more sizes with the oracle (which
reproduces those outputs bit for bit), within the bf16 tolerance
(max|gpu - ref| / max|ref| <= 2e-2, cosine >= 0.9995); lse within 2e-3.
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

HQ, HKV, D = 64, 8, 64
SM_SCALE = 0.125


def yarn_table():
    lib = G._lib.load()
    inv = (ctypes.c_float * 32)()
    conc = ctypes.c_float()
    assert lib.gptoss_yarn_inv_freq(64, 150000.0, 32.0, 32.0, 1.0, 4096, inv, ctypes.byref(conc)) == 0
    return inv, conc.value


def test_yarn_table_matches_reference_formula():
    """inv_freq in fp32 with the reference's operation order (attention.py:39-61)."""
    inv, conc = yarn_table()
    f = np.arange(32, dtype=np.float32)
    e = (f * 2 % 64).astype(np.float32) / np.float32(64)
    fp = np.power(np.float32(150000.0), e, dtype=np.float32)
    import math
    low = max((64 * math.log(4096 / (32 * 2 * math.pi))) / (2 * math.log(150000)), 0)
    high = min((64 * math.log(4096 / (1 * 2 * math.pi))) / (2 * math.log(150000)), 63)
    v = np.minimum((f - np.float32(low)) / np.float32(high - low), np.float32(1))
    ramp = np.float32(1) - np.maximum(v, np.float32(0))
    ref = (np.float32(1) / (np.float32(32) * fp)) * (np.float32(1) - ramp) + (np.float32(1) / fp) * ramp
    np.testing.assert_allclose(np.array(inv[:]), ref, rtol=2e-7, atol=0)
    assert abs(conc - (0.1 * math.log(32) + 1)) < 1e-6


def test_rope_golden_reference():
    f = golden("rope.npz")
    S = synth()
    rng = np.random.default_rng(int(f["seed"]))
    n = int(f["n"])
    q = S.normal_bf16(rng, (n, 64, 64), 1.0)
    k = S.normal_bf16(rng, (n, 8, 64), 1.0)
    inv, conc = yarn_table()
    pos = G.dev(f["pos"].astype(np.int32))
    for x, ref in ((q, f["q_out"]), (k, f["k_out"])):
        xd = G.dev(x)
        out = torch.empty_like(xd)
        G.call("gptoss_rope_yarn", G.P(xd), G.P(pos), n, x.shape[1], 64, inv, ctypes.c_float(conc), G.P(out), G.S())
        torch.cuda.synchronize()
        got = G.host(out)
        # bit-exact except where CUDA's sin/cos and the reference's libm differ in
        # the last fp32 bit (then the bf16 result may differ by an ulp, or by
        # more ulps of a tiny value where x*cos - y*sin cancels)
        assert (got == ref).mean() > 0.99, (got == ref).mean()
        err = np.abs(G.f32(got) - G.f32(ref))
        assert err.max() <= 2.0 ** -7 * np.abs(G.f32(ref)).max(), err.max()
        G.tol_check(G.f32(got), G.f32(ref), what="rope vs reference")


def test_qkv_rope_append_matches_oracle(oracle):
    S_, rng = 37, np.random.default_rng(5)
    qkv = synth().normal_bf16(rng, (S_, (HQ + 2 * HKV) * D), 1.0)
    pos = (np.arange(S_) + 1000).astype(np.int32)
    slots = (np.arange(S_)[::-1] * 3 + 1).astype(np.int32)  # scattered cache rows
    inv, conc = yarn_table()
    qkvd, posd, slotd = G.dev(qkv), G.dev(pos), G.dev(slots)
    q_out = torch.empty(S_, HQ, D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(200, HKV, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros(200, HKV, D, dtype=torch.bfloat16, device="cuda")
    G.call("gptoss_qkv_rope_append", G.P(qkvd), G.P(posd), G.P(slotd), S_, HQ, HKV, D, inv, ctypes.c_float(conc),
           G.P(q_out), G.P(kc), G.P(vc), G.S())
    torch.cuda.synchronize()
    x = qkv.reshape(S_, HQ + 2 * HKV, D)
    q_ref = oracle.rope_yarn(np.ascontiguousarray(x[:, :HQ]), pos)
    k_ref = oracle.rope_yarn(np.ascontiguousarray(x[:, HQ:HQ + HKV]), pos)
    G.tol_check(G.f32(G.host(q_out)), G.f32(q_ref), max_rel=1e-2, what="q rope")
    G.tol_check(G.f32(G.host(kc)[slots]), G.f32(k_ref), max_rel=1e-2, what="k rope into cache")
    np.testing.assert_array_equal(G.host(vc)[slots], x[:, HQ + HKV:])


def _ref_attention(oracle, q, k, v, sinks, window, rows=None):
    """Oracle attention + sink for the query rows `rows` of q (queries are the
    last len(q) of the keys)."""
    Sq, Skv = q.shape[0], k.shape[0]
    if rows is None:
        o, lse = oracle.attention(q, k, v, causal=True, window=window, sm_scale=SM_SCALE)
        return oracle.sink_rescale(o, lse, sinks), lse
    outs, lses = [], []
    for i in rows:
        p = Skv - Sq + i
        o, lse = oracle.attention(q[i:i + 1], k[:p + 1], v[:p + 1], causal=True, window=window, sm_scale=SM_SCALE)
        outs.append(oracle.sink_rescale(o, lse, sinks))
        lses.append(lse)
    return np.concatenate(outs), np.concatenate(lses)


def _run_prefill(q, k, v, sinks, window, with_sinks=True):
    Sq, Skv = q.shape[0], k.shape[0]
    qd, kd, vd, sd = G.dev(q), G.dev(k), G.dev(v), G.dev(sinks)
    o = torch.empty(Sq, HQ, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(Sq, HQ, dtype=torch.float32, device="cuda")
    G.call("gptoss_attn_prefill", G.P(qd), G.P(kd), G.P(vd), G.P(sd) if with_sinks else None, Sq, Skv, HQ, HKV, D,
           window, ctypes.c_float(SM_SCALE), G.P(o), G.P(lse), G.S())
    torch.cuda.synchronize()
    return G.host(o), G.host(lse)


# window 0 and 700: the tcgen05 kernel; 128: the short-window mma.sync kernel
@pytest.mark.parametrize("window", [0, 128, 700])
@pytest.mark.parametrize("Sq,Skv", [(300, 300), (1, 77), (72, 200), (130, 130), (600, 900)])
def test_prefill_matches_oracle(oracle, Sq, Skv, window):
    q, k, v, sinks = synth().attention_inputs(Skv, seed=10 + Sq + window)
    q = np.ascontiguousarray(q[Skv - Sq:])
    o, lse = _run_prefill(q, k, v, sinks, window)
    o_ref, lse_ref = _ref_attention(oracle, q, k, v, sinks, window)
    G.tol_check(G.f32(o), G.f32(o_ref), what=f"prefill o (Sq={Sq}, Skv={Skv}, W={window})")
    np.testing.assert_allclose(lse, lse_ref, atol=2e-3, rtol=0)


def test_prefill_without_sinks_is_plain_attention(oracle):
    q, k, v, sinks = synth().attention_inputs(150, seed=3)
    o, lse = _run_prefill(q, k, v, sinks, 0, with_sinks=False)
    o_ref, lse_ref = oracle.attention(q, k, v, causal=True, window=0, sm_scale=SM_SCALE)
    G.tol_check(G.f32(o), G.f32(o_ref), what="prefill without sinks")


@pytest.mark.parametrize("window", [0, 128, 700])
def test_prefill_config1_seq4096_sampled_rows(oracle, window):
    """Config 1 prefill (seq 4096, 64 q / 8 kv heads): every row computed on the
    GPU, a sample of rows checked against the oracle."""
    q, k, v, sinks = synth().attention_inputs(4096, seed=1)
    o, lse = _run_prefill(q, k, v, sinks, window)
    rows = np.array([0, 1, 63, 64, 127, 128, 129, 1000, 2047, 4095])
    o_ref, lse_ref = _ref_attention(oracle, q, k, v, sinks, window, rows=rows)
    G.tol_check(G.f32(o[rows]), G.f32(o_ref), what=f"config1 prefill W={window}")
    np.testing.assert_allclose(lse[rows], lse_ref, atol=2e-3, rtol=0)


def _run_decode(q, kc, vc, kv_len, sinks, window, max_len):
    B = q.shape[0]
    lib = G._lib.load()
    nbytes = lib.gptoss_attn_decode_scratch_bytes(B, HQ, max_len, window)
    scratch = torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device="cuda")
    qd, kd, vd, ld, sd = G.dev(q), G.dev(kc), G.dev(vc), G.dev(kv_len), G.dev(sinks)
    o = torch.empty(B, HQ, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, HQ, dtype=torch.float32, device="cuda")
    G.call("gptoss_attn_decode", G.P(qd), G.P(kd), G.P(vd), G.P(ld), B, max_len, HQ, HKV, D, window,
           ctypes.c_float(SM_SCALE), G.P(sd), G.P(scratch), nbytes, G.P(o), G.P(lse), G.S())
    torch.cuda.synchronize()
    return G.host(o), G.host(lse)


@pytest.mark.parametrize("window", [0, 128])
def test_decode_ragged_lengths(oracle, window):
    rng = np.random.default_rng(7 + window)
    max_len = 1500
    lens = np.array([1, 2, 100, 128, 129, 1029, 1500], np.int32)
    B = len(lens)
    S = synth()
    q = S.normal_bf16(rng, (B, HQ, D), 1.0)
    kc = S.normal_bf16(rng, (B, max_len, HKV, D), 1.0)
    vc = S.normal_bf16(rng, (B, max_len, HKV, D), 1.0)
    sinks = S.normal_bf16(rng, (HQ,), 1.0)
    o, lse = _run_decode(q, kc, vc, lens, sinks, window, max_len)
    od, ld = oracle.attention_decode(q, kc, vc, lens, window=window, sm_scale=SM_SCALE)
    od = oracle.sink_rescale(od, ld, sinks)
    for b, L in enumerate(lens):
        G.tol_check(G.f32(o[b]), G.f32(od[b]), what=f"decode b={b} L={L} W={window}")
        np.testing.assert_allclose(lse[b], ld[b], atol=2e-3, rtol=0)


def test_decode_config1_batch32_kv8192(oracle):
    """Config 1 decode: batch 32 over KV length 8192 (full layer)."""
    rng = np.random.default_rng(1)
    B, L = 32, 8192
    S = synth()
    q = S.normal_bf16(rng, (B, HQ, D), 1.0)
    kc = S.normal_bf16(rng, (B, L, HKV, D), 1.0)
    vc = S.normal_bf16(rng, (B, L, HKV, D), 1.0)
    sinks = S.normal_bf16(rng, (HQ,), 1.0)
    lens = np.full(B, L, np.int32)
    o, lse = _run_decode(q, kc, vc, lens, sinks, 0, L)
    for b in (0, 13, 31):
        ob, lb = oracle.attention_decode(q[b:b + 1], kc[b:b + 1], vc[b:b + 1], lens[b:b + 1], window=0,
                                         sm_scale=SM_SCALE)
        ob = oracle.sink_rescale(ob, lb, sinks)
        G.tol_check(G.f32(o[b]), G.f32(ob[0]), what=f"config1 decode b={b}")
        np.testing.assert_allclose(lse[b], lb[0], atol=2e-3, rtol=0)


def test_merge_and_sink_match_oracle(oracle):
    """extend mode: attention over two disjoint key sets merged
    (merge_attn_output_inplace), then the sink rescale."""
    rng = np.random.default_rng(9)
    S = synth()
    T = 40
    q = S.normal_bf16(rng, (T, HQ, D), 1.0)
    k = S.normal_bf16(rng, (200, HKV, D), 1.0)
    v = S.normal_bf16(rng, (200, HKV, D), 1.0)
    sinks = S.normal_bf16(rng, (HQ,), 1.0)
    o1, l1 = oracle.attention(q, k[:120], v[:120], causal=False, window=0, sm_scale=SM_SCALE)
    o2, l2 = oracle.attention(q, k[120:], v[120:], causal=False, window=0, sm_scale=SM_SCALE)
    o_full, l_full = oracle.attention(q, k, v, causal=False, window=0, sm_scale=SM_SCALE)
    o1d, l1d, o2d, l2d = G.dev(o1), G.dev(l1), G.dev(o2), G.dev(l2)
    o = torch.empty_like(o1d)
    lse = torch.empty_like(l1d)
    G.call("gptoss_attn_merge", G.P(o1d), G.P(l1d), G.P(o2d), G.P(l2d), T, HQ, D, G.P(o), G.P(lse), G.S())
    sd = G.dev(sinks)
    G.call("gptoss_attn_sink_rescale", G.P(o), G.P(lse), G.P(sd), T, HQ, D, G.S())
    torch.cuda.synchronize()
    np.testing.assert_allclose(G.host(lse), l_full, atol=2e-3, rtol=0)
    G.tol_check(G.f32(G.host(o)), G.f32(oracle.sink_rescale(o_full, l_full, sinks)), what="merge + sink")
    om, lm = oracle.merge_states(o1, l1, o2, l2)
    np.testing.assert_allclose(G.host(lse), lm, atol=1e-4, rtol=0)


# ------------------------------------------- against TVM's own kernels ---
def _tvm_fixture():
    return golden("attention.npz")


@pytest.mark.parametrize("tag,window", [("full", 0), ("win", 128)])
def test_prefill_matches_tvm_kernels(tag, window):
    """gptoss_attn_prefill (no sinks: the plain self_attention output) against
    TVM's ragged CPU prefill kernel with the reference's sliding-window fix:
    192 queries over themselves, and the last 4 queries of a 4096-key prompt."""
    f = _tvm_fixture()
    S = synth()
    heads = f["heads_kept"]
    q, k, v, sinks = S.attention_inputs(int(f["pf_seq"]), seed=int(f["pf_seed"]))
    o, lse = _run_prefill(q, k, v, sinks, window, with_sinks=False)
    G.tol_check(G.f32(o[:, heads]), G.f32(f[f"pf_{tag}_o"]), what=f"prefill vs TVM ({tag})")
    np.testing.assert_allclose(lse, f[f"pf_{tag}_lse"], atol=2e-3, rtol=0)
    q, k, v, sinks = S.attention_inputs(int(f["tail_kv"]), seed=int(f["tail_seed"]))
    qo = int(f["tail_qo"])
    o, lse = _run_prefill(np.ascontiguousarray(q[-qo:]), k, v, sinks, window, with_sinks=False)
    G.tol_check(G.f32(o), G.f32(f[f"tail_{tag}_o"]), what=f"prefill tail vs TVM ({tag})")
    np.testing.assert_allclose(lse, f[f"tail_{tag}_lse"], atol=2e-3, rtol=0)


@pytest.mark.parametrize("tag,window", [("full", 0), ("win", 128)])
def test_decode_matches_tvm_kernels(oracle, tag, window):
    """gptoss_attn_decode (no sinks) against TVM's paged CPU decode kernel
    (page size 16; the sliding-window variant reads the last 128 keys), on
    sequences of 1, 17, 300 and 8192 cached keys."""
    f = _tvm_fixture()
    lens = tuple(int(x) for x in f["dec_lens"])
    q, ks, vs, sinks = synth().decode_inputs(lens, seed=int(f["dec_seed"]))
    kc, vc, kl = oracle.decode_caches(ks, vs)
    B, max_len = len(lens), kc.shape[1]
    lib = G._lib.load()
    nbytes = lib.gptoss_attn_decode_scratch_bytes(B, HQ, max_len, window)
    scratch = torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device="cuda")
    qd, kd, vd, ld = G.dev(q), G.dev(kc), G.dev(vc), G.dev(kl)
    o = torch.empty(B, HQ, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, HQ, dtype=torch.float32, device="cuda")
    G.call("gptoss_attn_decode", G.P(qd), G.P(kd), G.P(vd), G.P(ld), B, max_len, HQ, HKV, D, window,
           ctypes.c_float(SM_SCALE), None, G.P(scratch), nbytes, G.P(o), G.P(lse), G.S())
    torch.cuda.synchronize()
    for b in range(B):
        G.tol_check(G.f32(G.host(o)[b]), G.f32(f[f"dec_{tag}_o"][b]), what=f"decode vs TVM b={b} ({tag})")
    np.testing.assert_allclose(G.host(lse), f[f"dec_{tag}_lse"], atol=2e-3, rtol=0)


def test_merge_and_sink_rescale_match_tvm():
    """gptoss_attn_merge against TVM's merge_state_inplace CPU kernel, and
    gptoss_attn_sink_rescale against the reference's sink code
    (model/attention.py:240-247) compiled by TVM."""
    f = _tvm_fixture()
    S = synth()
    o1, l1, o2, l2 = S.merge_inputs(int(f["merge_n"]), seed=int(f["merge_seed"]))
    T = o1.shape[0]
    o1d, l1d, o2d, l2d = G.dev(o1), G.dev(l1), G.dev(o2), G.dev(l2)
    o = torch.empty_like(o1d)
    lse = torch.empty_like(l1d)
    G.call("gptoss_attn_merge", G.P(o1d), G.P(l1d), G.P(o2d), G.P(l2d), T, HQ, D, G.P(o), G.P(lse), G.S())
    torch.cuda.synchronize()
    G.tol_check(G.f32(G.host(o)), G.f32(f["merge_o"]), what="merge vs TVM")
    np.testing.assert_allclose(G.host(lse), f["merge_lse"], atol=1e-4, rtol=0)
    so, slse, sinks = S.sink_inputs(int(f["sink_n"]), seed=int(f["sink_seed"]))
    od, ld, sd = G.dev(so), G.dev(slse), G.dev(sinks)
    G.call("gptoss_attn_sink_rescale", G.P(od), G.P(ld), G.P(sd), so.shape[0], HQ, D, G.S())
    torch.cuda.synchronize()
    got, ref = G.host(od), f["sink_o"]
    G.tol_check(G.f32(got), G.f32(ref), what="sink rescale vs reference")
    # the scale is one bf16 value per (token, head); it may land one bf16 ulp
    # apart where CUDA's expf and glibc's differ in the last fp32 bit
    assert (got == ref).mean() > 0.99


def _block_reference(oracle, p, x_bits, k_prev, v_prev, pos0, window):
    """AttentionBlock.forward (model/attention.py:182-256) composed from oracle
    pieces; the dense projections in fp32 (rounded to bf16, as the block's
    outputs are bf16).  Returns (out bits, k_all, v_all)."""
    S = synth()
    T = x_bits.shape[0]
    t = oracle.rms_norm(x_bits, p["norm.weight"])
    qkv = S.bf16_bits(G.f32(t) @ G.f32(p["qkv.weight"]).T + G.f32(p["qkv.bias"]))
    qkv = qkv.reshape(T, HQ + 2 * HKV, D)
    pos = np.arange(pos0, pos0 + T, dtype=np.int32)
    q = oracle.rope_yarn(np.ascontiguousarray(qkv[:, :HQ]), pos)
    k = oracle.rope_yarn(np.ascontiguousarray(qkv[:, HQ:HQ + HKV]), pos)
    v = np.ascontiguousarray(qkv[:, HQ + HKV:])
    k_all = np.concatenate([k_prev, k]) if k_prev is not None else k
    v_all = np.concatenate([v_prev, v]) if v_prev is not None else v
    o, lse = oracle.attention(q, k_all, v_all, causal=True, window=window, sm_scale=SM_SCALE)
    o = oracle.sink_rescale(o, lse, p["sinks"])
    out = S.bf16_bits(G.f32(o.reshape(T, HQ * D)) @ G.f32(p["out.weight"]).T + G.f32(p["out.bias"]))
    res = S.bf16_bits(G.f32(x_bits) + G.f32(out))
    return res, k_all, v_all


@pytest.mark.parametrize("layer_idx", [0, 1], ids=["sliding", "full"])
def test_attention_block_prefill_then_decode(oracle, layer_idx):
    import importlib
    att = importlib.import_module("gpt-oss-tvm_b200.attention")
    cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
    cfg = cfgm.gpt_oss_20b()
    rng = np.random.default_rng(20 + layer_idx)
    S = synth()
    p = {"sinks": S.normal_bf16(rng, (HQ,), 1.0), "norm.weight": S.normal_bf16(rng, (2880,), 1.0),
         "qkv.weight": S.normal_bf16(rng, (5120, 2880), 0.02), "qkv.bias": S.normal_bf16(rng, (5120,), 0.02),
         "out.weight": S.normal_bf16(rng, (2880, 4096), 0.02), "out.bias": S.normal_bf16(rng, (2880,), 0.02)}
    blk = att.AttentionBlock(cfg, layer_idx).load_state(p)
    cache = att.KVCache(cfg, max_batch=1, max_len=512, num_layers=2)
    T = 200
    x = S.normal_bf16(rng, (T, 2880), 1.0)
    cache.begin_forward([0], [T])
    y, _ = blk.forward(G.dev(x).reshape(1, T, 2880), cache, None, "prefill")
    torch.cuda.synchronize()
    ref, k_all, v_all = _block_reference(oracle, p, x, None, None, 0, blk.sliding_window)
    G.tol_check(G.f32(G.host(y).reshape(T, 2880)) - G.f32(x), G.f32(ref) - G.f32(x), what="block prefill attn part")
    # one decode step on top of the cache
    x1 = S.normal_bf16(rng, (1, 2880), 1.0)
    cache.begin_forward([0], [1])
    y1, _ = blk.forward(G.dev(x1).reshape(1, 1, 2880), cache, None, "decode")
    torch.cuda.synchronize()
    ref1, _, _ = _block_reference(oracle, p, x1, k_all, v_all, T, blk.sliding_window)
    G.tol_check(G.f32(G.host(y1).reshape(1, 2880)) - G.f32(x1), G.f32(ref1) - G.f32(x1), what="block decode attn part")


@pytest.mark.parametrize("T", [1, 2, 3, 4])
@pytest.mark.parametrize("NK", [(5120, 2880), (2880, 4096)], ids=["qkv", "out"])
def test_dense_gemv_matches_fp32_linear(T, NK):
    """gptoss_dense_gemv (the attention projections at decode sizes) against an
    fp32 torch nn.Linear rounded once to bf16: within the bf16 tolerance, and
    at most 2 bf16 ulps apart (only the fp32 summation order differs)."""
    N, K = NK
    g = torch.Generator(device="cuda")
    g.manual_seed(100 * T + N)
    x = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    for bias in (b, None):
        out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        G.call("gptoss_dense_gemv", G.P(x), T, G.P(w), G.P(bias), N, K, G.P(out), G.S())
        ref = x.float() @ w.float().T + (bias.float() if bias is not None else 0.0)
        torch.cuda.synchronize()
        G.tol_check(out.float().cpu().numpy(), ref.to(torch.bfloat16).float().cpu().numpy(),
                    what=f"dense gemv T={T} N={N} K={K}")
        ulp = (ref.abs().clamp_min(1e-30).log2().floor() - 7).exp2()
        assert torch.all((out.float() - ref).abs() <= 2 * ulp + 1e-6), "more than 2 bf16 ulps from fp32"


def test_dense_gemv_rejects_large_batches():
    lib = G._lib.load()
    T = lib.gptoss_dense_gemv_max_tokens() + 1
    x = torch.zeros(T, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(T, 8, dtype=torch.bfloat16, device="cuda")
    assert lib.gptoss_dense_gemv(G.P(x), T, G.P(w), None, 8, 64, G.P(out), G.S()) != 0
