"""Pin the CPU oracle to outputs of the reference itself (CPU-only tests).

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py,
which compiles the reference's model/mlp.py and model/attention.py with
TVM's C target and runs them on seeded inputs.  Every comparison here is
bit-exact, including the fp32 intermediates.
"""
import hashlib

import numpy as np
import pytest

from conftest import golden, synth


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _moe_case(f, pre):
    S = synth()
    E, M = int(f[pre + "E"]), int(f[pre + "M"])
    p = S.moe_params(E, seed=int(f[pre + "wseed"]))
    x = S.activations(M, seed=int(f[pre + "xseed"]))
    assert _sha(x) == str(f[pre + "x_sha"]), "synthetic activation generator drifted"
    assert _sha(*[p[k] for k in sorted(p)]) == str(f[pre + "w_sha"]), "synthetic weight generator drifted"
    return p, x


@pytest.mark.parametrize("M", [1, 5, 16])
def test_moe_block_e8_bit_exact(oracle, M):
    f = golden("moe_e8.npz")
    pre = f"m{M}_"
    p, x = _moe_case(f, pre)
    r = oracle.moe_forward(x, p, return_all=True)
    np.testing.assert_array_equal(r["t"], f[pre + "t"])
    np.testing.assert_array_equal(r["logits"], f[pre + "logits"])
    np.testing.assert_array_equal(r["indices"], f[pre + "indices"])
    np.testing.assert_array_equal(r["weights"], f[pre + "weights"])
    if pre + "h1" in f:
        np.testing.assert_array_equal(r["h1"].view(np.uint32), f[pre + "h1"].view(np.uint32))
        np.testing.assert_array_equal(r["y"].view(np.uint32), f[pre + "y"].view(np.uint32))
        np.testing.assert_array_equal(r["h2"].view(np.uint32), f[pre + "h2"].view(np.uint32))
    np.testing.assert_array_equal(r["gated"], f[pre + "gated"].reshape(M, -1))
    np.testing.assert_array_equal(r["out"], f[pre + "out"])


def test_moe_block_config0_decode_bit_exact(oracle):
    f = golden("moe_cfg0.npz")
    p, x = _moe_case(f, "m1_")
    r = oracle.moe_forward(x, p, return_all=True)
    for k in ("t", "logits", "indices", "weights"):
        np.testing.assert_array_equal(r[k], f["m1_" + k])
    np.testing.assert_array_equal(r["h1"].view(np.uint32), f["m1_h1"].view(np.uint32))
    np.testing.assert_array_equal(r["h2"].view(np.uint32), f["m1_h2"].view(np.uint32))
    np.testing.assert_array_equal(r["out"], f["m1_out"])


def test_moe_router_config0_prefill_bit_exact(oracle):
    f = golden("moe_cfg0.npz")
    S = synth()
    p = S.moe_params(32, seed=0)
    x = S.activations(128, seed=1)
    t = oracle.rms_norm(x, p["norm_weight"])
    assert _sha(t) == str(f["m128_t_sha"])
    g = oracle.router(t, p["gate_weight"], p["gate_bias"])
    np.testing.assert_array_equal(g, f["m128_logits"])
    w, idx, _ = oracle.topk_softmax(g, 4)
    np.testing.assert_array_equal(idx, f["m128_indices"])
    np.testing.assert_array_equal(w, f["m128_weights"])


def test_moe_block_config0_prefill_tokens_bit_exact(oracle):
    """Full MLPBlock.forward output for a sample of the 128 prefill tokens
    (tokens are independent, so a row sample checks the same arithmetic)."""
    f = golden("moe_cfg0.npz")
    p, x = _moe_case(f, "m128_")
    rows = np.array([0, 1, 17, 63, 64, 100, 127])
    mask = np.zeros(128, np.uint8)
    mask[rows] = 1
    out = oracle.moe_forward(x, p, rows_mask=mask)
    np.testing.assert_array_equal(out[rows], f["m128_out"][rows])


def test_router_e128_bit_exact(oracle):
    f = golden("router_e128.npz")
    S = synth()
    p = S.moe_params(128, seed=int(f["wseed"]))
    x = S.activations(512, seed=int(f["xseed"]))
    assert _sha(x) == str(f["x_sha"])
    t = oracle.rms_norm(x, p["norm_weight"])
    assert _sha(t) == str(f["t_sha"])
    g = oracle.router(t, p["gate_weight"], p["gate_bias"])
    np.testing.assert_array_equal(g, f["logits"])
    w, idx, _ = oracle.topk_softmax(g, 4)
    np.testing.assert_array_equal(idx, f["indices"])
    np.testing.assert_array_equal(w, f["weights"])


def test_topk_ties_bit_exact(oracle):
    f = golden("topk_ties.npz")
    w, idx, vals = oracle.topk_softmax(f["logits"], 4)
    np.testing.assert_array_equal(idx, f["indices"])
    np.testing.assert_array_equal(vals, f["values"])
    np.testing.assert_array_equal(w, f["weights"])


def test_mxfp4_decode_matches_reference(oracle):
    """The reference einsum with one-hot activations and zero bias returns
    the decoded weight itself; the oracle's decode must agree bit for bit."""
    f = golden("mxfp4_decode.npz")
    rng = np.random.default_rng(5)
    blocks = rng.integers(0, 256, size=(2, 5760, 90, 16), dtype=np.uint8)
    scales = rng.integers(100, 150, size=(2, 5760, 90), dtype=np.uint8)
    scales[0, :8, :] = np.arange(8 * 90).reshape(8, 90) % 256
    scales[0, :8, :][scales[0, :8, :] == 255] = 254
    assert _sha(blocks, scales) == str(f["blocks_sha"])
    S = synth()
    dec = S.bf16_to_f32(oracle.mxfp4_dequant(blocks[:, :64], scales[:, :64]))  # [2, 64, 2880]
    kpos = f["kpos"]
    ref = f["out_rows"]  # [64 tokens, 4 ranks (experts 0,1,0,1), 64 cols]
    for s in range(64):
        for r, e in enumerate((0, 1, 0, 1)):
            got = dec[e, :, kpos[s]]
            np.testing.assert_array_equal(got + np.float32(0.0), ref[s, r] + np.float32(0.0))
    np.testing.assert_array_equal(f["lut"], np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6],
                                                     np.float32))


def test_rope_yarn_bit_exact(oracle):
    f = golden("rope.npz")
    S = synth()
    rng = np.random.default_rng(int(f["seed"]))
    n = int(f["n"])
    q = S.normal_bf16(rng, (n, 64, 64), 1.0)
    k = S.normal_bf16(rng, (n, 8, 64), 1.0)
    assert _sha(q) == str(f["q_sha"]) and _sha(k) == str(f["k_sha"])
    np.testing.assert_array_equal(oracle.rope_yarn(q, f["pos"]), f["q_out"])
    np.testing.assert_array_equal(oracle.rope_yarn(k, f["pos"]), f["k_out"])


# ------------------------------------------------------------ attention ---
# tests/golden/attention.npz: outputs of TVM's own attention kernels (the
# paged KV cache's CPU kernels, with the reference's tvm_fix.patch applied)
# and of the reference's sink rescale, made by tests/golden/make_attn_golden.py.
def _attn_fixture():
    return golden("attention.npz")


@pytest.mark.parametrize("tag,window", [("full", 0), ("win", 128)])
def test_attention_prefill_bit_exact_vs_tvm(oracle, tag, window):
    f = _attn_fixture()
    S = synth()
    heads = f["heads_kept"]
    q, k, v, _ = S.attention_inputs(int(f["pf_seq"]), seed=int(f["pf_seed"]))
    assert _sha(q, k, v) == str(f["pf_sha"]), "attention input generator drifted"
    o, lse = oracle.attention(q, k, v, causal=True, window=window, sm_scale=float(f["sm_scale"]))
    np.testing.assert_array_equal(o[:, heads], f[f"pf_{tag}_o"])
    np.testing.assert_array_equal(lse.view(np.uint32), f[f"pf_{tag}_lse"].view(np.uint32))
    q, k, v, _ = S.attention_inputs(int(f["tail_kv"]), seed=int(f["tail_seed"]))
    assert _sha(q, k, v) == str(f["tail_sha"])
    qo = int(f["tail_qo"])
    o, lse = oracle.attention(q[-qo:], k, v, causal=True, window=window, sm_scale=float(f["sm_scale"]))
    np.testing.assert_array_equal(o, f[f"tail_{tag}_o"])
    np.testing.assert_array_equal(lse.view(np.uint32), f[f"tail_{tag}_lse"].view(np.uint32))


@pytest.mark.parametrize("tag,window", [("full", 0), ("win", 128)])
def test_attention_decode_bit_exact_vs_tvm(oracle, tag, window):
    f = _attn_fixture()
    lens = tuple(int(x) for x in f["dec_lens"])
    q, ks, vs, _ = synth().decode_inputs(lens, seed=int(f["dec_seed"]))
    assert _sha(q, *ks, *vs) == str(f["dec_sha"])
    kc, vc, kl = oracle.decode_caches(ks, vs)
    o, lse = oracle.attention_decode(q, kc, vc, kl, window=window, sm_scale=float(f["sm_scale"]))
    np.testing.assert_array_equal(o, f[f"dec_{tag}_o"])
    np.testing.assert_array_equal(lse.view(np.uint32), f[f"dec_{tag}_lse"].view(np.uint32))


def test_attention_merge_and_sink_bit_exact_vs_tvm(oracle):
    f = _attn_fixture()
    S = synth()
    o1, l1, o2, l2 = S.merge_inputs(int(f["merge_n"]), seed=int(f["merge_seed"]))
    assert _sha(o1, l1, o2, l2) == str(f["merge_sha"])
    o, lse = oracle.merge_states(o1, l1, o2, l2)
    np.testing.assert_array_equal(o, f["merge_o"])
    np.testing.assert_array_equal(lse.view(np.uint32), f["merge_lse"].view(np.uint32))
    so, slse, sinks = S.sink_inputs(int(f["sink_n"]), seed=int(f["sink_seed"]))
    assert _sha(so, slse, sinks) == str(f["sink_sha"])
    np.testing.assert_array_equal(oracle.sink_rescale(so, slse, sinks), f["sink_o"])
