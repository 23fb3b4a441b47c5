"""GPU parity of the full model (GPTOssForCausalLM / Engine) on a two-layer
gpt-oss-20b-shaped model with a small vocabulary.

* layer by layer, teacher-forced: each attention block's output is compared
  with the oracle composition of the block (RMSNorm, fp32 qkv projection,
  YaRN RoPE, sink attention over the GPU cache's earlier keys, fp32 out
  projection) on the same input, and each MoE block's output with the
  oracle MoE block on the same input, within the bf16 tolerance
  (max rel err <= 2e-2, cosine >= 0.9995);
* the final logits with the oracle RMSNorm and an fp32 unembedding of the
  same hidden states, within the same tolerance;
* GPTOssForCausalLM.prefill / decode equal that layer-by-layer chain bit
  for bit, and the CUDA-graph greedy decoder equals the eager decoder bit for
  bit (logits and tokens) on ragged batches.
"""
import numpy as np
import pytest

from conftest import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402

HQ, HKV, D, H = 64, 8, 64, 2880


def modules():
    import importlib
    return (importlib.import_module("gpt-oss-tvm_b200.model"), importlib.import_module("gpt-oss-tvm_b200.config"),
            importlib.import_module("gpt-oss-tvm_b200.engine"))


def tiny_config(cfgm, layers=2, vocab=1024):
    return cfgm.GPTOssConfig(num_hidden_layers=layers, num_experts=32, vocab_size=vocab, context_window_size=4096)


def attn_reference(oracle, attn, x_bits, k_prev, v_prev, pos0):
    S = synth()
    p = {n: G.host(getattr(attn, a)) for n, a in attn.PARAM_NAMES.items()}
    T = x_bits.shape[0]
    t = oracle.rms_norm(x_bits, p["norm.weight"])
    qkv = S.bf16_bits(G.f32(t) @ G.f32(p["qkv.weight"]).T + G.f32(p["qkv.bias"])).reshape(T, HQ + 2 * HKV, D)
    pos = np.arange(pos0, pos0 + T, dtype=np.int32)
    q = oracle.rope_yarn(np.ascontiguousarray(qkv[:, :HQ]), pos)
    k = oracle.rope_yarn(np.ascontiguousarray(qkv[:, HQ:HQ + HKV]), pos)
    v = np.ascontiguousarray(qkv[:, HQ + HKV:])
    k_all = np.concatenate([k_prev, k]) if pos0 else k
    v_all = np.concatenate([v_prev, v]) if pos0 else v
    o, lse = oracle.attention(q, k_all, v_all, causal=True, window=attn.sliding_window, sm_scale=0.125)
    o = oracle.sink_rescale(o, lse, p["sinks"])
    out = S.bf16_bits(G.f32(o.reshape(T, HQ * D)) @ G.f32(p["out.weight"]).T + G.f32(p["out.bias"]))
    return S.bf16_bits(G.f32(x_bits) + G.f32(out))


def moe_params(mlp):
    return {attr: G.host(getattr(mlp, attr)) for attr in mlp.PARAM_NAMES.values()}


def chain(oracle, model, cache, ids, seq, mode):
    """Layer-by-layer forward on the GPU, each block checked against the
    oracle on the GPU block's own input; returns the fp32 logits."""
    S = synth()
    x = model.embed(ids)
    T = x.shape[1] if mode != "decode" else 1
    pos0 = int(cache.lengths[seq])
    if mode == "decode":
        cache.begin_forward([0], [1])
        x = x.reshape(1, 1, H)
    else:
        cache.begin_forward([seq], [T])
    for i, blk in enumerate(model.model.block):
        x_in = G.host(x).reshape(T, H)
        lo = max(0, pos0 - cache.window) if cache.windowed[i] else 0  # a window layer keeps its window only
        kp, vp = cache.read_rows(i, seq, lo, pos0 - lo)
        k_prev, v_prev = G.host(kp), G.host(vp)
        x, _ = blk.attn(x, cache, cache.positions, mode)
        torch.cuda.synchronize()
        got = G.host(x).reshape(T, H)
        ref = attn_reference(oracle, blk.attn, x_in, k_prev, v_prev, pos0)
        G.tol_check(G.f32(got) - G.f32(x_in), G.f32(ref) - G.f32(x_in), what=f"layer {i} attention ({mode})")
        x = blk.mlp(x)
        torch.cuda.synchronize()
        got2 = G.host(x).reshape(T, H)
        ref2 = oracle.moe_forward(got, moe_params(blk.mlp))
        G.tol_check(G.f32(got2) - G.f32(got), G.f32(ref2) - G.f32(got), what=f"layer {i} MoE ({mode})")
    h = G.host(x).reshape(T, H)[-1:]
    hn = oracle.rms_norm(h, G.host(model.model.norm.weight))
    ref_logits = S.bf16_bits(G.f32(hn) @ G.f32(G.host(model.unembedding.weight)).T)
    x = model.model.norm(x).reshape(-1, H)[-1:]
    logits = model.unembedding(x).float()
    G.tol_check(G.host(logits), G.f32(ref_logits), what=f"logits ({mode})")
    return logits


def test_full_model_matches_oracle_layer_by_layer(oracle):
    modm, cfgm, _ = modules()
    cfg = tiny_config(cfgm)
    # E8M0 codes 115..121 keep every block's contribution of the same order
    # as the residual stream, so the per-block differences are not lost in
    # the bf16 rounding of the residual sum
    model = modm.random_init(modm.GPTOssForCausalLM(cfg), seed=5, scale_lo=115, scale_hi=121)
    rng = np.random.default_rng(3)
    ids = torch.from_numpy(rng.integers(0, cfg.vocab_size, 150).astype(np.int64)).cuda()
    c1 = model.create_paged_kv_cache(1, 512)
    c2 = model.create_paged_kv_cache(1, 512)
    ref_prefill = chain(oracle, model, c1, ids, 0, "prefill")
    c2.begin_forward([0], [ids.numel()])
    logits, _ = model.prefill(model.embed(ids), c2)
    assert torch.equal(logits.reshape(-1), ref_prefill.reshape(-1)), "prefill differs from the layer chain"
    tok = torch.argmax(logits.reshape(-1)).reshape(1)
    ref_dec = chain(oracle, model, c1, tok, 0, "decode")
    c2.begin_forward([0], [1])
    logits2, _ = model.decode(model.embed(tok), c2)
    assert torch.equal(logits2.reshape(-1), ref_dec.reshape(-1)), "decode differs from the layer chain"
    model.release()


@pytest.mark.parametrize("use_graph", [True, False], ids=["graph", "eager"])
def test_greedy_decode_graph_matches_eager_ragged(use_graph):
    modm, cfgm, engm = modules()
    cfg = tiny_config(cfgm)
    model = modm.random_init(modm.GPTOssForCausalLM(cfg), seed=7)
    rng = np.random.default_rng(11)
    B, steps = 3, 5
    lens = [37, 130, 9]  # ragged: windowed and full layers see different spans
    prompts = [torch.from_numpy(rng.integers(0, cfg.vocab_size, n).astype(np.int64)).cuda() for n in lens]
    caches = [model.create_paged_kv_cache(B, 256) for _ in range(2)]
    first = []
    for c in caches:
        for s, pr in enumerate(prompts):
            c.begin_forward([s], [pr.numel()])
            lg, _ = model.prefill(model.embed(pr), c)
            if c is caches[0]:
                first.append(int(torch.argmax(lg.reshape(-1))))
    tok = torch.tensor(first, dtype=torch.int64, device="cuda")
    # eager reference
    eager_tokens, eager_logits = [], []
    cur = tok.clone()
    for _ in range(steps):
        caches[0].begin_forward(list(range(B)), [1] * B)
        lg, _ = model.decode(model.embed(cur), caches[0])
        cur = torch.argmax(lg.reshape(B, -1), dim=-1)
        eager_tokens.append(cur.cpu())
        eager_logits.append(lg.clone())
    dec = engm.GreedyDecodeGraph(model, caches[1], B, use_graph=use_graph)
    dec.set_tokens(tok)
    for s in range(steps):
        lg, nxt = dec.step()
        assert torch.equal(lg, eager_logits[s]), f"step {s}: logits differ"
        assert torch.equal(nxt.cpu(), eager_tokens[s]), f"step {s}: tokens differ"
    assert caches[1].lengths.tolist() == [n + steps for n in lens]
    assert caches[1].dev_lengths.cpu().tolist() == [n + steps for n in lens]
    dec.close()
    model.release()


def test_engine_random_generate_and_reference_api():
    _, cfgm, engm = modules()
    cfg = tiny_config(cfgm)
    cfg.context_window_size = 1024
    eng = engm.Engine.random(cfg, seed=1, max_batch_size=2)
    sid = eng.begin_sequence()
    assert sid == 0
    prompt = np.arange(20, dtype=np.int32)
    logits = eng.prefill(prompt, sid)
    assert logits.shape == (1, 1, cfg.vocab_size) and logits.dtype == torch.float32
    assert eng.get_kv_total_seq_len() == 20
    t = eng.sample(logits)
    assert 0 <= t < cfg.vocab_size
    lg = eng.decode(np.array([t], np.int32), sid)
    assert lg.shape == (1, 1, cfg.vocab_size)
    eng.popn(sid, 1)
    assert eng.get_kv_total_seq_len() == 20
    # the same decode again after popn gives the same logits
    lg2 = eng.decode(np.array([t], np.int32), sid)
    assert torch.equal(lg, lg2)
    eng.clear_kv_cache()
    assert eng.get_kv_total_seq_len() == 0
    # greedy generation is deterministic
    a = eng.generate(prompt, 4)
    eng.clear_kv_cache()
    b = eng.generate(prompt, 4)
    assert a == b
    with pytest.raises(ValueError):
        engm.Engine(None, "cpu", config=cfg, seed=0)
    engm.Engine.next_seq_id = 0
    eng.model.release()
