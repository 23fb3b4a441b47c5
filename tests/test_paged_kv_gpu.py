"""The paged KV cache on the GPU (page size 16, the reference's PagedKVCache).

* gptoss_attn_decode_paged over pages in a shuffled order (full layers) and
  over a 9-page ring per sequence (sliding-window layers) gives the same bits
  as gptoss_attn_decode over the same keys in contiguous caches;
* gptoss_kv_pages_copy writes and reads back rows exactly;
* an AttentionBlock on the paged cache -- prefill, an extend whose window
  reaches back into the pages, decode steps that wrap the window ring -- is
  within the bf16 tolerance of the oracle on both layer kinds.
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

from test_attention_gpu import _block_reference  # noqa: E402

HQ, HKV, D = 64, 8, 64


def _pages_from_contiguous(kc, vc, lens, stride, ring, rng):
    """Pools + page table holding the contiguous caches kc/vc [B, L, Hkv, D]:
    shuffled physical pages (full) or a per-sequence ring of `stride` pages."""
    B = kc.shape[0]
    if ring:
        table = np.arange(B * stride, dtype=np.int32).reshape(B, stride)
    else:
        table = rng.permutation(B * stride).astype(np.int32).reshape(B, stride)
    kp = np.zeros((B * stride * 16, HKV, D), np.uint16)
    vp = np.zeros_like(kp)
    for b in range(B):
        L = int(lens[b])
        lo = max(0, L - (stride - 1) * 16 - (L % 16 or 16)) if ring else 0
        for j in range(lo, L):
            row = table[b, (j // 16) % stride] * 16 + j % 16
            kp[row] = kc[b, j]
            vp[row] = vc[b, j]
    return kp, vp, table


@pytest.mark.parametrize("window", [0, 128])
def test_decode_paged_equals_contiguous(window):
    S = synth()
    rng = np.random.default_rng(31 + window)
    B, L = 5, 1040                      # 65 pages
    lens = np.array([1, 16, 17, 700, 1040], np.int32)
    q = S.normal_bf16(rng, (B, HQ, D), 1.0)
    kc = S.normal_bf16(rng, (B, L, HKV, D), 1.0)
    vc = S.normal_bf16(rng, (B, L, HKV, D), 1.0)
    sinks = S.normal_bf16(rng, (HQ,), 1.0)
    ring = window > 0
    stride = 9 if ring else L // 16
    kp, vp, table = _pages_from_contiguous(kc, vc, lens, stride, ring, rng)
    lib = G._lib.load()
    qd, sd, ld = G.dev(q), G.dev(sinks), G.dev(lens)
    o1, o2 = torch.empty_like(qd), torch.empty_like(qd)
    l1 = torch.empty(B, HQ, dtype=torch.float32, device="cuda")
    l2 = torch.empty_like(l1)
    nb = lib.gptoss_attn_decode_scratch_bytes(B, HQ, L, window)
    sc = torch.empty(max(nb // 4, 1), dtype=torch.float32, device="cuda")
    # device tensors held in names: a temporary's memory could be reused by the next upload
    kcd, vcd, kpd, vpd, td = G.dev(kc), G.dev(vc), G.dev(kp), G.dev(vp), G.dev(table)
    G.call("gptoss_attn_decode", G.P(qd), G.P(kcd), G.P(vcd), G.P(ld), B, L, HQ, HKV, D, window,
           ctypes.c_float(0.125), G.P(sd), G.P(sc), nb, G.P(o1), G.P(l1), G.S())
    nb2 = lib.gptoss_attn_decode_scratch_bytes(B, HQ, stride * 16, window)
    sc2 = torch.empty(max(nb2 // 4, 1), dtype=torch.float32, device="cuda")
    G.call("gptoss_attn_decode_paged", G.P(qd), G.P(kpd), G.P(vpd), G.P(td), stride, G.P(ld),
           B, HQ, HKV, D, window, ctypes.c_float(0.125), G.P(sd), G.P(sc2), nb2, G.P(o2), G.P(l2), G.S())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_kv_pages_copy_round_trip():
    S = synth()
    rng = np.random.default_rng(5)
    stride, n = 12, 150
    table = rng.permutation(2 * stride).astype(np.int32).reshape(2, stride)
    kp = torch.zeros(2 * stride * 16, HKV, D, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    kr, vr = G.dev(S.normal_bf16(rng, (n, HKV, D), 1.0)), G.dev(S.normal_bf16(rng, (n, HKV, D), 1.0))
    td = G.dev(table)
    G.call("gptoss_kv_pages_copy", G.P(kp), G.P(vp), HKV, D, G.P(td), stride, 1, 7, n, G.P(kr), G.P(vr), 1, G.S())
    k2, v2 = torch.empty_like(kr), torch.empty_like(vr)
    G.call("gptoss_kv_pages_copy", G.P(kp), G.P(vp), HKV, D, G.P(td), stride, 1, 7, n, G.P(k2), G.P(v2), 0, G.S())
    torch.cuda.synchronize()
    assert torch.equal(kr, k2) and torch.equal(vr, v2)
    rows = torch.from_numpy((table[1][(np.arange(7, 7 + n) // 16) % stride] * 16 + np.arange(7, 7 + n) % 16))
    assert torch.equal(kp[rows.long().cuda()], kr)


@pytest.mark.parametrize("layer_idx", [0, 1], ids=["sliding", "full"])
def test_attention_block_paged_prefill_extend_decode(oracle, layer_idx):
    """300-token prefill, a 60-token extend (its window reaches back into the
    pages), then 40 decode steps that wrap the 9-page window ring."""
    att = importlib.import_module("gpt-oss-tvm_b200.attention")
    cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
    cfg = cfgm.gpt_oss_20b()
    rng = np.random.default_rng(50 + layer_idx)
    S = synth()
    p = {"sinks": S.normal_bf16(rng, (HQ,), 1.0), "norm.weight": S.normal_bf16(rng, (2880,), 1.0),
         "qkv.weight": S.normal_bf16(rng, (5120, 2880), 0.02), "qkv.bias": S.normal_bf16(rng, (5120,), 0.02),
         "out.weight": S.normal_bf16(rng, (2880, 4096), 0.02), "out.bias": S.normal_bf16(rng, (2880,), 0.02)}
    blk = att.AttentionBlock(cfg, layer_idx).load_state(p)
    cache = att.KVCache(cfg, max_batch=1, max_len=512, num_layers=2)
    assert cache.windowed[layer_idx] == (layer_idx == 0)
    k_all = v_all = None
    pos = 0
    for mode, T in (("prefill", 300), ("extend", 60)) + tuple(("decode", 1) for _ in range(40)):
        x = S.normal_bf16(rng, (T, 2880), 1.0)
        cache.begin_forward([0], [T])
        y, _ = blk.forward(G.dev(x).reshape(1, T, 2880), cache, None, mode)
        torch.cuda.synchronize()
        ref, k_all, v_all = _block_reference(oracle, p, x, k_all, v_all, pos, blk.sliding_window)
        G.tol_check(G.f32(G.host(y).reshape(T, 2880)) - G.f32(x), G.f32(ref) - G.f32(x),
                    what=f"{mode} at position {pos} (layer {layer_idx})")
        pos += T
    # what the pages hold equals the keys the oracle rotated, over the kept span
    lo = max(0, pos - 128) if layer_idx == 0 else 0
    kk, vv = cache.read_rows(layer_idx, 0, lo, pos - lo)
    # both come out of the bf16 qkv projection, whose rounding differs from the oracle's sum order
    G.tol_check(G.f32(G.host(kk)), G.f32(k_all[lo:pos]), max_rel=1e-2, what="cached keys")
    G.tol_check(G.f32(G.host(vv)), G.f32(v_all[lo:pos]), max_rel=1e-2, what="cached values")
    if layer_idx == 0:
        assert cache.k[0].shape[0] == 9 * 16  # the window layer holds 144 rows for a 512-token sequence
