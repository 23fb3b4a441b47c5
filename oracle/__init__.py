"""CPU oracle for the gpt-oss MoE block and sink/YaRN attention.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline legs of ``bench.py`` may import this package.  The product
path (``libgptoss_b200.so`` behind the ``gpt-oss-tvm_b200`` package) never
imports, links or calls it, and fails loudly when its CUDA library is absent.

``gptoss_oracle.c`` restates, step by step, the arithmetic that the
reference's TIR (model/mlp.py, model/attention.py) lowers to on a TVM CPU
target.  Parity is pinned by ``tests/golden/*.npz``: outputs of the reference
itself, compiled by TVM's C target (``tests/golden/make_golden.py``), which
``tests/test_oracle_golden.py`` compares with this oracle bit for bit.
The attention core (TVM/MLC paged-cache kernels, third-party and absent from
the reference tree) is pinned by ``tests/golden/attention.npz``, outputs of
TVM's own CPU kernels (``tests/golden/make_attn_golden.py``).  The sampler
(``sample_top_p_from_logits``: TVM's ``vm.builtin.sample_top_p_from_logits``,
src/runtime/vm/lm_support.cc, which the reference's Engine.sample calls) is
pinned by ``tests/golden/sampling.npz``, tokens returned by that function
(``tests/golden/make_sampling_golden.py``).  The MoE permutation
(mlc_llm.op.moe_misc, absent) is a restatement of the published algorithm,
pinned by the property tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgptoss_oracle.so")
SRC_PATH = os.path.join(_HERE, "gptoss_oracle.c")

# fp32 literals that the reference's YaRN constants become in generated code
# (model/attention.py:15-36, :148-153 with config.py:41-49 defaults).
YARN_THETA = 150000.0
YARN_FACTOR = 32.0
YARN_LOW = 8.092779
YARN_HIGH_MINUS_LOW = 9.305244
YARN_CONC = 1.346574


def build(force: bool = False) -> str:
    """Compile the C restatement (gcc, no FMA contraction, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC_PATH):
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
               SRC_PATH, "-o", LIB_PATH, "-lm"]
        subprocess.run(cmd, check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_I = ctypes.c_int64
_F = ctypes.c_float
_I32 = ctypes.c_int32


def _declare(L):
    L.orc_rms_norm.argtypes = [_P, _P, _I, _I, _F, _P]
    L.orc_router.argtypes = [_P, _P, _P, _I, _I, _I, _P]
    L.orc_topk_softmax.argtypes = [_P, _I, _I, _I, _P, _P, _P]
    L.orc_mxfp4_dequant.argtypes = [_P, _P, _I, _I, _P]
    L.orc_moe_einsum.argtypes = [_P, ctypes.c_int, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]
    L.orc_swiglu.argtypes = [_P, _I, _I, _F, _F, _P]
    L.orc_gating_residual.argtypes = [_P, _P, _P, _I, _I, _I, _P, _P]
    L.orc_moe_permute.argtypes = [_P, _I, _I, _I, _P, _P, _P, _P]
    L.orc_rope_yarn.argtypes = [_P, _P, _I, _I, _I, _F, _F, _F, _F, _F, _P]
    L.orc_attention.argtypes = [_P, _P, _P, _I, _I, _I, _I, _I, _I32, _I32, _F, _P, _P]
    L.orc_sink_rescale.argtypes = [_P, _P, _P, _I, _I, _I]
    L.orc_merge_states.argtypes = [_P, _P, _P, _P, _I, _I, _I, _P, _P]
    L.orc_attention_decode.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I32, _F, _P, _P]


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# bf16 tensors are carried as uint16 bit patterns throughout.
def bf16_bits_from_f32(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


def f32_from_bf16_bits(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rms_norm(x, w, eps=1e-5):
    x = _c(x, np.uint16)
    M, H = x.shape
    out = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(_c(w, np.uint16)), M, H, eps, _p(out))
    return out


def router(t, W, b):
    t = _c(t, np.uint16)
    W = _c(W, np.uint16)
    M, H = t.shape
    E = W.shape[0]
    out = np.empty((M, E), np.uint16)
    lib().orc_router(_p(t), _p(W), _p(_c(b, np.uint16)), M, E, H, _p(out))
    return out


def topk_softmax(logits, k=4):
    logits = _c(logits, np.uint16)
    M, E = logits.shape
    w = np.empty((M, k), np.uint16)
    idx = np.empty((M, k), np.int32)
    vals = np.empty((M, k), np.uint16)
    lib().orc_topk_softmax(_p(logits), M, E, k, _p(w), _p(idx), _p(vals))
    return w, idx, vals


def mxfp4_dequant(blocks, scales):
    blocks = _c(blocks, np.uint8)
    scales = _c(scales, np.uint8)
    G = blocks.shape[-2]
    rows = int(np.prod(blocks.shape[:-2]))
    out = np.empty(blocks.shape[:-2] + (G * 32,), np.uint16)
    lib().orc_mxfp4_dequant(_p(blocks), _p(scales), rows, G, _p(out))
    return out


def moe_einsum(x, idx, blocks, scales, bias, rows_mask=None):
    """x: bf16 bits [S, K] (mlp1) or float32 [S, R, K] (mlp2)."""
    idx = _c(idx, np.int32)
    S, R = idx.shape
    E, N, G, _ = blocks.shape
    K = G * 32
    is_f32 = x.dtype == np.float32
    x = _c(x, np.float32 if is_f32 else np.uint16)
    out = np.zeros((S, R, N), np.float32)
    mask = None if rows_mask is None else _c(rows_mask, np.uint8)
    lib().orc_moe_einsum(_p(x), int(is_f32), _p(idx), _p(_c(blocks, np.uint8)), _p(_c(scales, np.uint8)),
                         _p(_c(bias, np.uint16)), S, R, N, K, _p(mask), _p(out))
    return out


def swiglu(h, alpha=1.702, limit=7.0):
    h = _c(h, np.float32)
    lead = h.shape[:-1]
    D = h.shape[-1] // 2
    T = int(np.prod(lead))
    out = np.empty(lead + (D,), np.float32)
    lib().orc_swiglu(_p(h), T, D, alpha, limit, _p(out))
    return out


def gating_residual(y, w, x):
    y = _c(y, np.float32)
    S, R, H = y.shape
    gated = np.empty((S, H), np.uint16)
    out = np.empty((S, H), np.uint16)
    lib().orc_gating_residual(_p(y), _p(_c(w, np.uint16)), _p(_c(x, np.uint16)), S, R, H, _p(gated), _p(out))
    return gated, out


def moe_permute(idx, num_experts):
    idx = _c(idx, np.int32)
    S, R = idx.shape
    indptr = np.empty(num_experts + 1, np.int32)
    tok = np.empty(S * R, np.int32)
    rev = np.empty(S * R, np.int32)
    exp = np.empty(S * R, np.int32)
    lib().orc_moe_permute(_p(idx), S, R, num_experts, _p(indptr), _p(tok), _p(rev), _p(exp))
    return indptr, tok, rev, exp


def moe_forward(x, p, k=4, rows_mask=None, eps=1e-5, return_all=False):
    """Full MLPBlock.forward (model/mlp.py:371-402) on bf16-bit arrays.

    ``p`` holds the reference parameter names: norm_weight, gate_weight,
    gate_bias, mlp1_weight_blocks, mlp1_weight_scales, mlp1_bias,
    mlp2_weight_blocks, mlp2_weight_scales, mlp2_bias.  x: [M, 2880].
    """
    x = _c(x, np.uint16)
    t = rms_norm(x, p["norm_weight"], eps)
    g = router(t, p["gate_weight"], p["gate_bias"])
    w, idx, _ = topk_softmax(g, k)
    h1 = moe_einsum(t, idx, p["mlp1_weight_blocks"], p["mlp1_weight_scales"], p["mlp1_bias"], rows_mask)
    y = swiglu(h1)
    h2 = moe_einsum(y, idx, p["mlp2_weight_blocks"], p["mlp2_weight_scales"], p["mlp2_bias"], rows_mask)
    gated, out = gating_residual(h2, w, x)
    if return_all:
        return dict(t=t, logits=g, weights=w, indices=idx, h1=h1, y=y, h2=h2, gated=gated, out=out)
    return out


def rope_yarn(x, pos, theta=YARN_THETA, factor=YARN_FACTOR, low=YARN_LOW,
              high_minus_low=YARN_HIGH_MINUS_LOW, conc=YARN_CONC):
    x = _c(x, np.uint16)
    S, Hh, D = x.shape
    out = np.empty_like(x)
    lib().orc_rope_yarn(_p(x), _p(_c(pos, np.int32)), S, Hh, D, theta, factor, low, high_minus_low, conc, _p(out))
    return out


def attention(q, k, v, causal=True, window=0, sm_scale=0.125):
    q = _c(q, np.uint16)
    k = _c(k, np.uint16)
    v = _c(v, np.uint16)
    qo, Hq, D = q.shape
    kv, Hkv, _ = k.shape
    o = np.empty_like(q)
    lse = np.empty((qo, Hq), np.float32)
    lib().orc_attention(_p(q), _p(k), _p(v), qo, kv, Hq, Hkv, D, int(causal), int(window), sm_scale, _p(o), _p(lse))
    return o, lse


def sink_rescale(o, lse, sinks):
    o = np.array(o, dtype=np.uint16, copy=True, order="C")
    T, Hq, D = o.shape
    lib().orc_sink_rescale(_p(o), _p(_c(lse, np.float32)), _p(_c(sinks, np.uint16)), T, Hq, D)
    return o


def merge_states(o1, l1, o2, l2):
    o1 = _c(o1, np.uint16)
    T, Hq, D = o1.shape
    o = np.empty_like(o1)
    lse = np.empty((T, Hq), np.float32)
    lib().orc_merge_states(_p(o1), _p(_c(l1, np.float32)), _p(_c(o2, np.uint16)), _p(_c(l2, np.float32)),
                           T, Hq, D, _p(o), _p(lse))
    return o, lse


def attention_decode(q, k_cache, v_cache, kv_len, window=0, sm_scale=0.125):
    """One decode query per sequence (TVM's online-softmax decode kernel):
    q [B, Hq, D], caches [B, max_len, Hkv, D] bf16 bits, kv_len [B] int32."""
    q = _c(q, np.uint16)
    kc = _c(k_cache, np.uint16)
    vc = _c(v_cache, np.uint16)
    lens = _c(kv_len, np.int32)
    B, Hq, D = q.shape
    _, max_len, Hkv, _ = kc.shape
    o = np.empty_like(q)
    lse = np.empty((B, Hq), np.float32)
    lib().orc_attention_decode(_p(q), _p(kc), _p(vc), _p(lens), B, max_len, Hq, Hkv, D, int(window), sm_scale,
                               _p(o), _p(lse))
    return o, lse


def decode_caches(ks, vs):
    """Per-sequence keys / values [L_b, Hkv, D] -> contiguous caches
    [B, max(L_b), Hkv, D] (zero padded) and kv_len [B]."""
    B = len(ks)
    max_len = max(1, max(len(k) for k in ks))
    Hkv, D = ks[0].shape[1:]
    kc = np.zeros((B, max_len, Hkv, D), np.uint16)
    vc = np.zeros_like(kc)
    for b, (k, v) in enumerate(zip(ks, vs)):
        kc[b, :len(k)] = k
        vc[b, :len(v)] = v
    return kc, vc, np.array([len(k) for k in ks], np.int32)


def attention_block_core(q, k, v, sinks, causal=True, window=0, sm_scale=0.125):
    """self_attention + sink rescale (model/attention.py:218-247)."""
    o, lse = attention(q, k, v, causal, window, sm_scale)
    return sink_rescale(o, lse, sinks), lse


def sample_top_p_from_logits(logits, temperature, top_p, uniform):
    """Top-p sampling as TVM's SampleTopPFromLogits (src/runtime/vm/lm_support.cc,
    called by the reference's Engine.sample, engine.py:38-39, :172-174), step
    by step in float32: sort (logit, index) by descending logit; argmax when
    temperature < 1e-6; e = expf((l - max) * float(1 / temperature)) with the
    sum taken sequentially in that order; prob = e / sum; a sequential cumsum
    of prob, with top_p_sum = the probabilities added while the running sum was
    below top_p; the token is the first whose cumsum / top_p_sum exceeds the
    uniform draw (compared in double).  Ties among logits are ordered by index
    (std::sort leaves their order unspecified)."""
    z = np.ascontiguousarray(logits, np.float32).reshape(-1)
    order = np.argsort(-z, kind="stable")
    if temperature < 1e-6:
        return int(order[0])
    zs = z[order]
    scale = np.float32(1.0 / float(temperature))
    e = np.exp((zs - zs[0]) * scale, dtype=np.float32)
    total = np.cumsum(e, dtype=np.float32)[-1]
    prob = (e / total).astype(np.float32)
    cum = np.cumsum(prob, dtype=np.float32)
    before = np.concatenate([np.zeros(1, np.float32), cum[:-1]])
    k = int(np.count_nonzero(before.astype(np.float64) < float(top_p)))  # float running sum vs the double top_p
    top_p_sum = cum[k - 1] if k > 0 else np.float32(0.0)
    ratio = (cum / top_p_sum).astype(np.float32)
    hit = np.nonzero(float(uniform) < ratio.astype(np.float64))[0]
    return int(order[hit[0]]) if hit.size else int(order[0])
