"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no checkpoint or dataset is involved).

MoE block (gpt-oss-20b: 32 experts; gpt-oss-120b: 128 experts), top-4,
hidden = intermediate = 2880, MXFP4 weights stored exactly as the reference
parameters (model/mlp.py:100-143):
  norm_weight         [H]            bf16  = 1
  gate_weight         [E, H]         bf16  ~ N(0, 0.02)
  gate_bias           [E]            bf16  ~ N(0, 0.02)
  mlp1_weight_blocks  [E, 2I, 90, 16] u8   bytes uniform (each nibble uniform over 16 E2M1 codes)
  mlp1_weight_scales  [E, 2I, 90]    u8   uniform in 118..124 (E8M0)
  mlp1_bias           [E, 2I]        bf16  ~ N(0, 0.02)
  mlp2_weight_blocks  [E, H, 90, 16] u8   as mlp1
  mlp2_weight_scales  [E, H, 90]     u8   as mlp1
  mlp2_bias           [E, H]         bf16  ~ N(0, 0.02)
Activations are bf16 ~ N(0, 1).  bf16 values are produced from float32
normals by round-to-nearest-even and carried as uint16 bit patterns.
Generator: numpy PCG64 (seed 0 = weights, seed 1 = activations by default).
"""
from __future__ import annotations

import numpy as np

HIDDEN = 2880
INTERMEDIATE = 2880
GROUPS = 90


def bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) & 0xFFFFFFFF
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_bf16(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    return bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def moe_params(num_experts: int, seed: int = 0, hidden: int = HIDDEN, intermediate: int = INTERMEDIATE,
               scale_lo: int = 118, scale_hi: int = 124) -> dict:
    rng = np.random.default_rng(seed)
    E, H, N1 = num_experts, hidden, 2 * intermediate
    p = {}
    p["norm_weight"] = bf16_bits(np.ones(H, np.float32))
    p["gate_weight"] = normal_bf16(rng, (E, H), 0.02)
    p["gate_bias"] = normal_bf16(rng, (E,), 0.02)
    p["mlp1_weight_blocks"] = rng.integers(0, 256, size=(E, N1, GROUPS, 16), dtype=np.uint8)
    p["mlp1_weight_scales"] = rng.integers(scale_lo, scale_hi + 1, size=(E, N1, GROUPS), dtype=np.uint8)
    p["mlp1_bias"] = normal_bf16(rng, (E, N1), 0.02)
    p["mlp2_weight_blocks"] = rng.integers(0, 256, size=(E, H, GROUPS, 16), dtype=np.uint8)
    p["mlp2_weight_scales"] = rng.integers(scale_lo, scale_hi + 1, size=(E, H, GROUPS), dtype=np.uint8)
    p["mlp2_bias"] = normal_bf16(rng, (E, H), 0.02)
    return p


def activations(num_tokens: int, seed: int = 1, hidden: int = HIDDEN) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return normal_bf16(rng, (num_tokens, hidden), 1.0)


def attention_inputs(seq: int, n_q: int = 64, n_kv: int = 8, head_dim: int = 64, seed: int = 2):
    """q [seq, n_q, d], k/v [seq, n_kv, d] bf16 ~ N(0,1); sinks [n_q] ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    q = normal_bf16(rng, (seq, n_q, head_dim), 1.0)
    k = normal_bf16(rng, (seq, n_kv, head_dim), 1.0)
    v = normal_bf16(rng, (seq, n_kv, head_dim), 1.0)
    sinks = normal_bf16(rng, (n_q,), 1.0)
    return q, k, v, sinks


def decode_inputs(lens, n_q: int = 64, n_kv: int = 8, head_dim: int = 64, seed: int = 3):
    """One decode query per sequence: q [B, n_q, d] and, per sequence b, its
    cached keys / values [lens[b], n_kv, d] (bf16 ~ N(0,1)); sinks [n_q]."""
    rng = np.random.default_rng(seed)
    q = normal_bf16(rng, (len(lens), n_q, head_dim), 1.0)
    ks = [normal_bf16(rng, (int(L), n_kv, head_dim), 1.0) for L in lens]
    vs = [normal_bf16(rng, (int(L), n_kv, head_dim), 1.0) for L in lens]
    sinks = normal_bf16(rng, (n_q,), 1.0)
    return q, ks, vs, sinks


def merge_inputs(n: int, n_q: int = 64, head_dim: int = 64, seed: int = 4):
    """Two partial attention states over disjoint keys: o1, o2 [n, n_q, d]
    bf16 ~ N(0,1) and base-2 log-sum-exps lse1, lse2 [n, n_q] fp32; lse2 - lse1
    cycles through equal values, small and large gaps of either sign."""
    rng = np.random.default_rng(seed)
    o1 = normal_bf16(rng, (n, n_q, head_dim), 1.0)
    o2 = normal_bf16(rng, (n, n_q, head_dim), 1.0)
    l1 = rng.uniform(-8.0, 24.0, size=(n, n_q)).astype(np.float32)
    gaps = np.array([0.0, 0.5, -0.5, 3.0, -3.0, 20.0, -20.0, 1e-3], np.float32)
    l2 = (l1 + gaps[np.arange(n * n_q).reshape(n, n_q) % len(gaps)]
          + rng.uniform(-0.25, 0.25, size=(n, n_q)).astype(np.float32) * (np.arange(n)[:, None] % 2))
    return o1, l1, o2, l2.astype(np.float32)


def sink_inputs(n: int, n_q: int = 64, head_dim: int = 64, seed: int = 5):
    """Attention output o [n, n_q, d] bf16 ~ N(0,1), base-2 lse [n, n_q] fp32
    uniform in [-6, 26], sinks [n_q] bf16 ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    o = normal_bf16(rng, (n, n_q, head_dim), 1.0)
    lse = rng.uniform(-6.0, 26.0, size=(n, n_q)).astype(np.float32)
    sinks = normal_bf16(rng, (n_q,), 1.0)
    return o, lse, sinks
