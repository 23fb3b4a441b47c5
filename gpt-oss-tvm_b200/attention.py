"""AttentionBlock: gpt-oss attention with sinks and YaRN RoPE on B200.

Same construction and call signature as the reference
(``AttentionBlock(config, layer_idx=0, dtype=None).forward(x, kv_cache,
query_positions, forward_to)``, model/attention.py:70-256), the same parameter
names (``sinks``, ``norm.weight``, ``qkv.weight/bias``, ``out.weight/bias``)
and the same result ``(x + attn, kv_cache)``.

Kernels (libgptoss_b200.so): RMSNorm; the fused QKV split + YaRN RoPE + cache
append; FlashAttention-style prefill / extend with the sliding-window or full
causal mask and the sink rescale fused; split-KV decode.  The two dense
projections (qkv 5120 x 2880, out 2880 x 4096) are plain bf16 GEMMs through
torch (cuBLAS); they are outside the MoE/attention hot path.

The KV cache here is contiguous per sequence ([B, max_len, Hkv, D] per
layer) instead of the reference's paged cache (PagedKVCache); the attention
semantics (append before attention, window of the last W keys including the
current token) are the same (tvm_fix.patch:35-47, :194-281).
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib
from .config import GPTOssConfig


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class KVCache:
    """Per-layer contiguous KV cache for up to `max_batch` sequences."""

    def __init__(self, config: GPTOssConfig, max_batch: int, max_len: int, num_layers: int | None = None,
                 device="cuda"):
        self.config = config
        self.max_batch, self.max_len = max_batch, max_len
        L = num_layers if num_layers is not None else config.num_hidden_layers
        Hkv, D = config.num_key_value_heads, config.head_dim
        self.k = [torch.zeros(max_batch, max_len, Hkv, D, dtype=torch.bfloat16, device=device) for _ in range(L)]
        self.v = [torch.zeros(max_batch, max_len, Hkv, D, dtype=torch.bfloat16, device=device) for _ in range(L)]
        self.lengths = torch.zeros(max_batch, dtype=torch.int32)  # host copy
        self.device = torch.device(device)
        self._cur = None

    def begin_forward(self, seq_ids, append_lengths):
        """Plan one forward pass (kv_state_begin_forward, engine.py:135-139):
        returns the query positions of the appended tokens."""
        pos, slots = [], []
        for s, n in zip(seq_ids, append_lengths):
            start = int(self.lengths[s])
            if start + n > self.max_len:
                raise ValueError("KV cache full")
            pos.extend(range(start, start + n))
            slots.extend(s * self.max_len + start + i for i in range(n))
            self.lengths[s] = start + n
        self._cur = (list(seq_ids), list(append_lengths))
        dev = self.device
        self.positions = torch.tensor(pos, dtype=torch.int32, device=dev)
        self.slots = torch.tensor(slots, dtype=torch.int32, device=dev)
        self.kv_len = torch.tensor([int(self.lengths[s]) for s in seq_ids], dtype=torch.int32, device=dev)
        return self.positions

    def popn(self, seq_id: int, n: int):
        self.lengths[seq_id] = max(0, int(self.lengths[seq_id]) - n)

    def clear(self):
        self.lengths.zero_()


class AttentionBlock:
    """Attention with sinks, sliding window on even layers, YaRN RoPE (model/attention.py:70-256)."""

    def __init__(self, config: GPTOssConfig, layer_idx: int = 0, dtype: str | None = None, device="cuda"):
        self.config = config
        self.dtype = dtype or config.dtype
        self.head_dim = config.head_dim
        self.num_attention_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.sliding_window = config.sliding_window_size if layer_idx % 2 == 0 else 0
        self.layer_idx = layer_idx
        self.sm_scale = 1.0 / (config.head_dim ** 0.5)
        dev = torch.device(device)
        self.device = dev
        H, D, Hq, Hkv = config.hidden_size, config.head_dim, config.num_attention_heads, config.num_key_value_heads
        qkv_dim = D * (Hq + 2 * Hkv)
        self.sinks = torch.zeros(Hq, dtype=torch.bfloat16, device=dev)
        self.norm_weight = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.qkv_weight = torch.zeros(qkv_dim, H, dtype=torch.bfloat16, device=dev)
        self.qkv_bias = torch.zeros(qkv_dim, dtype=torch.bfloat16, device=dev)
        self.out_weight = torch.zeros(H, D * Hq, dtype=torch.bfloat16, device=dev)
        self.out_bias = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        rs = config.rope_scaling
        inv = (ctypes.c_float * (D // 2))()
        conc = ctypes.c_float()
        _lib.call("gptoss_yarn_inv_freq", D, ctypes.c_float(float(rs.get("rope_theta", config.rope_theta))),
                  ctypes.c_float(float(rs["factor"])), ctypes.c_float(float(rs["beta_fast"])),
                  ctypes.c_float(float(rs["beta_slow"])), int(rs["original_max_position_embeddings"]), inv,
                  ctypes.byref(conc))
        self._inv_freq = inv
        self._conc = conc.value
        self._scratch = None

    PARAM_NAMES = {"sinks": "sinks", "norm.weight": "norm_weight", "qkv.weight": "qkv_weight",
                   "qkv.bias": "qkv_bias", "out.weight": "out_weight", "out.bias": "out_bias"}

    def load_state(self, params: dict) -> "AttentionBlock":
        import numpy as np
        for key, value in params.items():
            dst = getattr(self, self.PARAM_NAMES.get(key, key))
            if isinstance(value, np.ndarray):
                t = torch.from_numpy(np.ascontiguousarray(value).view(np.int16)).view(torch.bfloat16) \
                    if value.dtype == np.uint16 else torch.from_numpy(np.ascontiguousarray(value))
            else:
                t = value
            dst.copy_(t.to(dst.device))
        return self

    def _scratch_for(self, B, max_len):
        nbytes = int(_lib.load().gptoss_attn_decode_scratch_bytes(B, self.num_attention_heads, max_len,
                                                                   self.sliding_window))
        if self._scratch is None or self._scratch.numel() * 4 < nbytes:
            self._scratch = torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=self.device)
        return self._scratch, nbytes

    def forward(self, x: torch.Tensor, kv_cache: KVCache, query_positions: torch.Tensor | None, forward_to: str):
        """x [b, s, hidden] bf16.  prefill / extend: one sequence (b = 1, the
        reference's batch size); decode: one token per sequence of the batch."""
        H, D = self.config.hidden_size, self.head_dim
        Hq, Hkv = self.num_attention_heads, self.num_key_value_heads
        shape = x.shape
        x2 = x.reshape(-1, H).contiguous()
        T = x2.shape[0]
        S = _stream()
        t = torch.empty_like(x2)
        _lib.call("gptoss_rms_norm", _ptr(x2), _ptr(self.norm_weight), T, H, ctypes.c_float(1e-5), _ptr(t), S)
        qkv = F.linear(t, self.qkv_weight, self.qkv_bias)
        q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=x.device)
        kc, vc = kv_cache.k[self.layer_idx], kv_cache.v[self.layer_idx]
        pos = query_positions if query_positions is not None else kv_cache.positions
        _lib.call("gptoss_qkv_rope_append", _ptr(qkv), _ptr(pos), _ptr(kv_cache.slots), T, Hq, Hkv, D,
                  self._inv_freq, ctypes.c_float(self._conc), _ptr(q), _ptr(kc), _ptr(vc), S)
        o = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=x.device)
        seq_ids, lens = kv_cache._cur
        if forward_to in ("prefill", "extend"):
            if len(seq_ids) != 1:
                raise ValueError("prefill / extend take one sequence (batch size 1, as in the reference)")
            sid = seq_ids[0]
            Skv = int(kv_cache.lengths[sid])
            _lib.call("gptoss_attn_prefill", _ptr(q), _ptr(kc[sid]), _ptr(vc[sid]), _ptr(self.sinks), T, Skv, Hq, Hkv, D,
                      self.sliding_window, ctypes.c_float(self.sm_scale), _ptr(o), None, S)
        elif forward_to == "decode":
            if any(n != 1 for n in lens) or min(seq_ids) != 0 or list(seq_ids) != list(range(len(seq_ids))):
                raise ValueError("decode takes one token for each of sequences 0..B-1")
            B = len(seq_ids)
            scratch, nbytes = self._scratch_for(B, kv_cache.max_len)
            _lib.call("gptoss_attn_decode", _ptr(q), _ptr(kc), _ptr(vc), _ptr(kv_cache.kv_len), B, kv_cache.max_len,
                      Hq, Hkv, D, self.sliding_window, ctypes.c_float(self.sm_scale), _ptr(self.sinks), _ptr(scratch),
                      nbytes, _ptr(o), None, S)
        else:
            raise ValueError(f"forward_to {forward_to} not supported")
        out = F.linear(o.reshape(T, Hq * D), self.out_weight, self.out_bias)
        return (x2 + out).reshape(shape), kv_cache

    __call__ = forward
