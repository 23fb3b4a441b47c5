"""AttentionBlock: gpt-oss attention with sinks and YaRN RoPE on B200.

Same construction and call signature as the reference
(``AttentionBlock(config, layer_idx=0, dtype=None).forward(x, kv_cache,
query_positions, forward_to)``, model/attention.py:70-256), the same parameter
names (``sinks``, ``norm.weight``, ``qkv.weight/bias``, ``out.weight/bias``)
and the same result ``(x + attn, kv_cache)``.

Kernels (libgptoss_b200.so): RMSNorm; the fused QKV split + YaRN RoPE + cache
append; FlashAttention-style prefill / extend with the sliding-window or full
causal mask and the sink rescale fused; split-KV decode.  The two dense
projections (qkv 5120 x 2880, out 2880 x 4096) are bf16 GEMMs through torch
(cuBLAS); with ``DENSE_GEMV = True`` decode sizes (up to
gptoss_dense_gemv_max_tokens() tokens) use the library's bf16 GEMV instead
(measured on B200: the same step time as cuBLAS, so cuBLAS stays the default).

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
    """Per-layer contiguous KV cache for up to `max_batch` sequences.

    The host keeps the authoritative sequence lengths (``lengths``); the
    device keeps a mirror (``dev_lengths``) so that a decode step can plan
    itself on the device (``begin_decode_on_device``) inside a CUDA graph.
    The decode-step buffers (positions, slots, kv_len) are allocated once and
    never move, so a captured graph keeps reading the current values."""

    def __init__(self, config: GPTOssConfig, max_batch: int, max_len: int, num_layers: int | None = None,
                 device="cuda"):
        if max_batch < 1 or max_len < 1 or max_batch * max_len >= 2 ** 31:
            raise ValueError(f"KVCache: max_batch x max_len = {max_batch} x {max_len} must fit int32 slots")
        self.config = config
        self.max_batch, self.max_len = max_batch, max_len
        L = num_layers if num_layers is not None else config.num_hidden_layers
        Hkv, D = config.num_key_value_heads, config.head_dim
        self.k = [torch.zeros(max_batch, max_len, Hkv, D, dtype=torch.bfloat16, device=device) for _ in range(L)]
        self.v = [torch.zeros(max_batch, max_len, Hkv, D, dtype=torch.bfloat16, device=device) for _ in range(L)]
        self.lengths = torch.zeros(max_batch, dtype=torch.int32)  # host copy
        self.device = torch.device(device)
        dev = self.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.dev_lengths = torch.zeros(max_batch, **i32)
        self._seq_base = torch.arange(max_batch, **i32) * max_len
        self._dec_pos = torch.zeros(max_batch, **i32)
        self._dec_slot = torch.zeros(max_batch, **i32)
        self._kv_len = torch.zeros(max_batch, **i32)
        self._pos = torch.zeros(max_batch, **i32)
        self._slot = torch.zeros(max_batch, **i32)
        self._cur = None

    def _sync_dev_lengths(self):
        self.dev_lengths.copy_(self.lengths.to(self.device))

    def begin_forward(self, seq_ids, append_lengths):
        """Plan one forward pass (kv_state_begin_forward, engine.py:135-139):
        returns the query positions of the appended tokens."""
        pos, slots = [], []
        new_len = self.lengths.clone()
        for s, n in zip(seq_ids, append_lengths):
            if not 0 <= s < self.max_batch:
                raise ValueError(f"sequence id {s} outside the cache's {self.max_batch} sequences")
            start = int(new_len[s])
            if start + n > self.max_len:
                raise ValueError("KV cache full")
            p = torch.arange(start, start + n, dtype=torch.int32)
            pos.append(p)
            slots.append(p + s * self.max_len)
            new_len[s] = start + n
        self.lengths.copy_(new_len)
        self._cur = (list(seq_ids), list(append_lengths))
        pos = torch.cat(pos) if pos else torch.zeros(0, dtype=torch.int32)
        slots = torch.cat(slots) if slots else torch.zeros(0, dtype=torch.int32)
        T = pos.numel()
        if T > self._pos.numel():
            self._pos = torch.zeros(T, dtype=torch.int32, device=self.device)
            self._slot = torch.zeros(T, dtype=torch.int32, device=self.device)
        self._pos[:T].copy_(pos)
        self._slot[:T].copy_(slots)
        nb = len(seq_ids)
        self._kv_len[:nb].copy_(torch.tensor([int(self.lengths[s]) for s in seq_ids], dtype=torch.int32))
        self._sync_dev_lengths()
        self.positions, self.slots, self.kv_len = self._pos[:T], self._slot[:T], self._kv_len[:nb]
        return self.positions

    def check_decode(self, batch: int, steps: int = 1):
        if not 1 <= batch <= self.max_batch:
            raise ValueError(f"decode batch {batch} outside 1..{self.max_batch}")
        if int(self.lengths[:batch].max()) + steps > self.max_len:
            raise ValueError("KV cache full")

    def begin_decode_on_device(self, batch: int):
        """begin_forward(range(batch), [1] * batch) done by device ops only
        (capturable in a CUDA graph): position = current length, slot =
        sequence base + position, length += 1.  The host mirror is advanced
        by ``commit_decode`` after the step has been issued."""
        self._cur = (list(range(batch)), [1] * batch)
        pos, slot, kvl = self._dec_pos[:batch], self._dec_slot[:batch], self._kv_len[:batch]
        pos.copy_(self.dev_lengths[:batch])
        torch.add(self._seq_base[:batch], pos, out=slot)
        self.dev_lengths[:batch].add_(1)
        kvl.copy_(self.dev_lengths[:batch])
        self.positions, self.slots, self.kv_len = pos, slot, kvl
        return pos

    def commit_decode(self, batch: int, steps: int = 1):
        self.lengths[:batch] += steps

    def rollback_device(self):
        """Forget device-side steps that were not committed (graph warm-up)."""
        self._sync_dev_lengths()

    def add_sequence(self, seq_id: int):
        """Start sequence `seq_id` empty (kv_state_add_sequence, engine.py:112)."""
        if not 0 <= seq_id < self.max_batch:
            raise ValueError(f"sequence id {seq_id} outside the cache's {self.max_batch} sequences")
        self.lengths[seq_id] = 0
        self._sync_dev_lengths()

    def remove_sequence(self, seq_id: int):
        """Forget sequence `seq_id` (its rows are reused by the next sequence
        started in that slot)."""
        self.add_sequence(seq_id)

    def end_forward(self):
        """Close the pass planned by begin_forward (kv_state_end_forward,
        engine.py:141): the appends are already in the cache, nothing is left
        to do for a contiguous cache."""
        self._cur = None

    def popn(self, seq_id: int, n: int):
        self.lengths[seq_id] = max(0, int(self.lengths[seq_id]) - n)
        self._sync_dev_lengths()

    def clear(self):
        self.lengths.zero_()
        self._sync_dev_lengths()

    def total_length(self) -> int:
        return int(self.lengths.sum())


DENSE_GEMV = False  # decode-size projections through gptoss_dense_gemv instead of cuBLAS


def _linear(x2: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """nn.Linear with bias on [T, K] bf16: cuBLAS, or with DENSE_GEMV the
    library GEMV for few tokens (a weight stream)."""
    T = x2.shape[0]
    if DENSE_GEMV and 0 < T <= _lib.dense_max_tokens():
        x2 = x2.contiguous()
        out = torch.empty(T, weight.shape[0], dtype=torch.bfloat16, device=x2.device)
        _lib.call("gptoss_dense_gemv", _ptr(x2), T, _ptr(weight), _ptr(bias), weight.shape[0], weight.shape[1],
                  _ptr(out), _stream())
        return out
    return F.linear(x2, weight, bias)


class DecodeScratch:
    """Split-KV partial results of the decode kernel; one buffer can serve
    every layer of a model (the layers run one after another on one stream).
    It only grows, and it is sized before a decode step is captured."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() * 4 < nbytes:
            self.buf = torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=self.device)
        return self.buf


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
        self.scratch = DecodeScratch(dev)

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
        return self.scratch.get(nbytes), nbytes

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
        qkv = _linear(t, self.qkv_weight, self.qkv_bias)
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
        out = _linear(o.reshape(T, Hq * D), self.out_weight, self.out_bias)
        return (x2 + out).reshape(shape), kv_cache

    __call__ = forward
