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

The KV cache is paged like the reference's PagedKVCache (page size 16):
full-attention layers hold every key in pages from a free list, the
sliding-window layers a ring of pages per sequence that keeps the last keys
only; the attention semantics (append before attention, window of the last W
keys including the current token) are the reference's (tvm_fix.patch:35-47,
:194-281).  A prefill / extend chunk attends over one contiguous buffer: the
cached keys its window can reach, gathered from the pages, then its own.
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


PAGE_SIZE = 16  # tokens per KV page (the reference's cache, engine.py:102)


class KVCache:
    """Paged KV cache (the reference's PagedKVCache, page size 16,
    engine.py:93-104), per layer one page pool per K and V
    ([pages * 16, Hkv, D] bf16).

    Full-attention layers: each sequence owns a list of pages taken from a free
    list as it grows (``table_full`` [max_batch, ceil(max_len / 16)], host copy
    and device mirror); ``popn`` returns the pages it empties.
    Sliding-window layers keep only the last keys: each sequence has a fixed
    ring of ``window_pages`` pages (by default ceil(window / 16) + 1 = 9 for the
    128-token window, 144 rows instead of max_len), logical page p living in
    ring slot p % window_pages -- the window of the last `window` keys plus the
    page being filled (tvm_fix.patch:194-281 reads the same last pages).  A
    ``popn`` that would need keys older than the ring holds raises.

    The host keeps the authoritative sequence lengths (``lengths``); the device
    keeps a mirror (``dev_lengths``) so that a decode step can plan itself on
    the device (``begin_decode_on_device``) inside a CUDA graph; the
    decode-step buffers never move, so a captured graph keeps reading the
    current values.  ``check_decode`` makes sure every decoding sequence has a
    page for its next token (host allocation, device table refreshed)."""

    def __init__(self, config: GPTOssConfig, max_batch: int, max_len: int, num_layers: int | None = None,
                 device="cuda", window_pages: int | None = None):
        if max_batch < 1 or max_len < 1 or max_batch * (max_len + PAGE_SIZE) >= 2 ** 31:
            raise ValueError(f"KVCache: max_batch x max_len = {max_batch} x {max_len} must fit int32 rows")
        self.config = config
        self.max_batch, self.max_len = max_batch, max_len
        L = num_layers if num_layers is not None else config.num_hidden_layers
        Hkv, D = config.num_key_value_heads, config.head_dim
        self.window = int(config.sliding_window_size)
        self.pages_per_seq = -(-max_len // PAGE_SIZE)                    # table stride, full layers
        self.window_pages = window_pages or (-(-self.window // PAGE_SIZE) + 1)
        if self.window_pages * PAGE_SIZE < self.window + PAGE_SIZE - 1:
            raise ValueError("window_pages must cover the window plus the page being filled")
        self.full_pool_pages = max_batch * self.pages_per_seq
        self.device = torch.device(device)
        dev = self.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.windowed = [(i % config.sliding_window_pattern == 0) and self.window > 0 for i in range(L)]
        self.k, self.v = [], []
        for w in self.windowed:
            rows = (max_batch * self.window_pages if w else self.full_pool_pages) * PAGE_SIZE
            self.k.append(torch.zeros(rows, Hkv, D, **bf))
            self.v.append(torch.zeros(rows, Hkv, D, **bf))
        i32 = dict(dtype=torch.int32, device=dev)
        # full layers: page lists (host) and their device mirror; windowed layers: fixed rings
        self._free = list(range(self.full_pool_pages - 1, -1, -1))
        self._pages = [[] for _ in range(max_batch)]
        self.table_full_host = torch.zeros(max_batch, self.pages_per_seq, dtype=torch.int32)
        self.table_full = torch.zeros(max_batch, self.pages_per_seq, **i32)
        self.table_win = (torch.arange(max_batch * self.window_pages, **i32)
                          .reshape(max_batch, self.window_pages))
        self._table_dirty = False
        self.lengths = torch.zeros(max_batch, dtype=torch.int32)  # host copy
        # highest position + 1 ever written per sequence since it started: the
        # window rings hold the pages up to it (a popn does not rewind them)
        self._written = [0] * max_batch
        self.dev_lengths = torch.zeros(max_batch, **i32)
        self._row_full = (torch.arange(max_batch, dtype=torch.int64, device=dev) * self.pages_per_seq)
        self._row_win = (torch.arange(max_batch, **i32) * self.window_pages)
        self._dec_pos = torch.zeros(max_batch, **i32)
        self._dec_slot = torch.zeros(max_batch, **i32)
        self._dec_slot_win = torch.zeros(max_batch, **i32)
        self._kv_len = torch.zeros(max_batch, **i32)
        self._pos = torch.zeros(max_batch, **i32)
        self._slot = torch.zeros(max_batch, **i32)
        self._slot_win = torch.zeros(max_batch, **i32)
        self._cur = None
        self.start = 0  # first position of the current prefill / extend chunk

    # ------------------------------------------------------------- pages --
    def table(self, layer_idx: int):
        """(page table, stride) of a layer's pools."""
        if self.windowed[layer_idx]:
            return self.table_win, self.window_pages
        return self.table_full, self.pages_per_seq

    def _ensure_pages(self, seq: int, length: int):
        need = -(-length // PAGE_SIZE)
        pages = self._pages[seq]
        if need > self.pages_per_seq:
            raise ValueError("KV cache full")
        while len(pages) < need:
            if not self._free:
                raise ValueError("KV cache full (no free pages)")
            p = self._free.pop()
            self.table_full_host[seq, len(pages)] = p
            pages.append(p)
            self._table_dirty = True

    def _release_pages(self, seq: int, length: int):
        keep = -(-length // PAGE_SIZE)
        pages = self._pages[seq]
        while len(pages) > keep:
            self._free.append(pages.pop())

    def _sync_tables(self):
        if self._table_dirty:
            self.table_full.copy_(self.table_full_host.to(self.device))
            self._table_dirty = False

    def _sync_dev_lengths(self):
        self.dev_lengths.copy_(self.lengths.to(self.device))

    def _slots(self, seq: int, pos: torch.Tensor):
        """Pool rows of positions `pos` of sequence `seq` (host): full, windowed."""
        page = pos // PAGE_SIZE
        full = self.table_full_host[seq][page.long()] * PAGE_SIZE + pos % PAGE_SIZE
        win = (seq * self.window_pages + page % self.window_pages) * PAGE_SIZE + pos % PAGE_SIZE
        return full.to(torch.int32), win.to(torch.int32)

    # ----------------------------------------------------------- planning --
    def begin_forward(self, seq_ids, append_lengths):
        """Plan one forward pass (kv_state_begin_forward, engine.py:135-139):
        allocates the pages the appended tokens need and returns their query
        positions."""
        pos, slots, slots_w = [], [], []
        new_len = self.lengths.clone()
        starts = []
        for s, n in zip(seq_ids, append_lengths):
            if not 0 <= s < self.max_batch:
                raise ValueError(f"sequence id {s} outside the cache's {self.max_batch} sequences")
            start = int(new_len[s])
            if start + n > self.max_len:
                raise ValueError("KV cache full")
            self._ensure_pages(s, start + n)
            p = torch.arange(start, start + n, dtype=torch.int32)
            sf, sw = self._slots(s, p)
            pos.append(p)
            slots.append(sf)
            slots_w.append(sw)
            starts.append(start)
            new_len[s] = start + n
            self._written[s] = max(self._written[s], start + n)
        self.lengths.copy_(new_len)
        self._cur = (list(seq_ids), list(append_lengths))
        self.start = starts[0] if len(starts) == 1 else 0
        cat = lambda xs: torch.cat(xs) if xs else torch.zeros(0, dtype=torch.int32)  # noqa: E731
        pos, slots, slots_w = cat(pos), cat(slots), cat(slots_w)
        T = pos.numel()
        if T > self._pos.numel():
            i32 = dict(dtype=torch.int32, device=self.device)
            self._pos, self._slot, self._slot_win = (torch.zeros(T, **i32), torch.zeros(T, **i32),
                                                     torch.zeros(T, **i32))
        self._pos[:T].copy_(pos)
        self._slot[:T].copy_(slots)
        self._slot_win[:T].copy_(slots_w)
        nb = len(seq_ids)
        self._kv_len[:nb].copy_(torch.tensor([int(self.lengths[s]) for s in seq_ids], dtype=torch.int32))
        self._sync_tables()
        self._sync_dev_lengths()
        self.positions, self.kv_len = self._pos[:T], self._kv_len[:nb]
        self.slots, self.slots_win = self._slot[:T], self._slot_win[:T]
        return self.positions

    def slots_for(self, layer_idx: int):
        return self.slots_win if self.windowed[layer_idx] else self.slots

    def check_decode(self, batch: int, steps: int = 1):
        """Before a decode step of sequences 0..batch-1: capacity, and a page
        for each sequence's next `steps` tokens (full layers)."""
        if not 1 <= batch <= self.max_batch:
            raise ValueError(f"decode batch {batch} outside 1..{self.max_batch}")
        if int(self.lengths[:batch].max()) + steps > self.max_len:
            raise ValueError("KV cache full")
        for s in range(batch):
            self._ensure_pages(s, int(self.lengths[s]) + steps)
        self._sync_tables()

    def begin_decode_on_device(self, batch: int):
        """begin_forward(range(batch), [1] * batch) done by device ops only
        (capturable in a CUDA graph): position = current length, the pool rows
        from the page tables, length += 1.  The host mirror is advanced by
        ``commit_decode`` after the step has been issued."""
        self._cur = (list(range(batch)), [1] * batch)
        pos, slot, slot_w, kvl = (self._dec_pos[:batch], self._dec_slot[:batch], self._dec_slot_win[:batch],
                                  self._kv_len[:batch])
        pos.copy_(self.dev_lengths[:batch])
        page = torch.bitwise_right_shift(pos, 4)
        off = torch.bitwise_and(pos, PAGE_SIZE - 1)
        idx = self._row_full[:batch] + page.long()
        slot.copy_(torch.take(self.table_full, idx) * PAGE_SIZE + off)
        slot_w.copy_((self._row_win[:batch] + torch.remainder(page, self.window_pages)) * PAGE_SIZE + off)
        self.dev_lengths[:batch].add_(1)
        kvl.copy_(self.dev_lengths[:batch])
        self.positions, self.slots, self.slots_win, self.kv_len = pos, slot, slot_w, kvl
        self.start = 0
        return pos

    def commit_decode(self, batch: int, steps: int = 1):
        self.lengths[:batch] += steps
        for s in range(batch):
            self._written[s] = max(self._written[s], int(self.lengths[s]))

    def rollback_device(self):
        """Forget device-side steps that were not committed (graph warm-up)."""
        self._sync_dev_lengths()

    def add_sequence(self, seq_id: int):
        """Start sequence `seq_id` empty (kv_state_add_sequence, engine.py:112)."""
        if not 0 <= seq_id < self.max_batch:
            raise ValueError(f"sequence id {seq_id} outside the cache's {self.max_batch} sequences")
        self._release_pages(seq_id, 0)
        self.lengths[seq_id] = 0
        self._written[seq_id] = 0
        self._sync_dev_lengths()

    def remove_sequence(self, seq_id: int):
        """Forget sequence `seq_id` and return its pages."""
        self.add_sequence(seq_id)

    def end_forward(self):
        """Close the pass planned by begin_forward (kv_state_end_forward,
        engine.py:141): the appends are already in the pages."""
        self._cur = None

    def popn(self, seq_id: int, n: int):
        """Drop the last n tokens of a sequence (kv_state_popn, engine.py:124-125):
        page-granular, the emptied pages go back to the free list.  On
        sliding-window layers the ring must still hold the new window."""
        cur = int(self.lengths[seq_id])
        new = max(0, cur - n)
        if self.window > 0 and new > 0 and any(self.windowed):
            hw = self._written[seq_id]
            oldest_kept = max(0, (hw - 1) // PAGE_SIZE - self.window_pages + 1) * PAGE_SIZE
            if max(0, new - self.window) < oldest_kept:
                raise ValueError(f"popn({seq_id}, {n}): the sliding-window layers keep positions from {oldest_kept} "
                                 f"on, the window after the pop needs {max(0, new - self.window)}")
        self.lengths[seq_id] = new
        self._release_pages(seq_id, new)
        self._sync_dev_lengths()

    def clear(self):
        for s in range(self.max_batch):
            self._release_pages(s, 0)
            self._written[s] = 0
        self.lengths.zero_()
        self._sync_dev_lengths()

    def total_length(self) -> int:
        return int(self.lengths.sum())

    def copy_sequence(self, src: int, dst: int):
        """Sequence `dst` becomes a copy of sequence `src` (its own pages with the
        same keys and values in every layer, the same length)."""
        n = int(self.lengths[src])
        self._release_pages(dst, 0)
        self._ensure_pages(dst, n)
        self._sync_tables()
        npg = -(-n // PAGE_SIZE)
        ar = torch.arange(PAGE_SIZE, dtype=torch.int64)
        if npg:
            src_rows = (self.table_full_host[src][:npg].long()[:, None] * PAGE_SIZE + ar).reshape(-1)
            dst_rows = (self.table_full_host[dst][:npg].long()[:, None] * PAGE_SIZE + ar).reshape(-1)
        R = self.window_pages
        ring = torch.arange(R * PAGE_SIZE, dtype=torch.int64)
        for i, w in enumerate(self.windowed):
            if w:
                a, b = (src * R * PAGE_SIZE + ring).to(self.device), (dst * R * PAGE_SIZE + ring).to(self.device)
            elif npg:
                a, b = src_rows.to(self.device), dst_rows.to(self.device)
            else:
                continue
            self.k[i].index_copy_(0, b, self.k[i].index_select(0, a))
            self.v[i].index_copy_(0, b, self.v[i].index_select(0, a))
        self.lengths[dst] = n
        self._written[dst] = self._written[src]
        self._sync_dev_lengths()

    def read_rows(self, layer_idx: int, seq: int, pos0: int, n: int):
        """Keys and values of positions pos0 .. pos0 + n - 1 of a sequence in a
        layer ([n, Hkv, D] each, copies); a sliding-window layer has only the
        positions its ring still holds."""
        table, stride = self.table(layer_idx)
        p = torch.arange(pos0, pos0 + n, dtype=torch.int64)
        if self.windowed[layer_idx]:
            rows = (seq * stride + (p // PAGE_SIZE) % stride) * PAGE_SIZE + p % PAGE_SIZE
        else:
            rows = self.table_full_host[seq][p // PAGE_SIZE].long() * PAGE_SIZE + p % PAGE_SIZE
        rows = rows.to(self.k[layer_idx].device)
        return self.k[layer_idx].index_select(0, rows), self.v[layer_idx].index_select(0, rows)

    def memory_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


DENSE_GEMV = False  # decode-size projections through gptoss_dense_gemv instead of cuBLAS
# Decode-size projections with a long reduction (the out projection, K = 4096)
# on the library's tcgen05 GEMM (split-K clusters), where it beats cuBLAS in
# the decode graphs (gpt-oss-20b batch 1: 3.26 -> 3.20 ms per step; batch 8:
# 5.85 -> 5.81); the qkv projection (K = 2880) stays on cuBLAS, which is faster
# there.  0 turns it off.
DENSE_TC_MAX_TOKENS = 8
DENSE_TC_MIN_K = 4096


def _linear(x2: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """nn.Linear with bias on [T, K] bf16: cuBLAS; the library's tcgen05 GEMM
    for few tokens and K >= DENSE_TC_MIN_K; with DENSE_GEMV the library GEMV
    for few tokens (a weight stream)."""
    T = x2.shape[0]
    if DENSE_GEMV and 0 < T <= _lib.dense_max_tokens():
        x2 = x2.contiguous()
        out = torch.empty(T, weight.shape[0], dtype=torch.bfloat16, device=x2.device)
        _lib.call("gptoss_dense_gemv", _ptr(x2), T, _ptr(weight), _ptr(bias), weight.shape[0], weight.shape[1],
                  _ptr(out), _stream())
        return out
    if 0 < T <= DENSE_TC_MAX_TOKENS and weight.shape[1] >= DENSE_TC_MIN_K and x2.is_cuda:
        x2 = x2.contiguous()
        out = torch.empty(T, weight.shape[0], dtype=torch.bfloat16, device=x2.device)
        _lib.call("gptoss_dense_gemm", _ptr(x2), T, _ptr(weight), _ptr(bias), weight.shape[0], weight.shape[1],
                  _ptr(out), None, _stream())
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
        L = self.layer_idx
        kc, vc = kv_cache.k[L], kv_cache.v[L]
        table, stride = kv_cache.table(L)
        pos = query_positions if query_positions is not None else kv_cache.positions
        o = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=x.device)
        seq_ids, lens = kv_cache._cur
        if forward_to in ("prefill", "extend"):
            if len(seq_ids) != 1:
                raise ValueError("prefill / extend take one sequence (batch size 1, as in the reference)")
            sid = seq_ids[0]
            start = kv_cache.start
            # keys attended: the cached ones the window (or the full causal mask)
            # can reach, then the chunk's own -- one contiguous buffer
            g0 = max(0, start - self.sliding_window) if self.sliding_window > 0 else 0
            ctx = start - g0
            kb = torch.empty(ctx + T, Hkv, D, dtype=torch.bfloat16, device=x.device)
            vb = torch.empty_like(kb)
            _lib.call("gptoss_qkv_rope_append", _ptr(qkv), _ptr(pos), None, T, Hq, Hkv, D, self._inv_freq,
                      ctypes.c_float(self._conc), _ptr(q), _ptr(kb[ctx:]), _ptr(vb[ctx:]), S)
            if ctx > 0:
                _lib.call("gptoss_kv_pages_copy", _ptr(kc), _ptr(vc), Hkv, D, _ptr(table), stride, sid, g0, ctx,
                          _ptr(kb), _ptr(vb), 0, S)
            # append_mha_kv: the chunk into the pages (a ring keeps its last rows only)
            keep = T if not kv_cache.windowed[L] else min(T, stride * PAGE_SIZE)
            _lib.call("gptoss_kv_pages_copy", _ptr(kc), _ptr(vc), Hkv, D, _ptr(table), stride, sid,
                      start + T - keep, keep, _ptr(kb[ctx + T - keep:]), _ptr(vb[ctx + T - keep:]), 1, S)
            _lib.call("gptoss_attn_prefill", _ptr(q), _ptr(kb), _ptr(vb), _ptr(self.sinks), T, ctx + T, Hq, Hkv, D,
                      self.sliding_window, ctypes.c_float(self.sm_scale), _ptr(o), None, S)
        elif forward_to == "decode":
            if any(n != 1 for n in lens) or min(seq_ids) != 0 or list(seq_ids) != list(range(len(seq_ids))):
                raise ValueError("decode takes one token for each of sequences 0..B-1")
            B = len(seq_ids)
            _lib.call("gptoss_qkv_rope_append", _ptr(qkv), _ptr(pos), _ptr(kv_cache.slots_for(L)), T, Hq, Hkv, D,
                      self._inv_freq, ctypes.c_float(self._conc), _ptr(q), _ptr(kc), _ptr(vc), S)
            scratch, nbytes = self._scratch_for(B, stride * PAGE_SIZE)
            _lib.call("gptoss_attn_decode_paged", _ptr(q), _ptr(kc), _ptr(vc), _ptr(table), stride,
                      _ptr(kv_cache.kv_len), B, Hq, Hkv, D, self.sliding_window, ctypes.c_float(self.sm_scale),
                      _ptr(self.sinks), _ptr(scratch), nbytes, _ptr(o), None, S)
        else:
            raise ValueError(f"forward_to {forward_to} not supported")
        out = _linear(o.reshape(T, Hq * D), self.out_weight, self.out_bias)
        return (x2 + out).reshape(shape), kv_cache

    __call__ = forward
