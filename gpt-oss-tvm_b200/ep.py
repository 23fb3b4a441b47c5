"""Expert parallelism for the MoE block: experts sharded across ranks.

The reference runs the whole MoE block on one device (world_size = 1,
model/mlp.py:79).  Here each rank (one process per GPU, torch.distributed
over NCCL) owns ``num_experts / world`` experts and routes its own tokens:

  1. RMSNorm + router + top-k on the local tokens (router weights replicated);
  2. expert-major permutation over the *global* expert ids -- since the
     experts of rank d are contiguous, this is also destination-rank major;
  3. an all-to-all of the per-(rank, expert) row counts (the only host sync);
  4. one NCCL all-to-all-v of the bf16 token rows;
  5. reorder of the received rows from source-major to expert-major
     (gptoss_moe_segment_copy), tile plan, grouped MXFP4 GEMMs (mlp1 + SwiGLU,
     mlp2) on the local experts;
  6. reorder back to source-major, one NCCL all-to-all-v of the expert
     outputs back to the owning ranks -- rounded to bf16 on the way (half the
     bytes; within the block's tolerance) unless ``exact_return`` keeps them
     fp32, which makes the result bit-equal to the single-GPU block;
  7. weighted combine + residual on the owning rank.

Steps 1-2, 5 and 7 run in libgptoss_b200.so.  Two ways to move the rows:

* ``peer=True`` (the default on CUDA): the ranks share their activation and
  return buffers through CUDA IPC and the kernels write each other's rows
  directly over NVLink -- ``gptoss_moe_dispatch_peer`` stores every token row
  at its final row of the owning rank's expert-major activation matrix
  (replacing the gather, the all-to-all-v and the reorder), and the
  down-projection GEMM's epilogue (``gptoss_moe_mlp2_peer``) stores each
  output row into the return buffer of the rank that owns the token
  (replacing the reorder and the second all-to-all-v).  NCCL carries only
  the per-expert row counts (all-gather) and two one-word all-reduces that
  order the ranks around the peer writes.  Plain stores, no multicast, no
  device-side waits on other GPUs.
* ``peer=False``: the exchanges are NCCL all-to-all-v collectives.

The orchestration is backend-agnostic so that the data movement can be
tested on CPU ranks (gloo) with a reference backend; ``peer_layout`` (the
row addressing of the peer path) is checked there against the layout of the
all-to-all path.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def peer_layout(counts_all, rank: int, local_experts: int):
    """Row addressing of the peer-memory path.

    counts_all: [world, E] integer tensor, rows of source rank s for global
    expert g (every rank's expert-major permutation counts).  Rank d owns
    experts [d*El, (d+1)*El); its activation matrix is expert-major over them
    and source-rank-major within an expert -- the layout the all-to-all path
    builds with its reorder.  Returns, for source rank `rank`:
      dst_base [world, El]: first row on rank d of this rank's rows of d's
        local expert e;
      indptr_local [El + 1]: row offsets of this rank's own local experts;
      recv_rows: rows this rank receives.
    """
    W, E = counts_all.shape
    El = local_experts
    c = counts_all.reshape(W, W, El).to(torch.int64)   # [source, destination, local expert]
    per_dest = c.sum(0)                                 # [destination, local expert]
    start = torch.cumsum(per_dest, 1) - per_dest         # first row of each local expert on its rank
    before = c[:rank].sum(0)                            # rows of lower source ranks
    dst_base = (start + before).to(torch.int32)
    own = per_dest[rank]
    indptr_local = torch.zeros(El + 1, dtype=torch.int32)
    indptr_local[1:] = torch.cumsum(own, 0).to(torch.int32)
    return dst_base, indptr_local, int(own.sum())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class CudaBackend:
    """Device steps of the expert-parallel MoE block, through the C ABI."""

    def __init__(self, blk, max_tokens: int, world: int, exact_return: bool = False):
        self.blk = blk
        self.world = world
        self.exact_return = exact_return
        E, El, k, H, I = blk.num_experts, blk.num_local_experts, blk.experts_per_token, blk.hidden_size, \
            blk.intermediate_size
        dev = blk.device
        self.E, self.El, self.k, self.H, self.I = E, El, k, H, I
        i32 = dict(dtype=torch.int32, device=dev)
        M, R = max_tokens, max_tokens * k
        self.max_tokens = M
        self.t = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        self.logits = torch.empty(M, E, dtype=torch.bfloat16, device=dev)
        self.w = torch.empty(M, k, dtype=torch.bfloat16, device=dev)
        self.idx = torch.empty(M, k, **i32)
        self.indptr = torch.empty(E + 1, **i32)
        self.tile_ptr_g = torch.empty(E + 1, **i32)
        self.tile_rows_g = torch.empty(E, **i32)
        self.tok = torch.empty(R, **i32)
        self.rev = torch.empty(R, **i32)
        self.exr = torch.empty(R, **i32)
        self.send = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        self.indptr_local = torch.empty(El + 1, **i32)
        self.tile_ptr = torch.empty(El + 1, **i32)
        self.tile_rows = torch.empty(El, **i32)
        self.err = torch.zeros(4, **i32)
        self.f16 = 1 if blk.f16_path else 0  # rows travel in the GEMM's activation type
        self._recv_cap = 0
        self.back_dtype = torch.float32 if exact_return else torch.bfloat16
        self.h2_back = torch.empty(R, H, dtype=self.back_dtype, device=dev)
        self.peer = None

    # -- peer-memory path: IPC buffers shared by the ranks of `group`
    def setup_peer(self, group, rank: int):
        """Allocate this rank's activation rows, row origins and return rows
        with cudaMalloc, exchange IPC handles with the other ranks and map
        theirs.  Capacities hold every rank's rows (world * max_tokens * k)."""
        W, H, I, k, M = self.world, self.H, self.I, self.k, self.max_tokens
        cap = W * M * k
        sizes = [cap * H * 2, cap * 4, M * k * H * self.h2_back.element_size()]
        own, handles = [], []
        for nbytes in sizes:
            ptr, h = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
            _lib.call("gptoss_ipc_alloc", ctypes.c_uint64(nbytes), ctypes.byref(ptr), h)
            own.append(ptr.value)
            handles.append(bytes(h))
        mine = torch.frombuffer(bytearray(b"".join(handles)), dtype=torch.uint8).to(self.blk.device)
        allh = torch.empty(W * mine.numel(), dtype=torch.uint8, device=self.blk.device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu().numpy().tobytes()
        ptrs = [[0] * W for _ in sizes]
        opened = []
        for r in range(W):
            for i in range(len(sizes)):
                if r == rank:
                    ptrs[i][r] = own[i]
                    continue
                h = (ctypes.c_ubyte * 64).from_buffer_copy(allh[(r * len(sizes) + i) * 64:(r * len(sizes) + i + 1) * 64])
                p = ctypes.c_void_p()
                _lib.call("gptoss_ipc_open", h, ctypes.byref(p))
                ptrs[i][r] = p.value
                opened.append(p.value)
        arr = ctypes.c_void_p * W
        self.peer = dict(cap=cap, own=own, opened=opened, rank=rank, group=group,
                         rows=arr(*ptrs[0]), origin=arr(*ptrs[1]), back=arr(*ptrs[2]),
                         act=ctypes.c_void_p(own[0]), org=ctypes.c_void_p(own[1]), back_local=ctypes.c_void_p(own[2]),
                         dst_base=torch.empty(W * self.El, dtype=torch.int32, device=self.blk.device),
                         one=torch.ones(1, dtype=torch.int32, device=self.blk.device),
                         y=torch.empty(cap, I, dtype=torch.bfloat16, device=self.blk.device))

    def close_peer(self):
        if self.peer is None:
            return
        torch.cuda.synchronize()
        for p in self.peer["opened"]:
            _lib.call("gptoss_ipc_close", ctypes.c_void_p(p))
        for p in self.peer["own"]:
            _lib.call("gptoss_ipc_free", ctypes.c_void_p(p))
        self.peer = None

    def route(self, x):
        """Steps 1-2 without the gather: norm, router, top-k, expert-major permutation."""
        blk, S = self.blk, _stream()
        M = x.shape[0]
        E, k, H = self.E, self.k, self.H
        _lib.call("gptoss_rms_norm", _ptr(x), _ptr(blk.norm_weight), M, H, ctypes.c_float(blk.rms_norm_eps),
                  _ptr(self.t), S)
        _lib.call("gptoss_moe_router", _ptr(self.t), _ptr(blk.gate_weight), _ptr(blk.gate_bias), M, E, H, k,
                  _ptr(self.logits), _ptr(self.w), _ptr(self.idx), _ptr(self.err), S)
        _lib.call("gptoss_moe_permute", _ptr(self.idx), M, k, E, _ptr(self.indptr), _ptr(self.tok), _ptr(self.rev),
                  _ptr(self.exr), _ptr(self.tile_ptr_g), _ptr(self.tile_rows_g), _ptr(self.err), S)
        return (self.indptr[1:] - self.indptr[:-1]).contiguous()

    def layout_peer(self, counts_all, rank: int):
        """Row addressing from the all-gathered counts, on the device (peer_layout)."""
        _lib.call("gptoss_moe_peer_layout", _ptr(counts_all), self.world, self.El, rank, _ptr(self.peer["dst_base"]),
                  _ptr(self.indptr_local), _stream())

    def dispatch_peer(self, M: int):
        P, S = self.peer, _stream()
        _lib.call("gptoss_moe_dispatch_peer", _ptr(self.t), _ptr(self.tok), _ptr(self.exr), _ptr(self.indptr),
                  M * self.k, self.H, self.E, self.El, P["rank"], _ptr(P["dst_base"]), P["rows"], P["origin"],
                  self.world, P["cap"], self.f16, S)

    def experts_peer(self):
        """mlp1 + mlp2 on this rank's rows; mlp2's rows go to their owners' return buffers.
        The row count stays on the device: the GEMMs are launched on the buffer
        capacity and take their tiles from the device-side plan."""
        blk, P, S = self.blk, self.peer, _stream()
        H, I, El = self.H, self.I, self.El
        recv_rows = P["cap"]
        _lib.call("gptoss_moe_plan_tiles", _ptr(self.indptr_local), El, _ptr(self.tile_ptr), _ptr(self.tile_rows), S)
        y = P["y"]
        _lib.call("gptoss_moe_mlp1", P["act"], recv_rows, _ptr(self.indptr_local), _ptr(self.tile_ptr),
                  _ptr(self.tile_rows), El, H, I, _ptr(blk.mlp1_weight_blocks), _ptr(blk.mlp1_weight_scales),
                  _ptr(blk.mlp1_bias), ctypes.c_float(blk.swiglu_alpha), ctypes.c_float(blk.swiglu_limit),
                  self.f16, _ptr(y), _ptr(self.err), S)
        _lib.call("gptoss_moe_mlp2_peer", _ptr(y), recv_rows, _ptr(self.indptr_local), _ptr(self.tile_ptr),
                  _ptr(self.tile_rows), El, H, I, _ptr(blk.mlp2_weight_blocks), _ptr(blk.mlp2_weight_scales),
                  _ptr(blk.mlp2_bias), self.f16, P["org"], P["back"], self.world, self.max_tokens * self.k,
                  0 if self.exact_return else 1,
                  _ptr(self.err), S)

    def combine_peer(self, x, out):
        """Step 7 from this rank's return buffer (rows in send order)."""
        M = x.shape[0]
        fn = "gptoss_moe_combine" if self.exact_return else "gptoss_moe_combine_bf16"
        _lib.call(fn, self.peer["back_local"], _ptr(self.rev), _ptr(self.w), _ptr(x), M, self.k, self.H, _ptr(out),
                  _stream())
        return out

    def _ensure_recv(self, rows: int):
        if rows > self._recv_cap:
            cap = max(rows, int(self._recv_cap * 1.25))
            dev, H, I = self.blk.device, self.H, self.I
            self.recv = torch.empty(cap, H, dtype=torch.bfloat16, device=dev)
            self.act = torch.empty(cap, H, dtype=torch.bfloat16, device=dev)
            self.y = torch.empty(cap, I, dtype=torch.bfloat16, device=dev)
            self.h2_local = torch.empty(cap, H, dtype=torch.float32, device=dev)
            self.h2_src = torch.empty(cap, H, dtype=self.back_dtype, device=dev)
            self._recv_cap = cap

    # -- step 1-2
    def route_and_pack(self, x):
        blk, S = self.blk, _stream()
        M = x.shape[0]
        E, k, H = self.E, self.k, self.H
        _lib.call("gptoss_rms_norm", _ptr(x), _ptr(blk.norm_weight), M, H, ctypes.c_float(blk.rms_norm_eps),
                  _ptr(self.t), S)
        _lib.call("gptoss_moe_router", _ptr(self.t), _ptr(blk.gate_weight), _ptr(blk.gate_bias), M, E, H, k,
                  _ptr(self.logits), _ptr(self.w), _ptr(self.idx), _ptr(self.err), S)
        _lib.call("gptoss_moe_permute", _ptr(self.idx), M, k, E, _ptr(self.indptr), _ptr(self.tok), _ptr(self.rev),
                  _ptr(self.exr), _ptr(self.tile_ptr_g), _ptr(self.tile_rows_g), _ptr(self.err), S)
        _lib.call("gptoss_moe_gather", _ptr(self.t), _ptr(self.tok), M * k, H, self.f16, _ptr(self.send), S)
        counts = self.indptr[1:] - self.indptr[:-1]
        return self.send[: M * k], counts.view(self.world, self.El)

    # -- step 5
    def experts(self, recv_rows: int, recv_counts):
        blk, S = self.blk, _stream()
        H, I, El = self.H, self.I, self.El
        self._ensure_recv(recv_rows)
        if recv_rows == 0:
            return self.h2_src[:0]
        _lib.call("gptoss_moe_segment_copy", _ptr(self.recv), _ptr(self.act), _ptr(recv_counts), self.world, El,
                  H * 2, 0, _ptr(self.indptr_local), S)
        _lib.call("gptoss_moe_plan_tiles", _ptr(self.indptr_local), El, _ptr(self.tile_ptr), _ptr(self.tile_rows), S)
        _lib.call("gptoss_moe_mlp1", _ptr(self.act), recv_rows, _ptr(self.indptr_local), _ptr(self.tile_ptr),
                  _ptr(self.tile_rows), El, H, I, _ptr(blk.mlp1_weight_blocks), _ptr(blk.mlp1_weight_scales),
                  _ptr(blk.mlp1_bias), ctypes.c_float(blk.swiglu_alpha), ctypes.c_float(blk.swiglu_limit),
                  self.f16, _ptr(self.y), _ptr(self.err), S)
        _lib.call("gptoss_moe_mlp2", _ptr(self.y), recv_rows, _ptr(self.indptr_local), _ptr(self.tile_ptr),
                  _ptr(self.tile_rows), El, H, I, _ptr(blk.mlp2_weight_blocks), _ptr(blk.mlp2_weight_scales),
                  _ptr(blk.mlp2_bias), self.f16, _ptr(self.h2_local), _ptr(self.err), S)
        _lib.call("gptoss_moe_segment_copy", _ptr(self.h2_local), _ptr(self.h2_src), _ptr(recv_counts), self.world, El,
                  H * 4, 1 if self.exact_return else 2, None, S)
        return self.h2_src[:recv_rows]

    def recv_buffer(self, rows: int):
        self._ensure_recv(rows)
        return self.recv[:rows]

    def back_buffer(self, rows: int):
        return self.h2_back[:rows]

    # -- step 7
    def combine(self, h2_back, x, out):
        M = x.shape[0]
        fn = "gptoss_moe_combine" if self.exact_return else "gptoss_moe_combine_bf16"
        _lib.call(fn, _ptr(h2_back), _ptr(self.rev), _ptr(self.w), _ptr(x), M, self.k, self.H, _ptr(out), _stream())
        return out

    def device_error(self) -> int:
        v = int(self.err[0].item())
        self.err.zero_()
        return v


class ExpertParallelMoE:
    """MLPBlock.forward with the experts sharded over the ranks of `group`."""

    def __init__(self, blk, max_tokens: int, group=None, backend=None, exact_return: bool = False,
                 peer: bool | None = None):
        """peer: move the rows through shared IPC buffers (default: True for the
        CUDA backend, False for a custom backend)."""
        self.blk = blk
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if blk.num_experts != blk.num_local_experts * self.world:
            raise ValueError("num_experts must equal num_local_experts * world size")
        if blk.expert_offset != self.rank * blk.num_local_experts:
            raise ValueError("rank r must own experts [r*El, (r+1)*El)")
        if hasattr(blk, "flags") and backend is None:
            # every rank must run the same GEMM path (the rows travel in its activation type)
            f = torch.tensor([int(blk.flags)], dtype=torch.int32, device=blk.device)
            dist.all_reduce(f, op=dist.ReduceOp.MIN, group=group)
            blk.flags = int(f.item())
        self.peer = (backend is None) if peer is None else peer
        self.backend = backend or CudaBackend(blk, max_tokens, self.world, exact_return)
        if self.peer:
            self.backend.setup_peer(group, self.rank)
        self._splits = None
        self._counts_all = None

    def use(self, blk) -> "ExpertParallelMoE":
        """Run the next forwards on `blk`'s weights (the same expert shard and
        shapes): one runner, with one set of exchange buffers, serves every MoE
        layer of a model.  Every rank must switch to the same layer, and the
        ranks must agree on each layer's GEMM path (flags)."""
        a, b = self.blk, blk
        if (a.num_experts, a.num_local_experts, a.expert_offset, a.hidden_size) != \
                (b.num_experts, b.num_local_experts, b.expert_offset, b.hidden_size):
            raise ValueError("ExpertParallelMoE.use: a block of another expert shard or shape")
        self.blk = blk
        self.backend.blk = blk
        if hasattr(self.backend, "f16"):
            self.backend.f16 = 1 if blk.f16_path else 0
        return self

    def _layout(self, counts):
        """All-gather the per-expert row counts and lay out the rows (no host round trip)."""
        counts_all = torch.empty(self.world * counts.numel(), dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(counts_all, counts, group=self.group)
        self._counts_all = counts_all.view(self.world, counts.numel())
        self.backend.layout_peer(self._counts_all, self.rank)

    @property
    def last_splits(self):
        """(rows sent to each rank, rows received from each rank) of the last step."""
        if self._splits is None and self._counts_all is not None:
            El = self.blk.num_local_experts
            per = self._counts_all.cpu().reshape(self.world, self.world, El).sum(2)  # [source, destination]
            self._splits = (per[self.rank].tolist(), per[:, self.rank].tolist())
        return self._splits

    @last_splits.setter
    def last_splits(self, v):
        self._splits = v

    def _order(self):
        """Every rank's kernels issued so far have completed (their peer stores are visible)."""
        dist.all_reduce(self.backend.peer["one"], op=dist.ReduceOp.MAX, group=self.group)

    def _forward_peer(self, x2, out2):
        b = self.backend
        self._splits = None
        counts = b.route(x2)
        self._layout(counts)
        b.dispatch_peer(x2.shape[0])
        self._order()
        b.experts_peer()
        self._order()
        b.combine_peer(x2, out2)

    def forward(self, x, out=None):
        b = self.backend
        x2 = x.reshape(-1, self.blk.hidden_size)
        cap = getattr(b, "max_tokens", None)  # the CUDA backend's buffers hold max_tokens rows
        if cap is not None and x2.shape[0] > cap:
            raise ValueError(f"ExpertParallelMoE: {x2.shape[0]} tokens exceed max_tokens={cap}")
        if out is None:
            out = torch.empty_like(x2)
        out2 = out.reshape(-1, self.blk.hidden_size)
        if self.peer:
            self._forward_peer(x2, out2)
            return out
        send, send_counts = b.route_and_pack(x2)
        send_counts = send_counts.contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        both = torch.stack([send_counts, recv_counts]).cpu()  # the one host synchronisation of the step
        in_splits = both[0].sum(1).tolist()
        out_splits = both[1].sum(1).tolist()
        recv_rows = int(sum(out_splits))
        recv = b.recv_buffer(recv_rows)
        dist.all_to_all_single(recv, send, output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)
        h2_src = b.experts(recv_rows, recv_counts)
        back = b.back_buffer(send.shape[0])
        dist.all_to_all_single(back, h2_src, output_split_sizes=in_splits, input_split_sizes=out_splits,
                               group=self.group)
        b.combine(back, x2, out2)
        self.last_splits = (in_splits, out_splits)
        return out

    __call__ = forward

    def _profile_peer(self, x, repeats: int) -> dict:
        b = self.backend
        best = None
        x2 = x.reshape(-1, self.blk.hidden_size)
        out = torch.empty_like(x2)
        names = ["route", "counts", "dispatch", "dispatch_sync", "mlp1", "mlp2_return", "return_sync", "combine"]
        for _ in range(repeats):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
            dist.barrier(group=self.group)
            ev[0].record()
            counts = b.route(x2)
            ev[1].record()
            self._layout(counts)
            ev[2].record()
            b.dispatch_peer(x2.shape[0])
            ev[3].record()
            self._order()
            ev[4].record()
            blk, P, S = self.blk, b.peer, _stream()
            H, I, El = b.H, b.I, b.El
            recv_rows = P["cap"]
            _lib.call("gptoss_moe_plan_tiles", _ptr(b.indptr_local), El, _ptr(b.tile_ptr), _ptr(b.tile_rows), S)
            _lib.call("gptoss_moe_mlp1", P["act"], recv_rows, _ptr(b.indptr_local), _ptr(b.tile_ptr),
                      _ptr(b.tile_rows), El, H, I, _ptr(blk.mlp1_weight_blocks), _ptr(blk.mlp1_weight_scales),
                      _ptr(blk.mlp1_bias), ctypes.c_float(blk.swiglu_alpha), ctypes.c_float(blk.swiglu_limit),
                      b.f16, _ptr(P["y"]), _ptr(b.err), S)
            ev[5].record()
            _lib.call("gptoss_moe_mlp2_peer", _ptr(P["y"]), recv_rows, _ptr(b.indptr_local), _ptr(b.tile_ptr),
                      _ptr(b.tile_rows), El, H, I, _ptr(blk.mlp2_weight_blocks), _ptr(blk.mlp2_weight_scales),
                      _ptr(blk.mlp2_bias), b.f16, P["org"], P["back"], b.world, b.max_tokens * b.k,
                      0 if b.exact_return else 1,
                      _ptr(b.err), S)
            ev[6].record()
            self._order()
            ev[7].record()
            b.combine_peer(x2, out)
            ev[8].record()
            torch.cuda.synchronize()
            tms = {f"{n}_ms": ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(names)}
            tms["recv_rows"] = int(b.indptr_local[-1].item())
            if best is None or tms["mlp1_ms"] < best["mlp1_ms"]:
                best = tms
        R = best.pop("recv_rows")
        best["mlp1_flops"] = 2.0 * R * 2 * b.I * b.H
        best["mlp2_flops"] = 2.0 * R * b.H * b.I
        best["gemm_flops"] = best["mlp1_flops"] + best["mlp2_flops"]
        best["gemm_ms"] = best["mlp1_ms"] + best["mlp2_return_ms"]
        # norm, router, topk, count, place, dispatch, plan, mlp1, mlp2 (+ return), combine
        best["launches_per_step"] = 10
        best["exchange"] = "peer memory (CUDA IPC, NVLink stores in dispatch and in the mlp2 epilogue)"
        return best

    def profile_stages(self, x, repeats: int = 3) -> dict:
        """Per-stage CUDA-event timing of one expert-parallel step (this rank)."""
        if self.peer:
            return self._profile_peer(x, repeats)
        b = self.backend
        best = None
        x2 = x.reshape(-1, self.blk.hidden_size)
        out = torch.empty_like(x2)
        for _ in range(repeats):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(9)]
            dist.barrier(group=self.group)
            ev[0].record()
            send, send_counts = b.route_and_pack(x2)
            send_counts = send_counts.contiguous()
            ev[1].record()
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            both = torch.stack([send_counts, recv_counts]).cpu()
            in_splits = both[0].sum(1).tolist()
            out_splits = both[1].sum(1).tolist()
            recv_rows = int(sum(out_splits))
            recv = b.recv_buffer(recv_rows)
            ev[2].record()
            dist.all_to_all_single(recv, send, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                   group=self.group)
            ev[3].record()
            S = _stream()
            H, I, El = b.H, b.I, b.El
            _lib.call("gptoss_moe_segment_copy", _ptr(b.recv), _ptr(b.act), _ptr(recv_counts), b.world, El, H * 2, 0,
                      _ptr(b.indptr_local), S)
            _lib.call("gptoss_moe_plan_tiles", _ptr(b.indptr_local), El, _ptr(b.tile_ptr), _ptr(b.tile_rows), S)
            ev[4].record()
            blk = self.blk
            _lib.call("gptoss_moe_mlp1", _ptr(b.act), recv_rows, _ptr(b.indptr_local), _ptr(b.tile_ptr),
                      _ptr(b.tile_rows), El, H, I, _ptr(blk.mlp1_weight_blocks), _ptr(blk.mlp1_weight_scales),
                      _ptr(blk.mlp1_bias), ctypes.c_float(blk.swiglu_alpha), ctypes.c_float(blk.swiglu_limit),
                      b.f16, _ptr(b.y), _ptr(b.err), S)
            ev[5].record()
            _lib.call("gptoss_moe_mlp2", _ptr(b.y), recv_rows, _ptr(b.indptr_local), _ptr(b.tile_ptr),
                      _ptr(b.tile_rows), El, H, I, _ptr(blk.mlp2_weight_blocks), _ptr(blk.mlp2_weight_scales),
                      _ptr(blk.mlp2_bias), b.f16, _ptr(b.h2_local), _ptr(b.err), S)
            _lib.call("gptoss_moe_segment_copy", _ptr(b.h2_local), _ptr(b.h2_src), _ptr(recv_counts), b.world, El,
                      H * 4, 1 if b.exact_return else 2, None, S)
            ev[6].record()
            back = b.back_buffer(send.shape[0])
            dist.all_to_all_single(back, b.h2_src[:recv_rows], output_split_sizes=in_splits,
                                   input_split_sizes=out_splits, group=self.group)
            ev[7].record()
            b.combine(back, x2, out)
            ev[8].record()
            torch.cuda.synchronize()
            names = ["route", "counts", "dispatch", "reorder", "mlp1", "mlp2", "combine_a2a", "combine"]
            tms = {f"{n}_ms": ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(names)}
            tms["recv_rows"] = recv_rows
            if best is None or tms["mlp1_ms"] < best["mlp1_ms"]:
                best = tms
        R = best.pop("recv_rows")
        best["mlp1_flops"] = 2.0 * R * 2 * b.I * b.H
        best["mlp2_flops"] = 2.0 * R * b.H * b.I
        best["gemm_flops"] = best["mlp1_flops"] + best["mlp2_flops"]
        best["gemm_ms"] = best["mlp1_ms"] + best["mlp2_ms"]
        # norm, router, topk, count, place, gather, reorder, plan, mlp1, mlp2, reorder, combine
        best["launches_per_step"] = 12
        return best

    def close(self):
        if self.peer and hasattr(self.backend, "close_peer"):
            self.backend.close_peer()
