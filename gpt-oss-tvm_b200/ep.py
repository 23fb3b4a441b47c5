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

Steps 1-2, 5 and 7 run in libgptoss_b200.so; the exchanges are plain NCCL
collectives (no peer-memory loads, no multicast).  The orchestration is
backend-agnostic so that the data movement can be tested on CPU ranks (gloo)
with a reference backend.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


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

    def __init__(self, blk, max_tokens: int, group=None, backend=None, exact_return: bool = False):
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
        self.backend = backend or CudaBackend(blk, max_tokens, self.world, exact_return)
        self.last_splits = None

    def forward(self, x, out=None):
        b = self.backend
        x2 = x.reshape(-1, self.blk.hidden_size)
        if out is None:
            out = torch.empty_like(x2)
        out2 = out.reshape(-1, self.blk.hidden_size)
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

    def profile_stages(self, x, repeats: int = 3) -> dict:
        """Per-stage CUDA-event timing of one expert-parallel step (this rank)."""
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
        pass
