"""MLPBlock: the gpt-oss MXFP4 mixture-of-experts block on B200.

Same construction and call signature as the reference
(``MLPBlock(config, rms_norm_eps=1e-5, dtype=None).forward(x)``,
model/mlp.py:63-402), the same parameter names and layouts, and the same
result: ``x + MoE(RMSNorm(x))`` for ``x`` of shape ``[b, s, hidden]`` bf16.
Parameters and activations are torch CUDA tensors; all compute runs in
libgptoss_b200.so (no CPU fallback).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .config import GPTOssConfig

GROUPS_PER_ROW = 90  # 32-element MXFP4 blocks per 2880-wide row (model/mlp.py:97)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class MLPBlock:
    """MXFP4 MoE block (model/mlp.py:63-402)."""

    def __init__(self, config: GPTOssConfig, rms_norm_eps: float = 1e-5, dtype: str | None = None,
                 device: str | torch.device = "cuda", expert_offset: int = 0, num_local_experts: int | None = None):
        self.config = config
        self.dtype = dtype or config.dtype
        if self.dtype != "bfloat16":
            raise ValueError("MLPBlock supports bfloat16 activations only")
        self.num_experts = config.num_experts
        self.experts_per_token = config.num_experts_per_tok
        self.swiglu_limit = float(config.swiglu_limit)
        self.swiglu_alpha = 1.702
        self.hidden_size = config.hidden_size
        self.intermediate_size = config.intermediate_size
        self.rms_norm_eps = float(rms_norm_eps)
        self.expert_offset = expert_offset
        self.num_local_experts = num_local_experts or config.num_experts
        self.device = torch.device(device)
        E, El, H, I = self.num_experts, self.num_local_experts, self.hidden_size, self.intermediate_size
        g_in, g_mid = H // 32, I // 32
        dev = self.device
        # parameters, named as in the reference (model/mlp.py:81-143)
        self.norm_weight = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.gate_weight = torch.zeros(E, H, dtype=torch.bfloat16, device=dev)
        self.gate_bias = torch.zeros(E, dtype=torch.bfloat16, device=dev)
        self.mlp1_weight_blocks = torch.zeros(El, 2 * I, g_in, 16, dtype=torch.uint8, device=dev)
        self.mlp1_weight_scales = torch.full((El, 2 * I, g_in), 127, dtype=torch.uint8, device=dev)
        self.mlp1_bias = torch.zeros(El, 2 * I, dtype=torch.bfloat16, device=dev)
        self.mlp2_weight_blocks = torch.zeros(El, H, g_mid, 16, dtype=torch.uint8, device=dev)
        self.mlp2_weight_scales = torch.full((El, H, g_mid), 127, dtype=torch.uint8, device=dev)
        self.mlp2_bias = torch.zeros(El, H, dtype=torch.bfloat16, device=dev)
        self._ws = None
        self._ws_tokens = 0
        self._ws_owner = self
        self.flags = 0            # GPTOSS_MOE_* bits (set by prepare())
        self.allow_f16 = True     # let prepare() enable the f16 GEMM path when it is exact

    # reference-style parameter names ------------------------------------
    PARAM_NAMES = {
        "norm.weight": "norm_weight", "gate.weight": "gate_weight", "gate.bias": "gate_bias",
        "mlp1_weight_blocks": "mlp1_weight_blocks", "mlp1_weight_scales": "mlp1_weight_scales",
        "mlp1_bias": "mlp1_bias", "mlp2_weight_blocks": "mlp2_weight_blocks",
        "mlp2_weight_scales": "mlp2_weight_scales", "mlp2_bias": "mlp2_bias",
    }

    def named_parameters(self):
        for ref_name, attr in self.PARAM_NAMES.items():
            yield ref_name, getattr(self, attr)

    def load_state(self, params: dict) -> "MLPBlock":
        """Copy parameters in (reference names or attribute names; torch
        tensors or numpy arrays, bf16 given as uint16 bit patterns)."""
        import numpy as np
        for key, value in params.items():
            attr = self.PARAM_NAMES.get(key, key)
            dst = getattr(self, attr)
            if isinstance(value, np.ndarray):
                t = torch.from_numpy(np.ascontiguousarray(value))
                if dst.dtype == torch.bfloat16 and t.dtype in (torch.uint16, torch.int16):
                    t = t.view(torch.int16).view(torch.bfloat16)
                elif dst.dtype == torch.bfloat16 and value.dtype == np.uint16:
                    t = torch.from_numpy(np.ascontiguousarray(value).view(np.int16)).view(torch.bfloat16)
            else:
                t = value
            if tuple(t.shape) != tuple(dst.shape):
                raise ValueError(f"{key}: shape {tuple(t.shape)} != {tuple(dst.shape)}")
            dst.copy_(t.to(dst.dtype) if t.dtype != dst.dtype else t)
        return self.prepare()

    def prepare(self) -> "MLPBlock":
        """One-time weight check: enables the f16 GEMM path when every E8M0
        scale code lies in 104..140 (then e2m1 x 2^k is an exact f16)."""
        w = self.c_weights()
        w.flags = 0
        _lib.call("gptoss_moe_weights_prepare", ctypes.byref(w), _stream())
        self.flags = int(w.flags) if self.allow_f16 else 0
        return self

    @property
    def f16_path(self) -> bool:
        return bool(self.flags & _lib.MOE_F16)

    def c_weights(self) -> _lib.gptoss_moe_weights:
        w = _lib.gptoss_moe_weights()
        w.num_experts = self.num_experts
        w.num_local_experts = self.num_local_experts
        w.expert_offset = self.expert_offset
        w.hidden = self.hidden_size
        w.intermediate = self.intermediate_size
        w.top_k = self.experts_per_token
        w.swiglu_alpha = self.swiglu_alpha
        w.swiglu_limit = self.swiglu_limit
        w.rms_eps = self.rms_norm_eps
        for f in ("norm_weight", "gate_weight", "gate_bias"):
            setattr(w, f, getattr(self, f).data_ptr())
        w.mlp1_blocks = self.mlp1_weight_blocks.data_ptr()
        w.mlp1_scales = self.mlp1_weight_scales.data_ptr()
        w.mlp1_bias = self.mlp1_bias.data_ptr()
        w.mlp2_blocks = self.mlp2_weight_blocks.data_ptr()
        w.mlp2_scales = self.mlp2_weight_scales.data_ptr()
        w.mlp2_bias = self.mlp2_bias.data_ptr()
        w.flags = self.flags
        return w

    def share_workspace(self, owner: "MLPBlock") -> None:
        """Run on ``owner``'s scratch workspace.  The workspace holds no state
        between forwards, so the layers of a model (run one after another on
        one stream) can share one."""
        if owner is not self:
            self.free_workspace()
        self._ws_owner = owner

    def workspace(self, tokens: int):
        if self._ws_owner is not self:
            return self._ws_owner.workspace(tokens)
        if self._ws is None or tokens > self._ws_tokens:
            self.free_workspace()
            n = max(tokens, 1)
            ws = _lib.load().gptoss_moe_workspace_create(n, self.num_experts, self.experts_per_token,
                                                         self.hidden_size, self.intermediate_size)
            if not ws:
                raise _lib.GptossError(_lib.load().gptoss_last_error().decode())
            self._ws, self._ws_tokens = ws, n
        return self._ws

    def free_workspace(self):
        if self._ws is not None:
            _lib.load().gptoss_moe_workspace_destroy(self._ws)
            self._ws = None
            self._ws_tokens = 0

    def __del__(self):
        try:
            self.free_workspace()
        except Exception:
            pass

    def device_error(self) -> int:
        o = self._ws_owner
        return int(_lib.load().gptoss_moe_workspace_error(o._ws)) if o._ws is not None else 0

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x: [b, s, hidden] (or [tokens, hidden]) bf16 CUDA -> x + MoE(norm(x))."""
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise TypeError("MLPBlock.forward expects a bf16 CUDA tensor")
        shape = x.shape
        x2 = x.reshape(-1, self.hidden_size).contiguous()
        M = x2.shape[0]
        if out is None:
            out = torch.empty_like(x2)
        ws = self.workspace(M)
        w = self.c_weights()
        _lib.call("gptoss_moe_forward", _ptr(x2), M, ctypes.byref(w), ws, _ptr(out), _stream())
        return out.reshape(shape)

    __call__ = forward


def _events(n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def profile_moe_stages(blk: "MLPBlock", x: torch.Tensor, repeats: int = 3, flush: torch.Tensor | None = None) -> dict:
    """Times each stage of the block (same kernels as forward, called one by
    one through the C ABI) with CUDA events on the current stream.  `flush`
    (a device buffer larger than L2) is overwritten before every repeat."""
    x2 = x.reshape(-1, blk.hidden_size).contiguous()
    M = x2.shape[0]
    E, El, k, H, I = blk.num_experts, blk.num_local_experts, blk.experts_per_token, blk.hidden_size, blk.intermediate_size
    R = M * k
    dev = x2.device
    f16 = 1 if blk.f16_path else 0
    i32 = dict(dtype=torch.int32, device=dev)
    t = torch.empty_like(x2)
    logits = torch.empty(M, E, dtype=torch.bfloat16, device=dev)
    w = torch.empty(M, k, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(M, k, **i32)
    indptr, tile_ptr, tile_rows = torch.empty(E + 1, **i32), torch.empty(E + 1, **i32), torch.empty(E, **i32)
    tok, rev, exr = torch.empty(R, **i32), torch.empty(R, **i32), torch.empty(R, **i32)
    act = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
    y = torch.empty(R, I, dtype=torch.bfloat16, device=dev)
    h2 = torch.empty(R, H, dtype=torch.float32, device=dev)
    out = torch.empty_like(x2)
    err = torch.zeros(4, **i32)
    S = _stream()
    wts = blk.c_weights()
    mx = bool(_lib.load().gptoss_moe_uses_block_scaled(M, ctypes.byref(wts)))
    if mx:  # block-scaled decode GEMMs: e4m3 activation terms and their exponents
        q = torch.empty(R, 2 * max(H, I), dtype=torch.uint8, device=dev)
        qs = torch.empty(R, 192, dtype=torch.uint8, device=dev)
        y = torch.empty(R, I, dtype=torch.float16, device=dev)
    names = ["norm", "router", "permute", "gather", "mlp1", "quant2", "mlp2", "combine"]
    best = None
    for _ in range(repeats):
        if flush is not None:
            flush.zero_()
        ev = _events(len(names) + 1)
        ev[0].record()
        _lib.call("gptoss_rms_norm", _ptr(x2), _ptr(blk.norm_weight), M, H, ctypes.c_float(blk.rms_norm_eps), _ptr(t), S)
        ev[1].record()
        _lib.call("gptoss_moe_router", _ptr(t), _ptr(blk.gate_weight), _ptr(blk.gate_bias), M, E, H, k, _ptr(logits),
                  _ptr(w), _ptr(idx), _ptr(err), S)
        ev[2].record()
        _lib.call("gptoss_moe_permute", _ptr(idx), M, k, E, _ptr(indptr), _ptr(tok), _ptr(rev), _ptr(exr),
                  _ptr(tile_ptr), _ptr(tile_rows), _ptr(err), S)
        ev[3].record()
        if mx:
            _lib.call("gptoss_moe_quantize_mx", _ptr(t), 0, _ptr(tok), R, H, _ptr(q), _ptr(qs), S)
            ev[4].record()
            _lib.call("gptoss_moe_mlp1_mx", _ptr(q), _ptr(qs), R, _ptr(indptr), _ptr(tile_ptr), _ptr(tile_rows), E, H,
                      I, _ptr(blk.mlp1_weight_blocks), _ptr(blk.mlp1_weight_scales), _ptr(blk.mlp1_bias),
                      ctypes.c_float(blk.swiglu_alpha), ctypes.c_float(blk.swiglu_limit), _ptr(y), _ptr(err), S)
            ev[5].record()
            _lib.call("gptoss_moe_quantize_mx", _ptr(y), 1, None, R, I, _ptr(q), _ptr(qs), S)
            ev[6].record()
            _lib.call("gptoss_moe_mlp2_mx", _ptr(q), _ptr(qs), R, _ptr(indptr), _ptr(tile_ptr), _ptr(tile_rows), E, H,
                      I, _ptr(blk.mlp2_weight_blocks), _ptr(blk.mlp2_weight_scales), _ptr(blk.mlp2_bias), _ptr(h2),
                      _ptr(err), S)
        else:
            _lib.call("gptoss_moe_gather", _ptr(t), _ptr(tok), R, H, f16, _ptr(act), S)
            ev[4].record()
            _lib.call("gptoss_moe_mlp1", _ptr(act), R, _ptr(indptr), _ptr(tile_ptr), _ptr(tile_rows), E, H, I,
                      _ptr(blk.mlp1_weight_blocks), _ptr(blk.mlp1_weight_scales), _ptr(blk.mlp1_bias),
                      ctypes.c_float(blk.swiglu_alpha), ctypes.c_float(blk.swiglu_limit), f16, _ptr(y), _ptr(err), S)
            ev[5].record()
            ev[6].record()
            _lib.call("gptoss_moe_mlp2", _ptr(y), R, _ptr(indptr), _ptr(tile_ptr), _ptr(tile_rows), E, H, I,
                      _ptr(blk.mlp2_weight_blocks), _ptr(blk.mlp2_weight_scales), _ptr(blk.mlp2_bias), f16, _ptr(h2),
                      _ptr(err), S)
        ev[7].record()
        _lib.call("gptoss_moe_combine", _ptr(h2), _ptr(rev), _ptr(w), _ptr(x2), M, k, H, _ptr(out), S)
        ev[8].record()
        torch.cuda.synchronize()
        times = {f"{n}_ms": ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(names)}
        if best is None or times["mlp1_ms"] < best["mlp1_ms"]:
            best = times
    if int(err[0].item()) != 0:
        raise _lib.GptossError(f"device error word {int(err[0].item()):#x}")
    best["mlp1_flops"] = 2.0 * R * (2 * I) * H
    best["mlp2_flops"] = 2.0 * R * H * I
    best["gemm_flops"] = best["mlp1_flops"] + best["mlp2_flops"]
    best["gemm_ms"] = best["mlp1_ms"] + best["mlp2_ms"]
    best["total_ms"] = sum(best[f"{n}_ms"] for n in names)
    # norm, router, topk, count/scan, place, gather (or quantize), mlp1, [quantize,] mlp2, combine
    best["launches_per_step"] = 10 if mx else 9
    best["expert_path"] = "block-scaled (kind::mxf8f6f4)" if mx else "kind::f16 / decode GEMV"
    return best


MLPBlock.profile_stages = profile_moe_stages
