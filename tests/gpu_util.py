"""Helpers for the GPU parity tests: numpy (bf16 as uint16 bits) <-> torch CUDA,
and direct C-ABI calls."""
import ctypes
import importlib

import numpy as np
import torch

_lib = importlib.import_module("gpt-oss-tvm_b200._lib")


def dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(a).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def S():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def call(name, *args):
    _lib.call(name, *args)


def tol_check(got, ref, max_rel=2e-2, min_cos=0.9995, what=""):
    """The bf16 tolerance of the expert and attention outputs:
    max|got-ref| / max|ref| <= 2e-2 and cosine(got, ref) >= 0.9995."""
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    assert np.all(np.isfinite(g)), f"{what}: non-finite output"
    rel = np.max(np.abs(g - r)) / max(np.max(np.abs(r)), 1e-30)
    cos = float(np.dot(g, r) / max(np.linalg.norm(g) * np.linalg.norm(r), 1e-30))
    assert rel <= max_rel and cos >= min_cos, f"{what}: max rel err {rel:.3e} (<= {max_rel}), cosine {cos:.6f} (>= {min_cos})"
    return rel, cos


class MoEPieces:
    """Runs the MoE block step by step through the C ABI (device buffers
    allocated here with torch) so each stage can be compared with the oracle."""

    def __init__(self, p: dict, k: int = 4, f16: bool | None = None, mx: bool | None = False):
        """f16: GEMM path (None = what gptoss_moe_weights_prepare allows);
        mx: the block-scaled decode GEMMs (activations quantized into two e4m3
        terms; y is f16 on that path); None = the expert path that
        gptoss_moe_forward takes for the same token count
        (gptoss_moe_uses_block_scaled)."""
        self.mx = mx
        self.p = {kk: dev(v) for kk, v in p.items()}
        self.E = p["gate_weight"].shape[0]
        self.H = p["gate_weight"].shape[1]
        self.I = p["mlp2_weight_blocks"].shape[2] * 32
        self.k = k
        self.err = torch.zeros(4, dtype=torch.int32, device="cuda")
        w = _lib.gptoss_moe_weights()
        w.num_experts = w.num_local_experts = self.E
        w.hidden, w.intermediate, w.top_k = self.H, self.I, k
        w.norm_weight = self.p["norm_weight"].data_ptr()
        w.mlp1_scales = self.p["mlp1_weight_scales"].data_ptr()
        w.mlp2_scales = self.p["mlp2_weight_scales"].data_ptr()
        w.mlp1_blocks = self.p["mlp1_weight_blocks"].data_ptr()
        w.mlp2_blocks = self.p["mlp2_weight_blocks"].data_ptr()
        call("gptoss_moe_weights_prepare", ctypes.byref(w), S())
        allowed = bool(w.flags & _lib.MOE_F16)
        self.f16 = allowed if f16 is None else (f16 and allowed)
        self.w = w

    def run(self, x_bits: np.ndarray, routing=None):
        """routing: optional (weights bf16 bits [M,k], indices int32 [M,k])
        that replaces the router output (exercises chosen expert loads)."""
        E, H, I, k = self.E, self.H, self.I, self.k
        x = dev(x_bits)
        M = x.shape[0]
        R = M * k
        mx = self.mx
        if mx is None:
            mx = bool(_lib.load().gptoss_moe_uses_block_scaled(M, ctypes.byref(self.w)))
        i32 = dict(dtype=torch.int32, device="cuda")
        t = torch.empty_like(x)
        logits = torch.empty(M, E, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(M, k, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(M, k, **i32)
        indptr = torch.empty(E + 1, **i32)
        tile_ptr = torch.empty(E + 1, **i32)
        tile_rows = torch.empty(E, **i32)
        tok = torch.empty(R, **i32)
        rev = torch.empty(R, **i32)
        exp_ = torch.empty(R, **i32)
        adt = torch.float16 if self.f16 else torch.bfloat16
        act = torch.empty(R, H, dtype=adt, device="cuda")
        y = torch.empty(R, I, dtype=adt, device="cuda")
        f16 = 1 if self.f16 else 0
        h2 = torch.empty(R, H, dtype=torch.float32, device="cuda")
        out = torch.empty_like(x)
        p = self.p
        call("gptoss_rms_norm", P(x), P(p["norm_weight"]), M, H, ctypes.c_float(1e-5), P(t), S())
        call("gptoss_moe_router", P(t), P(p["gate_weight"]), P(p["gate_bias"]), M, E, H, k, P(logits), P(w), P(idx),
             P(self.err), S())
        if routing is not None:
            w.copy_(dev(routing[0]))
            idx.copy_(dev(routing[1]))
        call("gptoss_moe_permute", P(idx), M, k, E, P(indptr), P(tok), P(rev), P(exp_), P(tile_ptr), P(tile_rows),
             P(self.err), S())
        if mx:
            y = torch.empty(R, I, dtype=torch.float16, device="cuda")
            q = torch.empty(R, 2 * max(H, I), dtype=torch.uint8, device="cuda")
            qs = torch.zeros(R, 192, dtype=torch.uint8, device="cuda")
            call("gptoss_moe_quantize_mx", P(t), 0, P(tok), R, H, P(q), P(qs), S())
            call("gptoss_moe_mlp1_mx", P(q), P(qs), R, P(indptr), P(tile_ptr), P(tile_rows), E, H, I,
                 P(p["mlp1_weight_blocks"]), P(p["mlp1_weight_scales"]), P(p["mlp1_bias"]), ctypes.c_float(1.702),
                 ctypes.c_float(7.0), P(y), P(self.err), S())
            call("gptoss_moe_quantize_mx", P(y), 1, None, R, I, P(q), P(qs), S())
            call("gptoss_moe_mlp2_mx", P(q), P(qs), R, P(indptr), P(tile_ptr), P(tile_rows), E, H, I,
                 P(p["mlp2_weight_blocks"]), P(p["mlp2_weight_scales"]), P(p["mlp2_bias"]), P(h2), P(self.err), S())
        else:
            call("gptoss_moe_gather", P(t), P(tok), R, H, f16, P(act), S())
            call("gptoss_moe_mlp1", P(act), R, P(indptr), P(tile_ptr), P(tile_rows), E, H, I,
                 P(p["mlp1_weight_blocks"]), P(p["mlp1_weight_scales"]), P(p["mlp1_bias"]), ctypes.c_float(1.702),
                 ctypes.c_float(7.0), f16, P(y), P(self.err), S())
            call("gptoss_moe_mlp2", P(y), R, P(indptr), P(tile_ptr), P(tile_rows), E, H, I,
                 P(p["mlp2_weight_blocks"]), P(p["mlp2_weight_scales"]), P(p["mlp2_bias"]), f16, P(h2), P(self.err),
                 S())
        call("gptoss_moe_combine", P(h2), P(rev), P(w), P(x), M, k, H, P(out), S())
        torch.cuda.synchronize()
        assert int(self.err.cpu()[0]) == 0, f"device error word {int(self.err.cpu()[0]):#x}"
        y_f32 = y.float().cpu().numpy()
        return dict(t=host(t), logits=host(logits), weights=host(w), indices=host(idx), indptr=host(indptr),
                    token_of_row=host(tok), row_of_pair=host(rev), expert_of_row=host(exp_), y=y_f32, h2=host(h2),
                    out=host(out), tile_ptr=host(tile_ptr), tile_rows=host(tile_rows))
