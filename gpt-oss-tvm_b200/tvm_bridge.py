"""The B200 MoE block as a TVM PackedFunc: ``gptoss.moe_forward``.

The reference calls its kernels through TVM's destination-passing
convention -- the Relax VM hands DLTensors to a registered function and
passes the output buffer last (nn.tensor_ir_op / nn.op.extern,
model/mlp.py:321-326).  ``register()`` registers, in the TVM of the running
process, a global function with exactly MLPBlock.forward's inputs and a
destination tensor:

    gptoss.moe_forward(x, norm.weight, gate.weight, gate.bias,
                       mlp1_weight_blocks, mlp1_weight_scales, mlp1_bias,
                       mlp2_weight_blocks, mlp2_weight_scales, mlp2_bias, out)

so that the reference's MLPBlock.forward becomes one
``nn.op.extern("gptoss.moe_forward", [...], out=...)`` call.  Arguments may
be TVM runtime Tensors or any other DLPack producer on the current CUDA
device; the library checks element types, shapes, device and layout
(gptoss_moe_weights_init_dl, gptoss_moe_forward_dl) and the function raises
GptossError with the library's message on a mismatch.  Calls run on the
legacy default CUDA stream, the one the Relax VM uses.

The prepared weight view (gptoss_moe_weights, including the f16-path check)
is cached per set of parameter tensors (their device addresses and shapes);
a workspace is kept per expert count and grown to the largest token count
seen.
"""
from __future__ import annotations

import ctypes

from . import _lib

FUNC_NAME = "gptoss.moe_forward"

_weights: dict = {}
_workspaces: dict = {}


def _check(rc: int) -> None:
    _lib.check(rc)


def moe_forward(x, norm_weight, gate_weight, gate_bias, mlp1_blocks, mlp1_scales, mlp1_bias, mlp2_blocks,
                mlp2_scales, mlp2_bias, out, top_k: int = 4, swiglu_limit: float = 7.0, rms_eps: float = 1e-5,
                stream=None):
    """out = x + MoE(RMSNorm(x)) for DLPack tensors (MLPBlock.forward,
    model/mlp.py:371-402); returns ``out``."""
    lib = _lib.load()
    params = [_lib.DLArg(t) for t in (norm_weight, gate_weight, gate_bias, mlp1_blocks, mlp1_scales, mlp1_bias,
                                      mlp2_blocks, mlp2_scales, mlp2_bias)]
    key = tuple((p.address, p.shape) for p in params) + (top_k, swiglu_limit, rms_eps)
    w = _weights.get(key)
    if w is None:
        w = _lib.gptoss_moe_weights()
        _check(lib.gptoss_moe_weights_init_dl(ctypes.byref(w), *params, top_k, ctypes.c_float(swiglu_limit),
                                              ctypes.c_float(rms_eps), 0, stream))
        _weights[key] = w
    xa, oa = _lib.DLArg(x), _lib.DLArg(out)
    M = 1
    for d in xa.shape[:-1]:
        M *= d
    wkey = (w.num_experts, w.top_k, w.hidden, w.intermediate)
    ws, cap = _workspaces.get(wkey, (None, 0))
    if ws is None or cap < max(M, 1):
        if ws is not None:
            lib.gptoss_moe_workspace_destroy(ws)
        cap = max(M, 1)
        ws = lib.gptoss_moe_workspace_create(cap, w.num_experts, w.top_k, w.hidden, w.intermediate)
        if not ws:
            raise _lib.GptossError(lib.gptoss_last_error().decode())
        _workspaces[wkey] = (ws, cap)
    _check(lib.gptoss_moe_forward_dl(xa, ctypes.byref(w), ctypes.c_void_p(ws), oa, stream))
    return out


def register(name: str = FUNC_NAME):
    """Registers ``moe_forward`` as the TVM global function ``name`` (needs an
    importable TVM with tvm.register_global_func, e.g. the one tilelang ships)."""
    import tvm

    def _packed(*args):
        moe_forward(*args)

    tvm.register_global_func(name, _packed, override=True)
    return tvm.get_global_func(name)


def release() -> None:
    """Frees the cached workspaces and forgets the prepared weight views."""
    lib = _lib.load()
    for ws, _ in _workspaces.values():
        lib.gptoss_moe_workspace_destroy(ws)
    _workspaces.clear()
    _weights.clear()
