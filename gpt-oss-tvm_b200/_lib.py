"""ctypes binding of libgptoss_b200.so (the C ABI in include/gptoss_b200.h).

The product path has no CPU fallback: loading fails loudly when the library
is missing, and every call raises GptossError when the C ABI reports an
error.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("GPTOSS_B200_LIB", os.path.join(HERE, "libgptoss_b200.so"))


class GptossError(RuntimeError):
    pass


class gptoss_moe_weights(ctypes.Structure):
    _fields_ = [
        ("num_experts", ctypes.c_int32), ("num_local_experts", ctypes.c_int32), ("expert_offset", ctypes.c_int32),
        ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("swiglu_alpha", ctypes.c_float), ("swiglu_limit", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("norm_weight", ctypes.c_void_p), ("gate_weight", ctypes.c_void_p), ("gate_bias", ctypes.c_void_p),
        ("mlp1_blocks", ctypes.c_void_p), ("mlp1_scales", ctypes.c_void_p), ("mlp1_bias", ctypes.c_void_p),
        ("mlp2_blocks", ctypes.c_void_p), ("mlp2_scales", ctypes.c_void_p), ("mlp2_bias", ctypes.c_void_p),
        ("flags", ctypes.c_uint32),
    ]


MOE_F16 = 1  # GPTOSS_MOE_F16


_P, _I64, _I32, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float

# name -> (restype, argtypes); mirrors include/gptoss_b200.h
SIGNATURES = {
    "gptoss_version": (ctypes.c_int, []),
    "gptoss_last_error": (ctypes.c_char_p, []),
    "gptoss_moe_workspace_create": (_P, [_I64, _I32, _I32, _I32, _I32]),
    "gptoss_moe_workspace_destroy": (None, [_P]),
    "gptoss_moe_workspace_error": (ctypes.c_uint32, [_P]),
    "gptoss_moe_forward": (ctypes.c_int, [_P, _I64, ctypes.POINTER(gptoss_moe_weights), _P, _P, _P]),
    "gptoss_rms_norm": (ctypes.c_int, [_P, _P, _I64, _I32, _F, _P, _P]),
    "gptoss_moe_router": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P]),
    "gptoss_moe_topk_softmax": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _P, _P, _P]),
    "gptoss_moe_permute": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gptoss_moe_route": (ctypes.c_int, [_P, _I64, ctypes.POINTER(gptoss_moe_weights), _P, _P, _P, _P, _P, _P, _P, _P,
                                         _P, _P, _P]),
    "gptoss_moe_gather": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _P, _P]),
    "gptoss_moe_mlp1": (ctypes.c_int, [_P, _I64, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _F, _F, _I32, _P, _P, _P]),
    "gptoss_moe_mlp2": (ctypes.c_int, [_P, _I64, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _P, _P]),
    "gptoss_moe_quantize_mx": (ctypes.c_int, [_P, _I32, _P, _I64, _I32, _P, _P, _P]),
    "gptoss_moe_mlp1_mx": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _F, _F, _P, _P,
                                          _P]),
    "gptoss_moe_mlp2_mx": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P]),
    "gptoss_moe_uses_block_scaled": (ctypes.c_int, [_I64, ctypes.POINTER(gptoss_moe_weights)]),
    "gptoss_moe_weights_prepare": (ctypes.c_int, [ctypes.POINTER(gptoss_moe_weights), _P]),
    "gptoss_moe_combine": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I32, _P, _P]),
    "gptoss_moe_combine_bf16": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I32, _P, _P]),
    "gptoss_mxfp4_dequant": (ctypes.c_int, [_P, _P, _I64, _I32, _P, _P]),
    "gptoss_moe_forward_noalloc": (ctypes.c_int, [_P, _I64, ctypes.POINTER(gptoss_moe_weights), _P, _P]),
    "gptoss_moe_noalloc_error": (ctypes.c_uint32, []),
    "gptoss_yarn_inv_freq": (ctypes.c_int, [_I32, _F, _F, _F, _F, _I32, _P, _P]),
    "gptoss_rope_yarn": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _P, _F, _P, _P]),
    "gptoss_qkv_rope_append": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _I32, _P, _F, _P, _P, _P, _P]),
    "gptoss_attn_prefill": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I32, _I32, _I32, _I32, _F, _P, _P, _P]),
    "gptoss_attn_decode_scratch_bytes": (ctypes.c_int64, [_I64, _I32, _I64, _I32]),
    "gptoss_attn_decode": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _I32, _I32, _I32, _I32, _F, _P, _P, _I64, _P,
                                          _P, _P]),
    "gptoss_attn_decode_paged": (ctypes.c_int, [_P, _P, _P, _P, _I32, _P, _I64, _I32, _I32, _I32, _I32, _F, _P, _P,
                                                _I64, _P, _P, _P]),
    "gptoss_kv_pages_copy": (ctypes.c_int, [_P, _P, _I32, _I32, _P, _I32, _I32, _I64, _I64, _P, _P, _I32, _P]),
    "gptoss_attn_merge": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I32, _P, _P, _P]),
    "gptoss_attn_sink_rescale": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _P]),
    "gptoss_moe_plan_tiles": (ctypes.c_int, [_P, _I32, _P, _P, _P]),
    "gptoss_moe_segment_copy": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I64, _I32, _P, _P]),
    "gptoss_stream_set_flag": (ctypes.c_int, [_P, ctypes.c_uint32, _P]),
    "gptoss_stream_wait_flag": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint32, _P, _P]),
    "gptoss_ipc_alloc": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(_P), _P]),
    "gptoss_ipc_open": (ctypes.c_int, [_P, ctypes.POINTER(_P)]),
    "gptoss_ipc_close": (ctypes.c_int, [_P]),
    "gptoss_ipc_free": (ctypes.c_int, [_P]),
    "gptoss_moe_peer_layout": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _P, _P]),
    "gptoss_moe_dispatch_peer": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _I32, _I64,
                                                _I32, _P]),
    "gptoss_moe_mlp2_peer": (ctypes.c_int, [_P, _I64, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _P, _I32,
                                            _I64, _I32, _P, _P]),
    "gptoss_moe_weights_init_dl": (ctypes.c_int, [ctypes.POINTER(gptoss_moe_weights), _P, _P, _P, _P, _P, _P, _P, _P,
                                                  _P, _I32, _F, _F, _I32, _P]),
    "gptoss_moe_forward_dl": (ctypes.c_int, [_P, ctypes.POINTER(gptoss_moe_weights), _P, _P, _P]),
    "gptoss_attn_prefill_dl": (ctypes.c_int, [_P, _P, _P, _P, _I32, _F, _P, _P, _P]),
    "gptoss_attn_decode_dl": (ctypes.c_int, [_P, _P, _P, _P, _I32, _F, _P, _P, _P, _P, _P]),
    "gptoss_ep_unique_id": (ctypes.c_int, [_P]),
    "gptoss_ep_init": (_P, [_P, _I32, _I32, _I64, _I32, _I32, _I32, _I32, _I32, _P]),
    "gptoss_ep_dispatch": (ctypes.c_int, [_P, _P, _I64, ctypes.POINTER(gptoss_moe_weights), _P]),
    "gptoss_ep_combine": (ctypes.c_int, [_P, _P, _I64, ctypes.POINTER(gptoss_moe_weights), _P, _P]),
    "gptoss_ep_forward": (ctypes.c_int, [_P, _P, _I64, ctypes.POINTER(gptoss_moe_weights), _P, _P]),
    "gptoss_ep_error": (ctypes.c_uint32, [_P]),
    "gptoss_ep_destroy": (None, [_P]),
    "gptoss_dense_gemv_max_tokens": (ctypes.c_int, []),
    "gptoss_dense_gemv": (ctypes.c_int, [_P, _I64, _P, _P, _I32, _I32, _P, _P]),
    "gptoss_dense_gemm": (ctypes.c_int, [_P, _I64, _P, _P, _I32, _I32, _P, _P, _P]),
    "gptoss_sample_top_p_scratch_bytes": (_I64, [_I64, _I64]),
    "gptoss_sample_top_p_from_logits": (ctypes.c_int, [_P, _I64, _I64, ctypes.c_double, ctypes.c_double, _P,
                                                        ctypes.c_double, _P, _I64, _P, _P]),
}

_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the CUDA library (raises if it was not built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise GptossError(f"libgptoss_b200.so not found at {p}; build it with __graft_entry__.build()")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


_capsule_ptr = ctypes.pythonapi.PyCapsule_GetPointer
_capsule_ptr.restype = ctypes.c_void_p
_capsule_ptr.argtypes = [ctypes.py_object, ctypes.c_char_p]
_capsule_valid = ctypes.pythonapi.PyCapsule_IsValid
_capsule_valid.restype = ctypes.c_int
_capsule_valid.argtypes = [ctypes.py_object, ctypes.c_char_p]
# DLManagedTensorVersioned: DLPackVersion (8 bytes), manager_ctx, deleter, flags, then the DLTensor
_VERSIONED_DLTENSOR_OFFSET = 32


class DLTensorView(ctypes.Structure):
    """The leading fields of DLPack's DLTensor (read-only view)."""
    _fields_ = [("data", ctypes.c_void_p), ("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32),
                ("ndim", ctypes.c_int32), ("dtype_code", ctypes.c_uint8), ("dtype_bits", ctypes.c_uint8),
                ("dtype_lanes", ctypes.c_uint16), ("shape", ctypes.POINTER(ctypes.c_int64)),
                ("strides", ctypes.POINTER(ctypes.c_int64)), ("byte_offset", ctypes.c_uint64)]


class DLArg:
    """A DLTensor* for the *_dl entry points from any DLPack producer (a torch
    tensor, a TVM runtime Tensor, a DLPack capsule); holds the capsule (and
    with it the producer's tensor) alive while the object lives.  None gives
    a NULL pointer."""

    def __init__(self, obj):
        self.capsule = None
        self.ptr = None
        if obj is None:
            return
        cap = obj
        if type(obj).__name__ != "PyCapsule":
            try:
                import torch
                if isinstance(obj, torch.Tensor):
                    cap = torch.utils.dlpack.to_dlpack(obj)
                else:
                    cap = obj.__dlpack__()
            except ImportError:
                cap = obj.__dlpack__()
        if _capsule_valid(cap, b"dltensor"):
            self.ptr = _capsule_ptr(cap, b"dltensor")
        elif _capsule_valid(cap, b"dltensor_versioned"):
            self.ptr = _capsule_ptr(cap, b"dltensor_versioned") + _VERSIONED_DLTENSOR_OFFSET
        else:
            raise GptossError("not a DLPack tensor (no unconsumed dltensor capsule)")
        self.capsule = cap

    @property
    def _as_parameter_(self):
        return ctypes.c_void_p(self.ptr)

    @property
    def view(self) -> DLTensorView:
        return DLTensorView.from_address(self.ptr)

    @property
    def shape(self) -> tuple:
        v = self.view
        return tuple(v.shape[i] for i in range(v.ndim))

    @property
    def address(self) -> int:
        v = self.view
        return (v.data or 0) + v.byte_offset


_dense_max = None


def dense_max_tokens() -> int:
    """Token rows up to which gptoss_dense_gemv runs (cached)."""
    global _dense_max
    if _dense_max is None:
        _dense_max = int(load().gptoss_dense_gemv_max_tokens())
    return _dense_max


def check(rc: int) -> None:
    if rc != 0:
        msg = load().gptoss_last_error()
        raise GptossError(f"gptoss call failed ({rc}): {msg.decode() if msg else ''}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
