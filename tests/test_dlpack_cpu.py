"""CPU checks of the DLTensor boundary (include/gptoss_b200_dlpack.h): DLPack
tensors from torch and from TVM are read correctly, the DLTensor entry points
reject tensors that are not on the current CUDA device (nothing is launched),
and the TVM bridge registers gptoss.moe_forward as a PackedFunc whose
argument errors surface as exceptions with the library's message."""
import ctypes
import importlib
import os

import numpy as np
import pytest

from conftest import REPO

LIB = os.path.join(REPO, "gpt-oss-tvm_b200", "libgptoss_b200.so")
pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="libgptoss_b200.so not built")

torch = pytest.importorskip("torch")
L = importlib.import_module("gpt-oss-tvm_b200._lib")


def test_dlarg_reads_torch_tensors():
    t = torch.arange(24, dtype=torch.float32).reshape(2, 3, 4)[:, 1:]
    a = L.DLArg(t)
    v = a.view
    assert a.shape == (2, 2, 4) and v.dtype_code == 2 and v.dtype_bits == 32 and v.dtype_lanes == 1
    assert a.address == t.data_ptr() and v.device_type == 1  # kDLCPU
    assert tuple(v.strides[i] for i in range(3)) == (12, 4, 1)
    b = L.DLArg(torch.zeros(5, dtype=torch.bfloat16))
    assert b.view.dtype_code == 4 and b.view.dtype_bits == 16  # kDLBfloat
    assert L.DLArg(None).ptr is None


def test_dlarg_reads_tvm_tensors():
    pytest.importorskip("tilelang")
    import tvm
    x = np.arange(12, dtype=np.int32).reshape(3, 4)
    # torch's CPU allocator aligns to 64 bytes, as TVM's from_dlpack requires; numpy's may not
    t = tvm.runtime.from_dlpack(torch.arange(12, dtype=torch.int32).reshape(3, 4))
    a = L.DLArg(t)
    assert a.shape == (3, 4) and a.view.dtype_code == 0 and a.view.dtype_bits == 32
    got = np.ctypeslib.as_array(ctypes.cast(ctypes.c_void_p(a.address), ctypes.POINTER(ctypes.c_int32)), (12,))
    np.testing.assert_array_equal(got, x.ravel())


def test_dl_entry_points_reject_host_tensors():
    lib = L.load()
    q = torch.zeros(4, 64, 64, dtype=torch.bfloat16)
    k = torch.zeros(4, 8, 64, dtype=torch.bfloat16)
    rc = lib.gptoss_attn_prefill_dl(L.DLArg(q), L.DLArg(k), L.DLArg(k), None, 0, ctypes.c_float(0.125),
                                    L.DLArg(q), None, None)
    assert rc == -1
    assert "CUDA device" in lib.gptoss_last_error().decode()
    w = L.gptoss_moe_weights()
    rc = lib.gptoss_moe_weights_init_dl(ctypes.byref(w), *([None] * 9), 4, ctypes.c_float(7.0),
                                        ctypes.c_float(1e-5), 0, None)
    assert rc == -1 and "gate_weight" in lib.gptoss_last_error().decode()


def test_tvm_bridge_registers_and_reports_argument_errors():
    pytest.importorskip("tilelang")
    import tvm
    bridge = importlib.import_module("gpt-oss-tvm_b200.tvm_bridge")
    f = bridge.register()
    assert tvm.get_global_func(bridge.FUNC_NAME) is not None
    E, H, I = 4, 64, 64
    mk = lambda *shape, dt=torch.bfloat16: tvm.runtime.from_dlpack(torch.zeros(*shape, dtype=dt))  # noqa: E731
    args = [mk(2, 3, H), mk(H), mk(E, H), mk(E), mk(E, 2 * I, H // 32, 16, dt=torch.uint8),
            mk(E, 2 * I, H // 32, dt=torch.uint8), mk(E, 2 * I), mk(E, H, I // 32, 16, dt=torch.uint8),
            mk(E, H, I // 32, dt=torch.uint8), mk(E, H), mk(2, 3, H)]
    with pytest.raises(Exception) as exc:
        f(*args)
    assert "CUDA device" in str(exc.value)
