"""The DLTensor boundary on the GPU (include/gptoss_b200_dlpack.h).

MLPBlock.forward through gptoss_moe_weights_init_dl + gptoss_moe_forward_dl,
and through the TVM PackedFunc "gptoss.moe_forward" called with TVM runtime
Tensors (the bridge a maintainer registers in the reference, see the TVM
section of the integration notes), must equal the plain-pointer entry point
bit for bit; the attention entry points likewise.  Wrong element types,
shapes or layouts are refused with a message and launch nothing.
"""
import ctypes
import importlib

import numpy as np
import pytest

from conftest import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402

L = importlib.import_module("gpt-oss-tvm_b200._lib")


@pytest.fixture(scope="module")
def block():
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfg = importlib.import_module("gpt-oss-tvm_b200.config").GPTOssConfig(num_experts=32)
    blk = mlp.MLPBlock(cfg).load_state(synth().moe_params(32, seed=70))
    yield blk
    blk.free_workspace()


def _params(blk):
    return [blk.norm_weight, blk.gate_weight, blk.gate_bias, blk.mlp1_weight_blocks, blk.mlp1_weight_scales,
            blk.mlp1_bias, blk.mlp2_weight_blocks, blk.mlp2_weight_scales, blk.mlp2_bias]


@pytest.mark.parametrize("M", [1, 24, 300])
def test_moe_forward_dl_equals_pointer_entry_point(block, M):
    lib = L.load()
    x = G.dev(synth().activations(M, seed=71 + M)).reshape(1, M, 2880)
    ref = block.forward(x)
    w = L.gptoss_moe_weights()
    G.call("gptoss_moe_weights_init_dl", ctypes.byref(w), *[L.DLArg(t) for t in _params(block)], 4,
           ctypes.c_float(7.0), ctypes.c_float(1e-5), 0, G.S())
    assert w.flags == block.flags and w.num_experts == 32 and w.hidden == 2880
    out = torch.empty_like(x)
    G.call("gptoss_moe_forward_dl", L.DLArg(x), ctypes.byref(w), block.workspace(M), L.DLArg(out), G.S())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert lib.gptoss_moe_workspace_error(block.workspace(M)) == 0


def test_tvm_packed_func_bridge(block):
    """gptoss.moe_forward registered in tilelang's TVM and called with TVM
    runtime Tensors that alias the block's CUDA tensors."""
    pytest.importorskip("tilelang")
    import tvm
    bridge = importlib.import_module("gpt-oss-tvm_b200.tvm_bridge")
    f = bridge.register()
    M = 40
    x = G.dev(synth().activations(M, seed=99)).reshape(1, M, 2880)
    torch.cuda.synchronize()
    ref = block.forward(x)
    out = torch.zeros_like(x)
    tv = [tvm.runtime.from_dlpack(t) for t in [x, *_params(block), out]]
    torch.cuda.synchronize()
    f(*tv)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # the same function refuses a float32 input with the library's message
    xf = tvm.runtime.from_dlpack(x.float())
    with pytest.raises(Exception) as exc:
        f(xf, *tv[1:])
    assert "bfloat16" in str(exc.value)
    bridge.release()


def test_dl_rejects_wrong_types_shapes_and_layouts(block):
    lib = L.load()
    w = block.c_weights()
    ws = block.workspace(8)
    x = G.dev(synth().activations(8, seed=5))
    out = torch.empty_like(x)
    cases = [
        (x.float(), out, "bfloat16"),
        (x[:, :2048].contiguous(), out[:, :2048], "dimension 1 must be 2880"),
        (torch.empty(2880, 16, dtype=torch.bfloat16, device="cuda").t(), torch.empty(16, 2880, dtype=torch.bfloat16,
                                                                                     device="cuda"), "dense row-major"),
        (x, out[:4], "dimension 0 must be 8"),
        (x.cpu(), out, "CUDA device"),
    ]
    for xi, oi, msg in cases:
        rc = lib.gptoss_moe_forward_dl(L.DLArg(xi), ctypes.byref(w), ws, L.DLArg(oi), G.S())
        assert rc == -1, msg
        assert msg in lib.gptoss_last_error().decode(), (msg, lib.gptoss_last_error().decode())
    torch.cuda.synchronize()


@pytest.mark.parametrize("window", [0, 128])
def test_attention_dl_entry_points_equal_pointer_ones(window):
    S = synth()
    q, k, v, sinks = S.attention_inputs(200, seed=8)
    qd, kd, vd, sd = G.dev(q), G.dev(k), G.dev(v), G.dev(sinks)
    o1, o2 = torch.empty_like(qd), torch.empty_like(qd)
    l1 = torch.empty(200, 64, dtype=torch.float32, device="cuda")
    l2 = torch.empty_like(l1)
    G.call("gptoss_attn_prefill", G.P(qd), G.P(kd), G.P(vd), G.P(sd), 200, 200, 64, 8, 64, window,
           ctypes.c_float(0.125), G.P(o1), G.P(l1), G.S())
    # with a leading batch dimension of 1, as AttentionBlock holds them
    G.call("gptoss_attn_prefill_dl", L.DLArg(qd[None]), L.DLArg(kd[None]), L.DLArg(vd[None]), L.DLArg(sd), window,
           ctypes.c_float(0.125), L.DLArg(o2[None]), L.DLArg(l2[None]), G.S())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    B, Lmax = 3, 300
    rng = np.random.default_rng(9)
    qb = G.dev(S.normal_bf16(rng, (B, 64, 64), 1.0))
    kc = G.dev(S.normal_bf16(rng, (B, Lmax, 8, 64), 1.0))
    vc = G.dev(S.normal_bf16(rng, (B, Lmax, 8, 64), 1.0))
    lens = G.dev(np.array([1, 150, 300], np.int32))
    lib = L.load()
    nb = lib.gptoss_attn_decode_scratch_bytes(B, 64, Lmax, window)
    scratch = torch.empty(max(nb // 4, 1), dtype=torch.float32, device="cuda")
    d1, d2 = torch.empty_like(qb), torch.empty_like(qb)
    G.call("gptoss_attn_decode", G.P(qb), G.P(kc), G.P(vc), G.P(lens), B, Lmax, 64, 8, 64, window,
           ctypes.c_float(0.125), G.P(sd), G.P(scratch), nb, G.P(d1), None, G.S())
    G.call("gptoss_attn_decode_dl", L.DLArg(qb), L.DLArg(kc), L.DLArg(vc), L.DLArg(lens), window,
           ctypes.c_float(0.125), L.DLArg(sd), L.DLArg(scratch), L.DLArg(d2), None, G.S())
    torch.cuda.synchronize()
    assert torch.equal(d1, d2)
