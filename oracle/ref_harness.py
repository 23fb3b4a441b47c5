"""Harness that loads the REFERENCE model files through TVM Relax and
compiles them for the CPU with TVM's C target.

TEST / BASELINE INFRASTRUCTURE ONLY (used by tests/golden/make_golden.py and
oracle/make_ref.py in the development container; it needs the reference tree
and the TVM Relax build that ships inside the `tilelang` package).

The reference's own model code (model/config.py, model/mlp.py,
model/attention.py) is loaded unmodified.  Three fixes are applied around
TVM, none to reference code:
  1. bf16 numpy constants (nn.Tensor.from_const at model/mlp.py:265) are
     built through torch/DLPack because this tvm_ffi rejects numpy bf16;
  2. the generated C spells bf16 constants as *(uint32_t*)(&<float literal>),
     which gcc rejects; it is rewritten to a memcpy helper;
  3. the vendored tvm.contrib.sort.topk has no bf16 branch, so topk inputs
     are cast to fp32 and back (exact: bf16 -> fp32 is lossless).
The generated C is built with gcc -O2 -ffp-contract=off (the image's libtvm
has no LLVM backend; the generic llvm target would not contract FMAs either).
"""
from __future__ import annotations

import importlib.util
import os
import re
import sys
import tempfile
import types

import numpy as np


class RefHarness:
    """Loads the reference model files through TVM Relax (C target)."""

    def __init__(self, ref_root: str):
        import tilelang  # noqa: F401  (provides the TVM Relax build)
        import torch
        import tvm
        from tvm import relax
        from tvm.relax.frontend import nn

        self.torch, self.tvm, self.relax, self.nn = torch, tvm, relax, nn
        # empty stand-ins for the mlc_llm modules the reference imports at module scope
        m = types.ModuleType("mlc_llm")
        sup = types.ModuleType("mlc_llm.support")
        cfgm = types.ModuleType("mlc_llm.support.config")
        sty = types.ModuleType("mlc_llm.support.style")
        mnn = types.ModuleType("mlc_llm.nn")
        import logging as _lg
        slog = types.ModuleType("mlc_llm.support.logging")
        slog.getLogger = _lg.getLogger

        class ConfigBase:  # noqa: D401
            pass

        cfgm.ConfigBase = ConfigBase
        sty.bold = lambda s: s
        mnn.PagedKVCache = object
        sup.logging = slog
        sys.modules.update({"mlc_llm": m, "mlc_llm.support": sup, "mlc_llm.support.config": cfgm,
                            "mlc_llm.support.style": sty, "mlc_llm.nn": mnn, "mlc_llm.support.logging": slog})
        pkg = types.ModuleType("refmodel")
        pkg.__path__ = [os.path.join(ref_root, "model")]
        sys.modules["refmodel"] = pkg
        self.config = self._load("refmodel.config", os.path.join(ref_root, "model", "config.py"))
        self.mlp = self._load("refmodel.mlp", os.path.join(ref_root, "model", "mlp.py"))
        self.attention = self._load("refmodel.attention", os.path.join(ref_root, "model", "attention.py"))

        # fix 1: bf16 numpy constants via torch/DLPack
        import ml_dtypes
        import tvm.runtime._tensor as tmod
        orig = tmod.tensor

        def _tensor(arr, device=None, mem_scope=None):
            if isinstance(arr, np.ndarray) and arr.dtype == ml_dtypes.bfloat16:
                t = torch.empty(arr.shape, dtype=torch.bfloat16)
                t.view(torch.int16).copy_(torch.from_numpy(arr.view(np.int16).copy()))
                return tvm.runtime.from_dlpack(t)
            return orig(arr, device) if device is not None else orig(arr)

        tmod.tensor = _tensor
        tvm.runtime.tensor = _tensor
        # fix 3: topk through fp32
        orig_topk = nn.op.topk

        def _topk(x, k=1, axis=-1, ret_type="both", largest=True, dtype="int32", name="topk"):
            v, i = orig_topk(x.astype("float32"), k=k, axis=axis, ret_type=ret_type, largest=largest,
                             dtype=dtype, name=name)
            return v.astype(x.dtype), i

        nn.op.topk = _topk
        self.tmpdir = tempfile.mkdtemp(prefix="gptoss_golden_")

    def _load(self, name, path):
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        return mod

    def _fcompile(self):
        from tvm.contrib import cc as _cc

        def _fix(path):
            s = open(path).read()
            s = re.sub(r"\(\*\(uint32_t \*\)\(&\(([^()]*?)\)\)\)", r"__tvm_f2u(\1)", s)
            hdr = ("#include <string.h>\n#include <stdint.h>\n"
                   "static inline uint32_t __tvm_f2u(float f){uint32_t u; memcpy(&u,&f,4); return u;}\n")
            open(path, "w").write(hdr + s)

        def fcompile(output, objects, options=None, **kw):
            for o in objects:
                if o.endswith(".c"):
                    _fix(o)
            return _cc.create_shared(output, objects, options=(options or []) + ["-O2", "-ffp-contract=off"], **kw)

        fcompile.output_format = "so"
        return fcompile

    def compile(self, module, spec, tag, out_dir=None):
        """export_tvm -> tvm.compile(target c) -> gcc (fix 2) -> Relax VM."""
        mod, params = module.export_tvm(spec=spec)
        ex = self.tvm.compile(mod, target="c")
        so = os.path.join(out_dir or self.tmpdir, tag + ".so")
        ex.export_library(so, fcompile=self._fcompile())
        vm = self.relax.VirtualMachine(self.tvm.runtime.load_module(so), self.tvm.cpu())
        return vm, [n for n, _ in params]

    def compile_tir(self, funcs: dict, tag: str):
        """TIR prim_funcs {name: prim_func} -> C target -> gcc (fix 2) -> a
        runtime module whose functions are called by name."""
        mod = self.tvm.IRModule({n: f.with_attr("global_symbol", n) for n, f in funcs.items()})
        ex = self.tvm.compile(mod, target="c")
        so = os.path.join(self.tmpdir, tag + ".so")
        ex.export_library(so, fcompile=self._fcompile())
        return self.tvm.runtime.load_module(so)

    def patched_kv_cache(self, ref_root: str):
        """TVM's kv_cache.py (the attention kernels of the paged KV cache, from
        the TVM build bundled with tilelang) with the reference's own fix
        applied: the kv_cache.py section of tvm_fix.patch (the sliding-window
        predicate of the ragged prefill kernels), patched into a temporary
        copy with `patch -p1`.  Returns the patched module."""
        import shutil
        import subprocess

        import tvm.relax.frontend.nn.llm as llm
        rel = "python/tvm/relax/frontend/nn/llm/kv_cache.py"
        root = tempfile.mkdtemp(prefix="gptoss_kvcache_")
        os.makedirs(os.path.join(root, os.path.dirname(rel)))
        shutil.copy(os.path.join(os.path.dirname(llm.__file__), "kv_cache.py"), os.path.join(root, rel))
        text = open(os.path.join(ref_root, "tvm_fix.patch")).read()
        section = [p for p in re.split(r"(?m)^(?=diff --git )", text) if p.startswith("diff --git a/" + rel)]
        if len(section) != 1:
            raise RuntimeError("tvm_fix.patch has no kv_cache.py section")
        r = subprocess.run(["patch", "-p1", "-d", root], input=section[0], text=True, capture_output=True)
        if r.returncode != 0:
            raise RuntimeError(f"patch failed: {r.stdout} {r.stderr}")
        name = "tvm.relax.frontend.nn.llm._kv_cache_reference_patched"
        spec = importlib.util.spec_from_file_location(name, os.path.join(root, rel))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        self.patch_log = r.stdout.strip()
        return mod

    # numpy <-> tvm (bf16 carried as uint16 bits)
    def _aligned(self, a):
        # torch's CPU allocator returns 64-byte aligned storage, which DLPack import requires
        src = self.torch.from_numpy(np.ascontiguousarray(a).copy())
        dst = self.torch.empty(src.shape, dtype=src.dtype)
        dst.copy_(src)
        return dst

    def bf(self, bits):
        t = self._aligned(np.ascontiguousarray(bits).view(np.int16)).view(self.torch.bfloat16)
        return self.tvm.runtime.from_dlpack(t)

    def raw(self, a):
        return self.tvm.runtime.from_dlpack(self._aligned(a))

    def out(self, t):
        tt = self.torch.from_dlpack(t)
        if tt.dtype == self.torch.bfloat16:
            return tt.view(self.torch.int16).numpy().view(np.uint16).copy()
        return tt.numpy().copy()


