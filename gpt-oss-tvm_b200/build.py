"""Build libgptoss_b200.so in-tree with nvcc for sm_100a.

The library is compiled from gpt-oss-tvm_b200/csrc/*.cu into one shared
object next to this file, so that it travels with the source tree.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libgptoss_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared",
         "-Xptxas", "-warn-spills"]


def dlpack_include() -> str:
    """A directory holding dlpack/dlpack.h (the DLPack C ABI of the DLTensor
    entry points): the copy that ships with tvm_ffi (the runtime of the TVM
    that runs the reference), else any installed package's copy."""
    import importlib.util
    cands = []
    for mod in ("tvm_ffi", "xgrammar"):
        spec = importlib.util.find_spec(mod)
        if spec and spec.submodule_search_locations:
            cands.append(os.path.join(list(spec.submodule_search_locations)[0], "include"))
    env = os.environ.get("DLPACK_INCLUDE")
    if env:
        cands.insert(0, env)
    for d in cands:
        if os.path.exists(os.path.join(d, "dlpack", "dlpack.h")):
            return d
    raise RuntimeError("dlpack/dlpack.h not found (set DLPACK_INCLUDE to the directory that holds dlpack/)")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return (sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + sorted(glob.glob(os.path.join(CSRC, "*.h")))
            + sorted(glob.glob(os.path.join(os.path.dirname(HERE), "include", "*.h"))))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in deps() if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *ARCH, *FLAGS, "-I", os.path.join(os.path.dirname(HERE), "include"), "-I", dlpack_include(),
           *sources(), "-o", LIB,
           "-lcuda" if False else "-lcudart"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
