"""Runs the reference MoE block compiled by TVM (oracle/_ref/) on the CPU.

BASELINE INFRASTRUCTURE ONLY.  oracle/_ref/moe_e{E}.so is the reference's
model/mlp.py MLPBlock lowered by TVM's C target (oracle/make_ref.py); it is
executed by the Relax VM of the TVM build inside `tilelang`, one process per
host core, each over its share of the token sample.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")


def so_path(num_experts: int) -> str:
    return os.path.join(REF_DIR, f"moe_e{num_experts}.so")


def available(num_experts: int) -> bool:
    if not os.path.exists(so_path(num_experts)):
        return False
    try:
        import importlib.util
        return importlib.util.find_spec("tilelang") is not None
    except Exception:
        return False


def _worker(args):
    num_experts, x_bits, wseed = args
    import importlib
    import sys
    sys.path.insert(0, os.path.dirname(HERE))
    import tilelang  # noqa: F401
    import torch
    import tvm
    from tvm import relax
    synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
    names = json.load(open(os.path.join(REF_DIR, f"moe_e{num_experts}.json")))
    p = synth.moe_params(num_experts, seed=wseed)
    key = {"norm.weight": "norm_weight", "gate.weight": "gate_weight", "gate.bias": "gate_bias"}

    def to_tvm(a):
        src = torch.from_numpy(np.ascontiguousarray(a).view(np.int16) if a.dtype == np.uint16 else np.ascontiguousarray(a))
        dst = torch.empty(src.shape, dtype=src.dtype)
        dst.copy_(src)
        if a.dtype == np.uint16:
            dst = dst.view(torch.bfloat16)
        return tvm.runtime.from_dlpack(dst)

    vals = [to_tvm(p[key.get(n, n)]) for n in names]
    vm = relax.VirtualMachine(tvm.runtime.load_module(so_path(num_experts)), tvm.cpu())
    M = x_bits.shape[0]
    xt = to_tvm(x_bits.reshape(1, M, -1))
    t0 = time.perf_counter()
    vm["forward"](xt, *vals)
    return time.perf_counter() - t0


def measure(tokens: int = 32, num_experts: int = 128, wseed: int = 0) -> dict:
    import importlib
    synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
    cores = len(os.sched_getaffinity(0))
    procs = max(1, min(cores, tokens))
    x = synth.activations(tokens, seed=1)
    shards = np.array_split(x, procs)
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(procs) as pool:
        per = pool.map(_worker, [(num_experts, s, wseed) for s in shards])
    wall = time.perf_counter() - t0
    # throughput of the compute itself: tokens over the slowest shard's forward
    dt = max(per)
    return {"value": tokens / dt, "unit": "tokens/s", "cores": procs, "kind": "reference",
            "sample": f"{tokens} tokens of the {num_experts}-expert MoE block: reference model/mlp.py compiled by "
                      f"TVM (C target), {procs} processes x {tokens // procs}-token shards",
            "seconds": dt, "wall_seconds_incl_setup": wall}
