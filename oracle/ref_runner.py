"""Runs the reference MoE block compiled by TVM (oracle/_ref/) on the CPU.

BASELINE INFRASTRUCTURE ONLY.  oracle/_ref/moe_e{E}.so is the reference's
model/mlp.py MLPBlock lowered by TVM's C target (oracle/make_ref.py); it is
executed by the Relax VM of the TVM build inside `tilelang`.  The generated
code is single-threaded, so the baseline uses one worker process per host
core, each running the block over its share of the token sample.  The
weights are generated once and shared with the workers through /dev/shm.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
_WORKER = {}


def so_path(num_experts: int) -> str:
    return os.path.join(REF_DIR, f"moe_e{num_experts}.so")


def available(num_experts: int) -> bool:
    if not os.path.exists(so_path(num_experts)):
        return False
    import importlib.util
    return importlib.util.find_spec("tilelang") is not None


def _init(num_experts, shm_dir, repo):
    import sys
    sys.path.insert(0, repo)
    import tilelang  # noqa: F401  (TVM Relax runtime)
    import torch
    import tvm
    from tvm import relax
    names = json.load(open(os.path.join(REF_DIR, f"moe_e{num_experts}.json")))
    key = {"norm.weight": "norm_weight", "gate.weight": "gate_weight", "gate.bias": "gate_bias"}

    def to_tvm(a):
        t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)
        if t.data_ptr() % 64:
            t = t.clone()
        if a.dtype == np.uint16:
            t = t.view(torch.bfloat16)
        return tvm.runtime.from_dlpack(t)

    arrays = {n: np.load(os.path.join(shm_dir, f"{key.get(n, n)}.npy"), mmap_mode="r+") for n in names}
    _WORKER["vals"] = [to_tvm(arrays[n]) for n in names]
    _WORKER["arrays"] = arrays
    _WORKER["vm"] = relax.VirtualMachine(tvm.runtime.load_module(so_path(num_experts)), tvm.cpu())
    _WORKER["to_tvm"] = to_tvm


def _forward(x_bits):
    to_tvm = _WORKER["to_tvm"]
    M = x_bits.shape[0]
    xt = to_tvm(np.ascontiguousarray(x_bits.reshape(1, M, -1)))
    t0 = time.perf_counter()
    _WORKER["vm"]["forward"](xt, *_WORKER["vals"])
    return time.perf_counter() - t0


class RefPool:
    """One worker per core, each holding the compiled reference block."""

    def __init__(self, num_experts: int = 128, procs: int | None = None, wseed: int = 0):
        import importlib
        synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
        self.num_experts = num_experts
        self.procs = procs or len(os.sched_getaffinity(0))
        base = "/dev/shm" if os.path.isdir("/dev/shm") else None
        self.shm = tempfile.mkdtemp(prefix="gptoss_ref_", dir=base)
        for k, v in synth.moe_params(num_experts, seed=wseed).items():
            np.save(os.path.join(self.shm, f"{k}.npy"), v)
        ctx = mp.get_context("spawn")
        repo = os.path.dirname(HERE)
        self.pool = ctx.Pool(self.procs, initializer=_init, initargs=(num_experts, self.shm, repo))
        self.synth = synth

    def step(self, tokens_per_proc: int = 1, seed: int = 1) -> tuple[float, int]:
        """One forward of procs x tokens_per_proc tokens; returns (seconds of
        the slowest shard, tokens)."""
        n = self.procs * tokens_per_proc
        x = self.synth.activations(n, seed=seed)
        per = self.pool.map(_forward, np.array_split(x, self.procs))
        return max(per), n

    def close(self):
        self.pool.close()
        self.pool.join()
        import shutil
        shutil.rmtree(self.shm, ignore_errors=True)


TOKENS_PER_PROC = 2  # token rows each worker runs per step (both CPU measurements use it)


def measure_pool(pool: "RefPool", steps: int | None = None, seconds: float | None = None,
                 tokens_per_proc: int = TOKENS_PER_PROC) -> dict:
    """Times `pool` the one way both CPU measurements use: steps of
    procs x tokens_per_proc tokens (each step's time is its slowest shard),
    either a fixed number of steps or until `seconds` have been measured.
    Returns tokens/s over everything measured, with the sample described."""
    tot_t, tot_n, k = 0.0, 0, 0
    while (steps is not None and k < steps) or (steps is None and tot_t < (seconds or 10.0)):
        dt, n = pool.step(tokens_per_proc, seed=1 + k)
        tot_t += dt
        tot_n += n
        k += 1
    return {"value": tot_n / tot_t, "unit": "tokens/s", "cores": pool.procs, "kind": "reference",
            "extrapolated_from_tokens": tot_n, "measured_seconds": round(tot_t, 3), "measured_steps": k,
            "sample": f"{k} steps of {pool.procs} processes x {tokens_per_proc} tokens of the {pool.num_experts}-expert "
                      f"MoE block: the reference's model/mlp.py compiled by TVM (C target), one process per core; "
                      f"tokens/s = tokens measured / seconds measured"}


def measure(seconds: float = 10.0, num_experts: int = 128, wseed: int = 0) -> dict:
    """The cpu_baseline of bench.py: about `seconds` of the reference block on
    every host core, after one warm-up step."""
    pool = RefPool(num_experts, None, wseed)
    try:
        pool.step(TOKENS_PER_PROC)  # warm-up (worker start-up and first-touch of the weights)
        return measure_pool(pool, seconds=seconds)
    finally:
        pool.close()
