"""CPU baseline timing for bench.py (BASELINE-measurement infrastructure).

Times the reference's CPU arithmetic for the MoE block on a bounded token
sample of the benchmark workload, using every host core:
  * kind "reference": the reference's own model/mlp.py compiled by TVM's C
    target into oracle/_ref/ (built in the development container by
    oracle/make_ref.py), run as one process per core over a token split;
  * kind "port": the C restatement in gptoss_oracle.c (OpenMP over the
    (token, expert) pairs), when oracle/_ref is absent.
"""
from __future__ import annotations

import importlib
import os
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


_PARAMS = {}


def _params(num_experts: int):
    if num_experts not in _PARAMS:
        synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
        _PARAMS[num_experts] = synth.moe_params(num_experts, seed=0)
    return _PARAMS[num_experts]


def measure(seconds: float = 10.0, num_experts: int = 128, tokens: int = 32) -> dict:
    ref = importlib.import_module("oracle.ref_runner")
    if ref.available(num_experts):
        try:
            return ref.measure(seconds=seconds, num_experts=num_experts)
        except Exception:  # the TVM runtime could not start here: fall back to the C restatement
            pass
    import oracle
    oracle.build()
    synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
    p = _params(num_experts)
    x = synth.activations(tokens, seed=1)
    cores = _cores()
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    t0 = time.perf_counter()
    oracle.moe_forward(x, p)
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "extrapolated_from_tokens": tokens, "measured_seconds": round(dt, 3),
            "sample": f"{tokens} tokens of the {num_experts}-expert MoE block (full MLPBlock.forward arithmetic, "
                      f"C restatement, OpenMP over token x expert pairs)", "seconds": dt}
