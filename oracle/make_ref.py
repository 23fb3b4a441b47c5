"""Compile the REFERENCE MoE block into oracle/_ref/ (CPU baseline).

BASELINE INFRASTRUCTURE ONLY.  Runs in the development container (it needs the
reference tree and the TVM Relax build inside `tilelang`): model/mlp.py's
MLPBlock, unmodified, is exported with TVM's Relax frontend and compiled for
the CPU with TVM's C target (see oracle/ref_harness.py for the three harness
fixes around TVM).  The outputs -- moe_e{E}.so and the parameter order
moe_e{E}.json -- are git-ignored build products that travel with the source
tree to the GPU box, where oracle/ref_runner.py executes them with the Relax VM.

    python -m oracle.make_ref [--ref /path/to/reference] [--experts 128 32]
"""
from __future__ import annotations

import argparse
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")


def build_ref(ref_root: str, experts=(128, 32), force: bool = False) -> list[str]:
    os.makedirs(REF_DIR, exist_ok=True)
    todo = [E for E in experts if force or not os.path.exists(os.path.join(REF_DIR, f"moe_e{E}.so"))]
    if not todo:
        return []
    from oracle.ref_harness import RefHarness

    h = RefHarness(ref_root)
    nn = h.nn
    built = []
    for E in todo:
        cfg = h.config.GPTOssConfig(num_experts=E, context_window_size=4096)
        blk = h.mlp.MLPBlock(cfg)
        spec = {"forward": {"x": nn.spec.Tensor([1, "seq_len", 2880], "bfloat16")}}
        _, names = h.compile(blk, spec, f"moe_e{E}", out_dir=REF_DIR)
        with open(os.path.join(REF_DIR, f"moe_e{E}.json"), "w") as f:
            json.dump(names, f)
        built.append(os.path.join(REF_DIR, f"moe_e{E}.so"))
    return built


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GPTOSS_REFERENCE", "/root/reference"))
    ap.add_argument("--experts", type=int, nargs="+", default=[128, 32])
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    for p in build_ref(a.ref, a.experts, a.force):
        print("built", p)


if __name__ == "__main__":
    main()
