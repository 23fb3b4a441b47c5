"""Benchmark: gpt-oss MoE layer tokens/s on B200.

Workload: one gpt-oss-120b MoE layer -- 128 experts,
top-4, hidden = intermediate = 2880, MXFP4 weights with e2m1 codes uniform
over 16 values and E8M0 scales uniform in 118..124, router N(0, 0.02) -- over
8192 prefill tokens of bf16 N(0,1) per GPU (synthetic, seeded).  A "step" is
one MLPBlock.forward (RMSNorm, router, top-4, permutation, grouped MXFP4
expert GEMMs, weighted combine, residual) over that batch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}]

With N > 1 (torchrun, one process per GPU) the experts are sharded E/N per
rank (expert parallelism) and every rank routes its own 8192 tokens (weak
scaling); the rows move through peer memory (stores into the other ranks'
CUDA-IPC buffers, `--exchange peer`, the default) or NCCL all-to-all-v
(`--exchange nccl`).

value: whole-job tokens/s with inputs resident in HBM; e2e: the same through
the public MLPBlock API with the input copied from pinned host memory and the
output copied back inside the timed region.  The 1.7 GB of expert weights per
GPU exceed the 126 MB L2, so no explicit flush is needed between steps.

At N = 1 the line also carries `full_model`: the whole gpt-oss-20b
and gpt-oss-120b forwards on random-init weights -- greedy decode
at batch 1 / 8 / 64 over a 2048-token context and at batch 256 over 4096, one
CUDA graph per step, plus 4096- and 16384-token prefills (`--full-model`).
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

TOKENS = 8192  # default; --tokens overrides (smaller cases for profiling)
NUM_EXPERTS = 128
TOP_K = 4
HIDDEN = 2880
INTER = 2880
METRIC = "MoE-layer tokens/s (gpt-oss-120b MoE layer, 8192-token prefill)"
FP4_DENSE_PEAK_TFLOPS = 9000.0  # nominal dense e2m1 tensor peak of one B200
# DRAM bytes (read + write) of one gate/up GEMM launch at the 8192-token workload, from the
# ncu capture summarised in profiles/moe_gemm_config3_prefill.md
MLP1_DRAM_TRAFFIC_BYTES = 1.335910e9 + 0.181591e9


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons through NVML while
    the timed region runs (read-only queries)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu, self.period = gpu_index, period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()

    def __enter__(self):
        # re-entering accumulates: the timed regions of one line share the record
        self._stop.clear()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self._nv = None
        return self

    def _run(self):
        nv, h = self._nv, self._h
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                bits = get_reasons(h)
                for bit, name in self.REASONS.items():
                    if bits & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._nv is not None:
            self._t.join(timeout=2)

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def run_b200(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
    lib = importlib.import_module("gpt-oss-tvm_b200._lib")
    ep = importlib.import_module("gpt-oss-tvm_b200.ep") if world > 1 else None
    cfg = cfgm.gpt_oss_120b()
    E_local = NUM_EXPERTS // world
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)

    # synthetic weights with the benchmark's distributions, generated on device
    blk = mlp.MLPBlock(cfg, device=dev, expert_offset=rank * E_local, num_local_experts=E_local)
    with torch.no_grad():
        gw = torch.Generator(device=dev)
        gw.manual_seed(99)  # router weights identical on every rank
        blk.gate_weight.copy_((torch.randn(NUM_EXPERTS, HIDDEN, generator=gw, device=dev) * 0.02).to(torch.bfloat16))
        blk.gate_bias.copy_((torch.randn(NUM_EXPERTS, generator=gw, device=dev) * 0.02).to(torch.bfloat16))
        for name in ("mlp1_weight_blocks", "mlp2_weight_blocks"):
            t = getattr(blk, name)
            t.copy_(torch.randint(0, 256, t.shape, generator=g, device=dev, dtype=torch.int32).to(torch.uint8))
        for name in ("mlp1_weight_scales", "mlp2_weight_scales"):
            t = getattr(blk, name)
            t.copy_(torch.randint(118, 125, t.shape, generator=g, device=dev, dtype=torch.int32).to(torch.uint8))
        for name in ("mlp1_bias", "mlp2_bias"):
            t = getattr(blk, name)
            t.copy_((torch.randn(t.shape, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    blk.prepare()  # one-time weight check (enables the f16 GEMM path for these scale codes)
    x = torch.randn(TOKENS, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    runner = ep.ExpertParallelMoE(blk, TOKENS, peer=args.exchange == "peer") if ep else None

    def step():
        if runner is not None:
            runner.forward(x, out)
        else:
            blk.forward(x, out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- device-timed region (inputs resident)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * TOKENS / (ms_per_step / 1e3)

    # ---- kernel-level timing of the dominant kernel (gate/up grouped GEMM)
    prof = blk.profile_stages(x) if runner is None else runner.profile_stages(x)
    assert blk.device_error() == 0, "device error flag set during the benchmark"

    # ---- end-to-end through the public API: pinned host in, host out.  Every
    # step copies its input host->device and its output device->host inside the
    # timed region; the copies run on their own streams, double-buffered, so the
    # input of step i+1 and the output of step i move while step i / i+1 compute.
    x_host = x.cpu().pin_memory()
    out_host = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(x) for _ in range(2)]
    od = [torch.empty_like(out) for _ in range(2)]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def fwd(xi, oi):
        if runner is not None:
            runner.forward(xi, oi)
        else:
            blk.forward(xi.reshape(1, TOKENS, HIDDEN), oi.reshape(1, TOKENS, HIDDEN))

    def run_e2e(n):
        in_ev = [torch.cuda.Event() for _ in range(2)]
        done_ev = [torch.cuda.Event() for _ in range(2)]
        out_ev = [torch.cuda.Event() for _ in range(2)]
        s_in.wait_stream(comp)
        with torch.cuda.stream(s_in):
            xd[0].copy_(x_host, non_blocking=True)
            in_ev[0].record(s_in)
        for i in range(n):
            b = i % 2
            comp.wait_event(in_ev[b])
            if i >= 2:
                comp.wait_event(out_ev[b])  # od[b] drained by the copy-out of step i-2
            fwd(xd[b], od[b])
            done_ev[b].record(comp)
            if i + 1 < n:
                nb = (i + 1) % 2
                if i >= 1:
                    s_in.wait_event(done_ev[nb])  # xd[nb] consumed by step i-1
                with torch.cuda.stream(s_in):
                    xd[nb].copy_(x_host, non_blocking=True)
                    in_ev[nb].record(s_in)
            s_out.wait_event(done_ev[b])
            with torch.cuda.stream(s_out):
                out_host[b].copy_(od[b], non_blocking=True)
                out_ev[b].record(s_out)
        comp.wait_event(out_ev[(n - 1) % 2])
        if n >= 2:
            comp.wait_event(out_ev[n % 2])

    run_e2e(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        e0.record()
        run_e2e(args.steps)
        e1.record()
        torch.cuda.synchronize()
    assert torch.equal(out_host[(args.steps - 1) % 2], od[(args.steps - 1) % 2].cpu())
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * TOKENS / (e2e_ms / args.steps / 1e3)

    peaks, peak_kind = measured_peaks()
    gemm_flops = prof["mlp1_flops"]
    achieved_tflops = gemm_flops / (prof["mlp1_ms"] / 1e3) / 1e12
    peak_tflops = float(peaks.get("bf16_tflops", 1590.0))
    total_gemm_tflops = prof["gemm_flops"] / (prof["gemm_ms"] / 1e3) / 1e12

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": ("f16 GEMM operands (MXFP4 weights decoded exactly on chip), fp32 accumulate; bf16 I/O"
                      if blk.f16_path else "bf16 (MXFP4 weights dequantised exactly on chip); fp32 accumulate"),
            "data": "synthetic (seeded; BASELINE configs[3] distributions)",
            "config": {"workload": "gpt-oss-120b MoE layer prefill (configs[3])", "tokens_per_gpu": TOKENS,
                       "num_experts": NUM_EXPERTS, "experts_per_gpu": E_local, "top_k": TOP_K, "hidden": HIDDEN,
                       "intermediate": INTER, "parallelism": f"ep{world}" if world > 1 else "single",
                       **({"exchange": "peer memory (CUDA IPC buffers, NVLink stores)" if args.exchange == "peer"
                           else "NCCL all-to-all-v"} if world > 1 else {}),
                       "l2": "no flush: 1.7 GB of expert weights per step exceed the 126 MB L2"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": TOKENS * HIDDEN * 2, "d2h_bytes_per_step": TOKENS * HIDDEN * 2,
                    "note": "MLPBlock.forward per step with its input copied from pinned host memory and its output "
                            "copied back, on copy streams double-buffered against the compute stream"},
            "gpu_launches": prof["launches_per_step"] * args.steps,
            "roofline": {"bound": "tensor", "kernel": "moe_gemm_tc_kernel<0> (gate/up + SwiGLU)",
                         "achieved": round(achieved_tflops, 1), "peak": peak_tflops, "unit": "TFLOP/s",
                         "frac": round(achieved_tflops / peak_tflops, 4), "peak_source": f"{peak_kind} bf16 dense (cuBLAS)",
                         "traffic": (MLP1_DRAM_TRAFFIC_BYTES if TOKENS == 8192 and world == 1 else None),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                         "algorithmic_bytes": 128 * (8294400 + 518400 + 11520) + 2 * TOKENS * TOP_K * HIDDEN * 2,
                         "mma_kind": "tcgen05.mma kind::f16 (" + ("f16" if blk.f16_path else "bf16") + " x same -> fp32)",
                         "frac_of_fp4_dense_peak": round(achieved_tflops / FP4_DENSE_PEAK_TFLOPS, 4),
                         "all_gemm_tflops": round(total_gemm_tflops, 1)},
            "stages_ms": {k: round(v, 4) for k, v in prof.items() if k.endswith("_ms")},
            "clocks": sampler.summary(),
        }
        if args.decode and world == 1:
            line["decode"] = {name: decode_bench(dev, E, M, 20, peaks) for name, (E, M) in DECODE_CASES.items()}
            line["attention"] = attention_bench(dev, peaks)
        if args.full_model != "none" and world == 1:
            names = [n for n in FULL_MODEL_CASES if args.full_model == "all" or n.startswith(args.full_model)]
            line["full_model"] = {n: full_model_bench(dev, peaks, n, steps=args.steps, warmup=args.warmup)
                                  for n in names}
        if args.cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args)
        print(json.dumps(with_headlines(line)), flush=True)
    if runner is not None:
        runner.close()
    blk.free_workspace()
    if world > 1:
        dist.destroy_process_group()


def with_headlines(line: dict) -> dict:
    """The same line with compact copies of the decode and attention
    measurements placed right after `e2e` (the long per-stage records stay
    at the end): ms, achieved GB/s or TFLOP/s and the roofline fraction."""
    head = {}
    for name, d in (line.get("decode") or {}).items():
        key = "configs4_moe_decode_256tok" if "256" in name else "configs0_moe_decode_1tok"
        head[key] = {"ms": d["ms_per_step"], "achieved_gbs": d["achieved_gbs"], "hbm_frac": d["hbm_frac"]}
    att = {}
    for name, d in (line.get("attention") or {}).items():
        if not isinstance(d, dict):
            continue
        key = ("prefill4096_full" if "full causal" in name else "prefill4096_window128" if "window" in name
               else "decode_b32_kv8192")
        att[key] = {"ms": d["ms"], **({"tflops": d["tflops"], "bf16_frac": d["frac"]} if "tflops" in d
                                      else {"achieved_gbs": d["achieved_gbs"], "hbm_frac": d["hbm_frac"]})}
    out = {}
    for k, v in line.items():
        out[k] = v
        if k == "e2e":
            if head:
                out["decode_headline"] = head
            if att:
                out["attention_headline"] = att
    return out


def _random_block(mlp, cfgm, E, dev, seed):
    cfg = cfgm.GPTOssConfig(num_experts=E)
    blk = mlp.MLPBlock(cfg, device=dev)
    g = torch_gen(dev, seed)
    import torch
    with torch.no_grad():
        blk.gate_weight.copy_((torch.randn(E, HIDDEN, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        blk.gate_bias.copy_((torch.randn(E, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        for name in ("mlp1_weight_blocks", "mlp2_weight_blocks"):
            t = getattr(blk, name)
            t.copy_(torch.randint(0, 256, t.shape, generator=g, device=dev, dtype=torch.int32).to(torch.uint8))
        for name in ("mlp1_weight_scales", "mlp2_weight_scales"):
            t = getattr(blk, name)
            t.copy_(torch.randint(118, 125, t.shape, generator=g, device=dev, dtype=torch.int32).to(torch.uint8))
        for name in ("mlp1_bias", "mlp2_bias"):
            t = getattr(blk, name)
            t.copy_((torch.randn(t.shape, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    return blk.prepare()


def torch_gen(dev, seed):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return g


DECODE_CASES = {
    "gpt-oss-20b (configs[0]) 1 token": (32, 1),
    "gpt-oss-120b batched decode (configs[4]) 256 tokens": (128, 256),
}


def decode_only(args):
    """--decode-only I: just decode case I on cuda:0 (a small, self-contained
    command for kernel profiles)."""
    import torch
    name = list(DECODE_CASES)[args.decode_only]
    E, M = DECODE_CASES[name]
    peaks, _ = measured_peaks()
    print(json.dumps({name: decode_bench(torch.device("cuda", 0), E, M, args.steps, peaks)}), flush=True)


def decode_bench(dev, E, M, steps, peaks):
    """MoE decode: M tokens through MLPBlock.forward replayed from a CUDA
    graph, L2 flushed (a 256 MB write) before every timed step.  Bytes =
    13,236,480 per distinct expert the step routes to (MXFP4 blocks, scales and
    biases of both projections) + router weights + activations."""
    import torch
    mlp = importlib.import_module("gpt-oss-tvm_b200.mlp")
    cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
    blk = _random_block(mlp, cfgm, E, dev, 7 + E)
    g = torch_gen(dev, 11 + M)
    xs = [torch.randn(M, HIDDEN, generator=g, device=dev).to(torch.bfloat16) for _ in range(4)]
    x = torch.empty_like(xs[0])
    out = torch.empty_like(x)
    x.copy_(xs[0])
    for _ in range(3):
        blk.forward(x, out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        blk.forward(x, out)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    times, bytes_ = [], []
    per_expert = 2 * (INTER * HIDDEN // 2 + INTER * HIDDEN // 32 + INTER) + \
        (HIDDEN * INTER // 2 + HIDDEN * INTER // 32 + HIDDEN)  # 13,236,480 B
    for i in range(steps + 3):
        x.copy_(xs[i % len(xs)])
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    # distinct experts per input (routing of each of the inputs)
    distinct = []
    for xi in xs:
        logits = torch.empty(M, E, dtype=torch.bfloat16, device=dev)
        w = torch.empty(M, 4, dtype=torch.bfloat16, device=dev)
        idx = torch.empty(M, 4, dtype=torch.int32, device=dev)
        t = torch.empty_like(xi)
        lib = importlib.import_module("gpt-oss-tvm_b200._lib")
        S = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        P = lambda a: ctypes.c_void_p(a.data_ptr())  # noqa: E731
        lib.call("gptoss_rms_norm", P(xi), P(blk.norm_weight), M, HIDDEN, ctypes.c_float(1e-5), P(t), S)
        lib.call("gptoss_moe_router", P(t), P(blk.gate_weight), P(blk.gate_bias), M, E, HIDDEN, 4, P(logits), P(w),
                 P(idx), None, S)
        distinct.append(int(torch.unique(idx).numel()))
    nbytes = statistics.mean(distinct) * per_expert + E * HIDDEN * 2 + E * 2 + HIDDEN * 2 + 2 * M * HIDDEN * 2
    ms = statistics.median(times)
    st = blk.profile_stages(xs[0], repeats=5, flush=flush)
    stages = {k: round(v, 4) for k, v in st.items() if k.endswith("_ms")}
    gbs = nbytes / (ms / 1e3) / 1e9
    del graph
    blk.free_workspace()
    return {"tokens": M, "experts": E, "ms_per_step": round(ms, 4), "tokens_per_s": round(M / (ms / 1e3), 1),
            "distinct_experts": statistics.mean(distinct), "bytes_per_step": int(nbytes),
            "achieved_gbs": round(gbs, 1), "hbm_peak_gbs": peaks.get("hbm_gbs"),
            "hbm_frac": round(gbs / float(peaks.get("hbm_gbs", 6650.0)), 4),
            "l2": "flushed before every step (256 MB write)", "cuda_graph": True,
            "stages_ms": stages, "expert_path": st.get("expert_path"),
            "stages_note": "kernels launched one by one (not graph-replayed), L2 flushed"}


def attention_bench(dev, peaks, iters=10):
    """Attention with sinks, gpt-oss config 1: prefill of
    4096 tokens on a full-causal and a 128-window layer, and decode of one token
    for 32 sequences over 8192 cached keys (full layer).  Inputs are bf16 N(0,1)
    resident on the device; CUDA events around `iters` back-to-back calls, the
    256 MB L2 flush before each call.  FLOPs (full prefill) = 4 x (S^2/2) x 64 x 64
    heads; bytes (windowed prefill) = q+k+v+o; bytes (decode) = K+V of the 32 caches."""
    import torch
    lib = importlib.import_module("gpt-oss-tvm_b200._lib")
    g = torch_gen(dev, 21)
    S, HQ, HKV, D = 4096, 64, 8, 64
    P = lambda a: ctypes.c_void_p(a.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    sinks = torch.randn(HQ, generator=g, device=dev).to(torch.bfloat16)

    def timed(fn):
        times = []
        for i in range(iters + 2):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= 2:
                times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    out = {}
    q = torch.randn(S, HQ, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(S, HKV, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(S, HKV, D, generator=g, device=dev).to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(S, HQ, dtype=torch.float32, device=dev)
    for window in (0, 128):
        ms = timed(lambda: lib.call("gptoss_attn_prefill", P(q), P(k), P(v), P(sinks), S, S, HQ, HKV, D, window,
                                    ctypes.c_float(0.125), P(o), P(lse), stream))
        if window == 0:
            flops = 4.0 * (S * S / 2) * D * HQ
            tf = flops / (ms / 1e3) / 1e12
            out["prefill 4096, full causal layer"] = {
                "ms": round(ms, 4), "tflops": round(tf, 1), "peak_tflops": peaks.get("bf16_tflops"),
                "frac": round(tf / float(peaks.get("bf16_tflops", 1590.0)), 4),
                "kernel": "attn_prefill_tc_kernel (tcgen05.mma kind::f16, S and O in TMEM, two query tiles "
                          "ping-pong)"}
        else:
            nbytes = S * (HQ + 2 * HKV + HQ) * D * 2
            gbs = nbytes / (ms / 1e3) / 1e9
            out["prefill 4096, window 128 layer"] = {
                "ms": round(ms, 4), "bytes": nbytes, "achieved_gbs": round(gbs, 1),
                "hbm_frac": round(gbs / float(peaks.get("hbm_gbs", 6650.0)), 4),
                "kernel": "attn_prefill_kernel (short windows: 64-query tiles, mma.sync bf16)"}
    del q, k, v, o, lse
    B, L = 32, 8192
    qd = torch.randn(B, HQ, D, generator=g, device=dev).to(torch.bfloat16)
    kc = torch.randn(B, L, HKV, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(B, L, HKV, D, generator=g, device=dev).to(torch.bfloat16)
    kv_len = torch.full((B,), L, dtype=torch.int32, device=dev)
    od = torch.empty_like(qd)
    lsed = torch.empty(B, HQ, dtype=torch.float32, device=dev)
    nb = int(lib.load().gptoss_attn_decode_scratch_bytes(B, HQ, L, 0))
    scratch = torch.empty(max(nb // 4, 1), dtype=torch.float32, device=dev)
    ms = timed(lambda: lib.call("gptoss_attn_decode", P(qd), P(kc), P(vc), P(kv_len), B, L, HQ, HKV, D, 0,
                                ctypes.c_float(0.125), P(sinks), P(scratch), nb, P(od), P(lsed), stream))
    nbytes = 2 * B * L * HKV * D * 2
    gbs = nbytes / (ms / 1e3) / 1e9
    out["decode B=32 x KV 8192, full layer"] = {
        "ms": round(ms, 4), "bytes": nbytes, "achieved_gbs": round(gbs, 1),
        "hbm_frac": round(gbs / float(peaks.get("hbm_gbs", 6650.0)), 4),
        "kernel": "attn_decode_kernel (split-KV, 8 GQA heads per mma) + merge"}
    out["note"] = "L2 flushed (256 MB write) before every call; inputs bf16 N(0,1) on the device"
    return out


FULL_MODEL_CASES = {
    # name: (config factory, decode context, decode batches, prompts prefilled for the decode context, prefill length)
    "gpt-oss-20b (configs[2])": ("gpt_oss_20b", 2048, (1, 8, 64), 64, 4096),
    "gpt-oss-120b (configs[4])": ("gpt_oss_120b", 4096, (256,), 16, 16384),
}
EXPERT_BYTES = (5760 * 90 * 16 + 5760 * 90 + 5760 * 2) + (2880 * 90 * 16 + 2880 * 90 + 2880 * 2)


def _routed_experts(model, cache, ids, lib):
    """Distinct experts each layer's router picks for one decode step of the
    batch (an extra, untimed forward; the cache is rolled back after it)."""
    import torch
    cfg = model.config
    E, H, K, B = cfg.num_experts, cfg.hidden_size, cfg.num_experts_per_tok, ids.numel()
    P = lambda a: ctypes.c_void_p(a.data_ptr())  # noqa: E731
    counts = []

    class Counting:
        def __init__(self, mlp):
            self.mlp = mlp

        def __call__(self, x, out=None):
            S = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            x2 = x.reshape(-1, H).contiguous()
            t = torch.empty_like(x2)
            lib.call("gptoss_rms_norm", P(x2), P(self.mlp.norm_weight), B, H, ctypes.c_float(1e-5), P(t), S)
            logits = torch.empty(B, E, dtype=torch.bfloat16, device=x.device)
            w = torch.empty(B, K, dtype=torch.bfloat16, device=x.device)
            idx = torch.empty(B, K, dtype=torch.int32, device=x.device)
            err = torch.zeros(4, dtype=torch.int32, device=x.device)
            lib.call("gptoss_moe_router", P(t), P(self.mlp.gate_weight), P(self.mlp.gate_bias), B, E, H, K, P(logits),
                     P(w), P(idx), P(err), S)
            counts.append(int(torch.unique(idx).numel()))
            return self.mlp.forward(x, out)

    blocks = model.model.block
    saved = [b.mlp for b in blocks]
    try:
        for b in blocks:
            b.mlp = Counting(b.mlp)
        cache.begin_decode_on_device(B)
        model.decode(model.embed(ids), cache)
        torch.cuda.synchronize()
    finally:
        for b, m in zip(blocks, saved):
            b.mlp = m
        cache.rollback_device()
    return counts


def full_model_bench(dev, peaks, name, steps=20, warmup=3, batches=None, prefill=True, ep=False):
    """Full-model forward (GPTOssForCausalLM, random-init weights from a
    seed): greedy decode at the configuration's batch sizes over its context
    (sequences 0..B-1, one CUDA graph per step: embedding, every layer, final
    norm, unembedding, argmax), and one long prefill.

    Decode: the context is prefilled for real (distinct prompts; with fewer
    distinct prompts than sequences their KV rows are copied to the others,
    each sequence then decoding its own token), every batch restarts at the
    same context length, W warm-up replays, K timed replays (CUDA events).
    Algorithmic bytes of a step = attention and router weights of every layer
    + the experts the routers pick (counted by an untimed forward of the same
    step) + the KV rows each layer reads (the window on sliding layers) +
    embedding rows, unembedding weight and the logits.  The >= 13 GB of
    weights read per step exceed the 126 MB L2 (no flush needed).
    e2e: the same steps with each step's input tokens copied from pinned host
    memory and its greedy tokens copied back (host sync every step).

    ep (torchrun, one process per GPU): the experts of every layer are sharded
    over the ranks and each rank runs attention for its own prompts and decode
    batch (weak scaling); times are the max over ranks, tokens/s count every
    rank's tokens, and the decode steps run eagerly (their exchanges hold
    collectives).  The bytes-per-step accounting is single-GPU only."""
    import torch.distributed as dist
    import numpy as np
    import torch
    modm = importlib.import_module("gpt-oss-tvm_b200.model")
    engm = importlib.import_module("gpt-oss-tvm_b200.engine")
    cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
    lib = importlib.import_module("gpt-oss-tvm_b200._lib")
    factory, ctx, case_batches, distinct, P_len = FULL_MODEL_CASES[name]
    batches = tuple(batches) if batches else case_batches
    cfg = getattr(cfgm, factory)()
    L, V, H = cfg.num_hidden_layers, cfg.vocab_size, cfg.hidden_size
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    tc_peak = float(peaks.get("bf16_tflops", 1590.0))
    world = dist.get_world_size() if ep else 1
    rank = dist.get_rank() if ep else 0

    def slowest(ms):
        if not ep:
            return ms
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    t0 = time.perf_counter()
    model = modm.random_init(modm.GPTOssForCausalLM(cfg, device=dev, expert_parallel=True if ep else None), seed=0)
    Bmax = max(batches)
    model.reserve(max(P_len, Bmax, ctx))
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    res = {"weights_gb": round(sum(t.numel() * t.element_size() for _, t in model.named_parameters()) / 1e9, 2),
           "init_s": round(time.perf_counter() - t0, 1)}

    def ev():
        return torch.cuda.Event(enable_timing=True)

    # ---- prefill of one P_len-token prompt
    if not prefill:
        P_len = 0
    pc = model.create_paged_kv_cache(1, max(P_len, 1))
    ids = torch.randint(0, V, (P_len,), generator=g, device=dev)

    def prefill(ids_dev):
        pc.clear()
        pc.begin_forward([0], [P_len])
        lg, _ = model.prefill(model.embed(ids_dev), pc)
        return lg

    for _ in range(2 if P_len else 0):
        prefill(ids)
    times = []
    for _ in range(3 if P_len else 0):
        a, b = ev(), ev()
        a.record()
        prefill(ids)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = slowest(statistics.median(times) if times else 0.0)
    ids_host = ids.cpu().pin_memory()
    tok_host = torch.empty(1, dtype=torch.int64).pin_memory()
    times = []
    for _ in range(3 if P_len else 0):
        a, b = ev(), ev()
        a.record()
        ids_d = ids_host.to(dev, non_blocking=True)
        tok_host.copy_(torch.argmax(prefill(ids_d).reshape(-1)).reshape(1), non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    e2e_ms = slowest(statistics.median(times) if times else 0.0)
    D, Hq, Hkv, W = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.sliding_window_size
    dense = 2 * P_len * H * (D * (Hq + 2 * Hkv)) + 2 * P_len * (D * Hq) * H
    attn = sum(4 * D * Hq * (P_len * P_len / 2 if i % 2 else P_len * min(W, P_len)) for i in range(L))
    moe = 2 * P_len * cfg.num_experts_per_tok * (2 * cfg.intermediate_size * H + H * cfg.intermediate_size)
    flops = L * (dense + moe) + attn + 2 * H * V
    res[f"prefill {P_len} tokens"] = {} if not P_len else {
        "ms": round(ms, 3), "tokens_per_s": round(world * P_len / ms * 1e3, 1),
        "tflops": round(world * flops / ms / 1e9, 1),
        "frac_of_bf16_peak": round(flops / ms / 1e9 / tc_peak, 4),
        "e2e_tokens_per_s": round(world * P_len / e2e_ms * 1e3, 1),
        "e2e": "prompt ids copied from pinned host memory, greedy token copied back, inside the timed region",
        "flops_per_prefill": flops}
    del pc
    torch.cuda.empty_cache()

    # ---- decode over a ctx-token context
    dc = model.create_paged_kv_cache(Bmax, ctx + steps + 8)
    distinct = min(distinct, Bmax)
    for s in range(distinct):
        p = torch.randint(0, V, (ctx,), generator=g, device=dev)
        dc.begin_forward([s], [ctx])
        model.prefill(model.embed(p), dc)
    for s in range(distinct, Bmax):
        dc.copy_sequence(s % distinct, s)
    torch.cuda.synchronize()
    if ep:
        # exchange buffers sized for the decode batch (the GEMMs of an
        # expert-parallel step are launched on the buffer capacity)
        model.release()
        model.reserve(Bmax)

    def restart():
        dc.lengths.fill_(ctx)
        dc.rollback_device()

    attn_w = L * 2 * ((D * (Hq + 2 * Hkv)) * (H + 1) + H * (D * Hq + 1) + Hq + H)
    router_w = L * 2 * (cfg.num_experts * (H + 1) + H)
    kv_span = [min(ctx + steps // 2, W) if i % 2 == 0 else ctx + steps // 2 for i in range(L)]
    for B in batches:
        restart()
        tokens = torch.randint(0, V, (B,), generator=g, device=dev)
        routed = _routed_experts(model, dc, tokens, lib) if not ep else None
        dec = engm.GreedyDecodeGraph(model, dc, B)
        dec.set_tokens(tokens)
        for _ in range(warmup):
            dec.step()
        restart()
        dec.set_tokens(tokens)
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record()
        for _ in range(steps):
            dec.step()
        b.record()
        torch.cuda.synchronize()
        ms = slowest(a.elapsed_time(b) / steps)
        # e2e through pinned host buffers, host sync every step
        restart()
        th = tokens.cpu().pin_memory()
        nh = torch.empty_like(th).pin_memory()
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record()
        for _ in range(steps):
            dec.set_tokens(th.to(dev, non_blocking=True))
            _, nxt = dec.step()
            nh.copy_(nxt, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            th.copy_(nh)
        b.record()
        torch.cuda.synchronize()
        e2e_ms = slowest(a.elapsed_time(b) / steps)
        dec.close()
        if ep:
            res[f"decode batch {B} per GPU over {ctx} context"] = {
                "ms_per_step": round(ms, 4), "tokens_per_s": round(world * B / ms * 1e3, 1),
                "e2e_tokens_per_s": round(world * B / e2e_ms * 1e3, 1), "n_gpus": world,
                "experts_per_gpu": cfg.num_experts // world}
            continue
        kv = B * sum(kv_span) * Hkv * D * 2 * 2
        nbytes = attn_w + router_w + sum(routed) * EXPERT_BYTES + kv + H * V * 2 + B * H * 2 + B * V * (4 + 2 * 2)
        gbs = nbytes / ms / 1e6
        res[f"decode batch {B} over {ctx} context"] = {
            "ms_per_step": round(ms, 4), "tokens_per_s": round(B / ms * 1e3, 1),
            "e2e_tokens_per_s": round(B / e2e_ms * 1e3, 1), "bytes_per_step": nbytes,
            "achieved_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
            "experts_read_per_layer": round(sum(routed) / L, 2)}
    del dc
    model.release()
    del model
    torch.cuda.empty_cache()
    res["note"] = ("random-init weights (seed 0), prompt and decode token ids uniform over the vocabulary; "
                   "decode = CUDA-graph replays of GreedyDecodeGraph; hbm_frac of the measured copy bandwidth")
    return res


def full_model_only(args):
    """--full-model-only: the full-model measurements alone.  Under torchrun
    (N > 1), or with --fm-ep, the model runs expert-parallel over the ranks."""
    import datetime

    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    peaks, _ = measured_peaks()
    names = list(FULL_MODEL_CASES) if args.full_model == "all" else [n for n in FULL_MODEL_CASES
                                                                      if n.startswith(args.full_model)]
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ep = world > 1 or args.fm_ep
    if ep:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
    batches = [int(b) for b in args.fm_batches.split(",")] if args.fm_batches else None
    out = {n: full_model_bench(dev, peaks, n, steps=args.steps, warmup=args.warmup, batches=batches,
                               prefill=args.fm_prefill, ep=ep) for n in names}
    if rank == 0:
        print(json.dumps({"full_model": out, "n_gpus": world}), flush=True)
    if ep:
        dist.barrier()
        dist.destroy_process_group()


def route_bench(dev, iters=10):
    """RMSNorm + router (logits, top-4, softmax) of the gpt-oss-120b MoE block
    (128 experts) at the configs[3] prefill size (8192 tokens: router_kernel)
    and the configs[4] decode batch (256 tokens: router_chain_kernel); CUDA
    events around each call, 256 MB L2 flush before each.  Inputs resident."""
    import torch
    lib = importlib.import_module("gpt-oss-tvm_b200._lib")
    g = torch_gen(dev, 31)
    E, K = NUM_EXPERTS, TOP_K
    P = lambda a: ctypes.c_void_p(a.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    gw = (torch.randn(E, HIDDEN, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    gb = (torch.randn(E, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    nw = torch.ones(HIDDEN, dtype=torch.bfloat16, device=dev)
    out = {}
    for M in (8192, 256):
        x = torch.randn(M, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        t = torch.empty_like(x)
        logits = torch.empty(M, E, dtype=torch.bfloat16, device=dev)
        w = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
        idx = torch.empty(M, K, dtype=torch.int32, device=dev)
        tn, tr = [], []
        for i in range(iters + 2):
            flush.zero_()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record()
            lib.call("gptoss_rms_norm", P(x), P(nw), M, HIDDEN, ctypes.c_float(1e-5), P(t), stream)
            ev[1].record()
            lib.call("gptoss_moe_router", P(t), P(gw), P(gb), M, E, HIDDEN, K, P(logits), P(w), P(idx), None, stream)
            ev[2].record()
            torch.cuda.synchronize()
            if i >= 2:
                tn.append(ev[0].elapsed_time(ev[1]))
                tr.append(ev[1].elapsed_time(ev[2]))
        chain_steps = M * E * HIDDEN
        rt = statistics.median(tr)
        out[f"{M} tokens x {E} experts"] = {
            "rmsnorm_ms": round(statistics.median(tn), 4), "router_topk_ms": round(rt, 4),
            "router_kernel": "router_kernel" if M > 512 else "router_chain_kernel",
            "chain_steps_per_ns": round(chain_steps / (rt * 1e6), 2)}
    out["note"] = "L2 flushed before every call; serial bf16 router chains (2880 dependent steps per token and expert)"
    return out


DENSE_SHAPES = {"qkv 5120x2880": (5120, 2880, True), "out 2880x4096": (2880, 4096, True),
                "unembedding 201088x2880": (201088, 2880, False)}


def dense_bench(dev, peaks, iters=10, tokens=(1, 8, 64, 256, 4096)):
    """The attention block's projections and the unembedding (bf16, fp32
    accumulation): gptoss_dense_gemm (tcgen05) beside torch's nn.Linear
    (cuBLAS), and for up to gptoss_dense_gemv_max_tokens() tokens the
    warp-per-row gptoss_dense_gemv, on the same inputs; CUDA events per call after a 256 MB L2
    flush, median of `iters`.  Inputs resident."""
    import torch
    import torch.nn.functional as F
    lib = importlib.import_module("gpt-oss-tvm_b200._lib")
    g = torch_gen(dev, 41)
    P = lambda a: ctypes.c_void_p(a.data_ptr()) if a is not None else None  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    tc_peak = float(peaks.get("bf16_tflops", 1590.0))
    res = {}
    for name, (N, K, has_bias) in DENSE_SHAPES.items():
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, generator=g, device=dev) * 0.02).to(torch.bfloat16) if has_bias else None
        for T in tokens:
            if T > 256 and not has_bias:
                continue  # the unembedding only sees the last token of each sequence
            x = torch.randn(T, K, generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty(T, N, dtype=torch.bfloat16, device=dev)

            def ours():
                lib.call("gptoss_dense_gemm", P(x), T, P(w), P(b), N, K, P(out), None, stream)

            def theirs():
                F.linear(x, w, b)

            def gemv():
                lib.call("gptoss_dense_gemv", P(x), T, P(w), P(b), N, K, P(out), stream)

            fns = [("gptoss_dense_gemm", ours), ("cublas", theirs)]
            if T <= lib.load().gptoss_dense_gemv_max_tokens():
                fns.append(("gptoss_dense_gemv", gemv))
            times = {}
            for tag, fn in fns:
                ts = []
                for i in range(iters + 2):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn()
                    e1.record()
                    torch.cuda.synchronize()
                    if i >= 2:
                        ts.append(e0.elapsed_time(e1))
                times[tag] = statistics.median(ts)
            bytes_ = N * K * 2 + T * K * 2 + T * N * 2
            flops = 2.0 * T * N * K
            ms = times["gptoss_dense_gemm"]
            res[f"{name} T={T}"] = {
                "ms": round(ms, 4), "cublas_ms": round(times["cublas"], 4),
                "speedup_vs_cublas": round(times["cublas"] / ms, 3),
                "achieved_gbs": round(bytes_ / ms / 1e6, 1), "hbm_frac": round(bytes_ / ms / 1e6 / hbm, 4),
                "tflops": round(flops / ms / 1e9, 1), "tensor_frac": round(flops / ms / 1e9 / tc_peak, 4)}
            if "gptoss_dense_gemv" in times:
                res[f"{name} T={T}"]["gemv_ms"] = round(times["gptoss_dense_gemv"], 4)
    res["note"] = "L2 flushed (256 MB write) before every call; bytes = weights + inputs + outputs once"
    return res


def kernel_case(args):
    """--kernel-case NAME: one family of kernels alone on cuda:0, printed as
    JSON (small, self-contained commands for ncu captures)."""
    import torch
    peaks, _ = measured_peaks()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    if args.kernel_case == "attention":
        res = attention_bench(dev, peaks, iters=args.steps)
    elif args.kernel_case == "dense":
        res = dense_bench(dev, peaks, iters=args.steps)
    else:
        res = route_bench(dev, iters=args.steps)
    print(json.dumps({args.kernel_case: res}), flush=True)


def cpu_baseline(args):
    """Reference CPU implementation on the host cores, on a bounded sample."""
    cb = importlib.import_module("oracle.cpu_baseline")
    return cb.measure(seconds=args.cpu_seconds, num_experts=NUM_EXPERTS)


def run_reference(args):
    """The reference's own CPU implementation of the path, on the host cores:
    model/mlp.py compiled by TVM (oracle/_ref, one process per core) when it
    was built, else the C restatement of the oracle (OpenMP)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    rr = importlib.import_module("oracle.ref_runner")
    if rr.available(NUM_EXPERTS):
        pool = rr.RefPool(NUM_EXPERTS)
        for _ in range(args.warmup):
            pool.step(rr.TOKENS_PER_PROC)
        cb = rr.measure_pool(pool, steps=args.steps)
        pool.close()
    else:
        import oracle
        oracle.build()
        synth = importlib.import_module("gpt-oss-tvm_b200.synthetic")
        p = synth.moe_params(NUM_EXPERTS, seed=0)
        cores = len(os.sched_getaffinity(0))
        for _ in range(args.warmup):
            oracle.moe_forward(synth.activations(cores, seed=1), p)
        tot_t, tot_n = 0.0, 0
        for k in range(args.steps):
            x = synth.activations(cores, seed=2 + k)
            t0 = time.perf_counter()
            oracle.moe_forward(x, p)
            tot_t += time.perf_counter() - t0
            tot_n += cores
        cb = {"value": tot_n / tot_t, "unit": "tokens/s", "cores": cores, "kind": "port",
              "extrapolated_from_tokens": tot_n, "measured_seconds": round(tot_t, 3), "measured_steps": args.steps,
              "sample": f"{args.steps} steps of {cores} tokens of the {NUM_EXPERTS}-expert MoE block, C restatement "
                        f"(OpenMP)"}
    tot_t, tot_n = cb["measured_seconds"], cb["extrapolated_from_tokens"]
    value = tot_n / tot_t
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(TOKENS / value * 1e3, 1),
        "ms_per_step_note": (f"extrapolated to the {TOKENS}-token step from {tot_n} tokens measured in "
                             f"{tot_t:.2f} s ({args.steps} steps of {tot_n // max(args.steps, 1)} tokens)"),
        "extrapolated_from_tokens": tot_n, "measured_seconds": round(tot_t, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 accumulate over bf16 activations and MXFP4 weights (reference CPU path)",
        "data": "synthetic (seeded; BASELINE configs[3] distributions)",
        "config": {"workload": "gpt-oss-120b MoE layer prefill (configs[3])", "tokens_per_gpu": TOKENS,
                   "num_experts": NUM_EXPERTS, "top_k": TOP_K, "hidden": HIDDEN, "intermediate": INTER,
                   "parallelism": "host cores"},
        "cpu_baseline": {k: (round(v, 3) if k == "value" else v) for k, v in cb.items()},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    global TOKENS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="measured seconds of the CPU baseline sample")
    ap.add_argument("--tokens", type=int, default=TOKENS, help="tokens per GPU (default: the configs[3] 8192)")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-decode", dest="decode", action="store_false", help="skip the MoE decode measurements")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel row exchange (N > 1): stores into the ranks' IPC-shared buffers or NCCL")
    ap.add_argument("--decode-only", type=int, default=None, choices=range(len(DECODE_CASES)),
                    help="run only this decode case (index into DECODE_CASES) and print its measurement")
    ap.add_argument("--full-model", default="all", choices=["none", "gpt-oss-20b", "gpt-oss-120b", "all"],
                    help="full-model decode/prefill measurements added to the line (1 GPU)")
    ap.add_argument("--full-model-only", action="store_true",
                    help="run only the --full-model measurements and print them")
    ap.add_argument("--fm-batches", default=None, help="with --full-model-only: comma-separated decode batch sizes")
    ap.add_argument("--fm-ep", action="store_true",
                    help="with --full-model-only: expert-parallel model even on one GPU (a one-rank group)")
    ap.add_argument("--no-fm-prefill", dest="fm_prefill", action="store_false",
                    help="with --full-model-only: skip the long-prompt prefill measurement")
    ap.add_argument("--kernel-case", default=None, choices=["attention", "route", "dense"],
                    help="run only this kernel family (attention prefill/decode, RMSNorm + router, or the dense "
                         "projections) and print it")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    TOKENS = args.tokens
    if args.kernel_case is not None:
        kernel_case(args)
    elif args.decode_only is not None:
        decode_only(args)
    elif args.full_model_only and args.impl != "reference":
        full_model_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
