#!/usr/bin/env python
"""Benchmark of the B200 kernel backend (one JSON line on rank 0).

Headline workload: C = A @ B, M = N = K = 4096, bf16 inputs ~ N(0,1)/sqrt(K),
fp32 accumulation, bf16 output — the matmul configuration of the B200
benchmark set, on the best configuration the search space offers for this
backend (tcgen05, BLOCK_M 256, BLOCK_N 256, BLOCK_K 128, GROUP_M 16, 8 warps,
3 stages: a persistent CTA pair per SM pair, M=256 cta_group::2 MMAs, two
TMEM accumulators so each tile's epilogue overlaps the next tile's MMAs).
One step = one matmul launch.
Steps cycle over 4 independent input sets (4 x 96 MiB > 126 MB L2), so every
launch streams its operands from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU; every rank multiplies its
own matrices (candidate evaluation shards with no exchange step), the
timed region is bracketed by barriers + synchronize, and the max time over
ranks is used.  ``value`` is whole-job TFLOP/s.  ``--impl reference`` times
the reference's own CPU implementation of the path (its torch reference:
fp32 matmul of the upcast operands) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPE = (4096, 4096, 4096)
# persistent CTA pair (8 warps), 256 x 256 tiles, 128-deep K stages
BEST = {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 128, "GROUP_M": 16, "num_warps": 8,
        "num_stages": 3, "dtype": "bfloat16"}
FLOPS = 2.0 * SHAPE[0] * SHAPE[1] * SHAPE[2]
N_SETS = 4
METRIC = "matmul_bf16_4096_tflops"
WORKLOAD = "matmul bf16 M=N=K=4096, fp32 accumulate, bf16 out"
# DRAM bytes (read + write) per launch of the headline kernel from one ncu
# capture of this exact kernel and configuration (69.61 MB read + 14.26 MB
# written); reported only while the headline runs that kernel.
TRAFFIC_KERNEL = "matmul_tc2_kernel<bf16,256,256,cta_pair_persistent>"
TRAFFIC_BYTES_PER_LAUNCH = 83_875_000


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip the per-task, search and CPU-baseline legs")
    return ap.parse_args()


# ------------------------------------------------------------ distributed
def dist_init(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        # control traffic only (barriers, scalar max/sum, the search batch's
        # work counter): a gloo group on host tensors, no NCCL
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allreduce_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: int) -> None:
        self.proc = None
        sel = []
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            sel = ["-i", uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"]
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", *sel, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], 0.0, set()
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                s, m = float(f[1]), float(f[2])
            except ValueError:
                continue
            mx = max(mx, m)
            sm.append(s)
            for name, val in zip(self.REASONS, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ our backend
def run_ours(args, rank, world, local):
    from gpu_optimizer_b200.harness import default_peaks
    from gpu_optimizer_b200.runner import build_callable, check_device_status, warm_compile
    from gpu_optimizer_b200.tasks import get_task

    task = get_task("matmul", "b200")
    sets = [task.make_inputs(SHAPE, "bfloat16", "cuda", seed=10 * i + rank)
            for i in range(N_SETS)]
    kcs = [build_callable("matmul", SHAPE, BEST, s) for s in sets]
    for kc in kcs:
        warm_compile(kc)
    stream = torch.cuda.current_stream()
    # the clock sampler starts first; the warm-up steps then run right
    # before the timed ones, so the timed region does not begin on a GPU
    # that idled (and lowered its clock) while the sampler started
    clocks = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    for i in range(args.warmup):
        kcs[i % N_SETS].fn()
    torch.cuda.synchronize()
    check_device_status()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        kcs[i % N_SETS].fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    check_device_status()
    ms_max = allreduce_max(ms, world)
    ms_per_step = ms_max / args.steps
    value = world * args.steps * FLOPS / (ms_max * 1e-3) / 1e12
    per_launch_ms = ms / args.steps
    achieved = FLOPS / (per_launch_ms * 1e-3) / 1e12
    peaks = default_peaks()
    # A timed region under a second runs at burst clocks, so the burst
    # cuBLAS figure is its denominator; a seconds-long region settles under
    # the power cap, where the sustained figure applies.
    sustained = ms >= 1000.0
    peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    measured = peaks["source"] == "measured"
    peak_source = (("measured sustained cuBLAS bf16 (MEASURED_PEAKS.json bf16_tflops_sustained)"
                    if sustained else "measured burst cuBLAS bf16 (MEASURED_PEAKS.json "
                    "bf16_tflops)") if measured else
                   f"fallback {peak:g} TFLOP/s ({'sustained' if sustained else 'burst'})")

    # correctness of the measured kernel (last output vs the device reference)
    from gpu_optimizer_b200.correctness import check_correctness

    out = kcs[0].fn()
    rep = check_correctness(out, task.reference(*sets[0]), *task.tolerance("bfloat16"))

    e2e = measure_e2e(args, world, task)

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)/sqrt(K) bf16 operands, 4 rotating input sets",
        "config": {"workload": WORKLOAD,
                   "candidate": BEST, "kernel": kcs[0].launch["kernel"],
                   "l2": "4 rotating input sets of 96 MiB (384 MiB > 126 MB L2)",
                   "parallelism": f"independent per-GPU problems x{world} (no collective)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_source,
                     "frac_of_burst": round(achieved / peaks["bf16_tflops"], 4),
                     "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4),
                     "timed_region_ms": round(ms, 2),
                     "sm_mhz_median": clk["sm_mhz"] if clk else None,
                     "traffic": (TRAFFIC_BYTES_PER_LAUNCH
                                 if kcs[0].launch["kernel"] == TRAFFIC_KERNEL else None),
                     "algorithmic_flops_per_launch": FLOPS},
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clk,
        "correctness": {"passed": rep.passed, "max_abs_err": rep.max_abs_err,
                        "rel_err_floored": rep.rel_err_floored,
                        "rel_err_normwise": rep.rel_err_normwise},
    }
    return line


def measure_e2e(args, world, task):
    """Same metric through build_callable/fn with pinned host operands: every
    step copies its A and B host->device, multiplies, and reads C back.  Two
    buffer sets on three streams (copy-in, compute, copy-out) let step i's
    copies overlap the neighbouring steps' work; all copies of all timed
    steps are inside the timed region."""
    from gpu_optimizer_b200.runner import build_callable

    a_h, b_h = (t.cpu().pin_memory() for t in task.make_inputs(SHAPE, "bfloat16", "cpu", 99))
    nb = 2
    a_d = [torch.empty_like(a_h, device="cuda") for _ in range(nb)]
    b_d = [torch.empty_like(b_h, device="cuda") for _ in range(nb)]
    kcs = [build_callable("matmul", SHAPE, BEST, (a_d[i], b_d[i])) for i in range(nb)]
    c_h = [torch.empty(SHAPE[0], SHAPE[1], dtype=torch.bfloat16).pin_memory() for _ in range(nb)]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731
    comp_done = [ev() for _ in range(nb)]
    out_done = [ev() for _ in range(nb)]
    in_done = [ev() for _ in range(nb)]
    for i in range(nb):  # mark both buffer sets free
        comp_done[i].record(s_comp)
        out_done[i].record(s_out)
    steps = max(10, min(args.steps, 200))

    def step(i):
        k = i % nb
        with torch.cuda.stream(s_in):
            s_in.wait_event(comp_done[k])  # step i-2 finished reading a_d/b_d[k]
            a_d[k].copy_(a_h, non_blocking=True)
            b_d[k].copy_(b_h, non_blocking=True)
            in_done[k].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[k])
            s_comp.wait_event(out_done[k])  # step i-2's C[k] has been read back
            c = kcs[k].fn()
            comp_done[k].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[k])
            c_h[k].copy_(c, non_blocking=True)
            out_done[k].record(s_out)

    for i in range(4):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    s_comp.wait_event(e0)
    s_out.wait_event(e0)
    for i in range(steps):
        step(i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_comp)
    e1.record(s_out)
    torch.cuda.synchronize()
    ms = allreduce_max(e0.elapsed_time(e1), world)
    return {"value": round(world * steps * FLOPS / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": a_h.numel() * 2 + b_h.numel() * 2,
            "d2h_bytes_per_step": c_h[0].numel() * 2, "steps": steps,
            "pipeline": "2 buffer sets; copy-in / compute / copy-out streams"}


# ------------------------------------------------------------ CPU legs
def cpu_matmul_sample(rows: int, seconds: float):
    """The reference's CPU path (fp32 matmul of upcast bf16 operands,
    benchmarks/matmul/task.py:32-34) on a row slice of the workload."""
    from oracle import reference as O

    a, b = O.make_inputs("matmul", SHAPE, "bfloat16", 0, profile="b200")
    a = a[:rows].contiguous()
    torch.set_num_threads(os.cpu_count() or 1)
    O.reference("matmul", (a, b))  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        O.reference("matmul", (a, b))
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    flops = 2.0 * rows * SHAPE[1] * SHAPE[2] * n
    return flops / el / 1e12, n, el


def cpu_baseline():
    rows = SHAPE[0]
    v, n, el = cpu_matmul_sample(rows, 10.0)
    return {"value": round(v, 4), "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} x ({rows}x4096 rows of A) @ B(4096x4096), fp32 upcast, "
                      f"{el:.1f} s, torch CPU with {os.cpu_count()} threads"}


# Per-task CPU samples: the reference's CPU path (the oracle's restatement of
# each task.reference) on a bounded slice of the benchmark workload, scaled
# to the unit of the task's roofline work.  (task, full shape, sample shape,
# work of the sample in the task's unit numerator)
def _cpu_samples():
    def attn_flops(bh, s, d, causal):
        return 4.0 * bh * d * (s * (s + 1) / 2 if causal else s * s)
    return [
        ("vecadd", (1 << 24,), (1 << 24,), lambda sh: 3 * sh[0] * 4),
        ("softmax", (16384, 8192), (512, 8192), lambda sh: 2 * sh[0] * sh[1] * 2),
        ("layernorm", (16384, 8192), (512, 8192),
         lambda sh: 2 * sh[0] * sh[1] * 2 + 2 * sh[1] * 2),
        ("reduction", (1 << 28,), (1 << 26,), lambda sh: 4 * sh[0]),
        ("fused_gelu", (1 << 26,), (1 << 24,), lambda sh: 3 * sh[0] * 2),
        ("attention_causal", (128, 4096, 128), (1, 4096, 128),
         lambda sh: attn_flops(sh[0], sh[1], sh[2], True)),
        ("attention", (128, 4096, 128), (1, 4096, 128),
         lambda sh: attn_flops(sh[0], sh[1], sh[2], False)),
        ("matmul", (8192, 8192, 8192), (128, 8192, 8192),
         lambda sh: 2.0 * sh[0] * sh[1] * sh[2]),
    ]


def cpu_task_baselines():
    """Reference CPU path per task (bounded samples, all host threads)."""
    from oracle import reference as O

    torch.set_num_threads(os.cpu_count() or 1)
    out = {}
    for name, full, sample, work in _cpu_samples():
        dtype = "float32" if name in ("vecadd", "reduction") else "bfloat16"
        ins = O.make_inputs(name, sample, dtype, 0, profile="b200")
        O.reference(name, ins)  # warm-up
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            O.reference(name, ins)
            times.append(time.perf_counter() - t0)
        t = sorted(times)[1]
        tensor = name.startswith("attention") or name == "matmul"
        v = work(sample) / t / (1e12 if tensor else 1e9)
        out[f"{name}{list(full)}"] = {
            "value": round(v, 4), "unit": "TFLOP/s" if tensor else "GB/s",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"{list(sample)} {dtype}, median of 3, {t * 1e3:.1f} ms"}
    return out


def run_reference(args, rank, world):
    if rank != 0:
        return None
    # size each step so the whole run stays within about a minute
    v1, _, el1 = cpu_matmul_sample(16, 0.5)
    per_row = 2.0 * SHAPE[1] * SHAPE[2] / (v1 * 1e12)
    budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(max(1, min(SHAPE[0], budget / per_row)))
    from oracle import reference as O

    a, b = O.make_inputs("matmul", SHAPE, "bfloat16", 0, profile="b200")
    a = a[:rows].contiguous()
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        O.reference("matmul", (a, b))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.reference("matmul", (a, b))
    el = time.perf_counter() - t0
    value = args.steps * 2.0 * rows * SHAPE[1] * SHAPE[2] / el / 1e12
    sample = (f"each step: {rows} rows of A (4096x4096 bf16 upcast to fp32) @ B, "
              f"torch CPU fp32 matmul, {os.cpu_count()} threads")
    return {
        "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------ extras
EXTRA_TASKS = [
    ("vecadd", (1 << 24,), {"BLOCK_SIZE": 2048, "num_warps": 4, "dtype": "float32"}),
    ("softmax", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 4, "num_stages": 2,
                                "dtype": "bfloat16"}),
    ("layernorm", (16384, 8192), {"BLOCK_N": 8192, "num_warps": 4, "num_stages": 2,
                                  "dtype": "bfloat16"}),
    ("reduction", (1 << 28,), {"BLOCK_SIZE": 8192, "num_warps": 16, "strategy": "atomic",
                               "dtype": "float32"}),
    ("fused_gelu", (1 << 26,), {"BLOCK_SIZE": 4096, "num_warps": 4, "strategy": "fused",
                                "dtype": "bfloat16"}),
    # two query tiles per CTA (BLOCK_M 256, 8 softmax warps)
    ("attention_causal", (128, 4096, 128), {"BLOCK_M": 256, "BLOCK_N": 128, "num_warps": 8,
                                            "num_stages": 2, "dtype": "bfloat16"}),
    ("attention", (128, 4096, 128), {"BLOCK_M": 256, "BLOCK_N": 128, "num_warps": 8,
                                     "num_stages": 2, "dtype": "bfloat16"}),
    ("matmul", (8192, 8192, 8192), {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 128,
                                    "GROUP_M": 16, "num_warps": 8, "num_stages": 3,
                                    "dtype": "bfloat16"}),
]


def run_extras(world):
    from gpu_optimizer_b200.correctness import NORMWISE_BOUND
    from gpu_optimizer_b200.harness import BenchmarkSettings, CudaBenchmarkEngine
    from gpu_optimizer_b200.tasks import get_task

    eng = CudaBenchmarkEngine(settings=BenchmarkSettings(warmup=5, iterations=20, flush_l2=True,
                                                         cache_inputs=1))
    out = {}
    for name, shape, cfg in EXTRA_TASKS:
        task = get_task(name, "b200")
        try:
            r = eng.benchmark_candidate(task, task.make_candidate(shape, cfg))
            out[f"{name}{list(shape)}"] = {
                "status": r.status, "kernel": r.kernel, "config": cfg,
                "median_ms": round(r.latency.median_ms, 4) if r.ok else None,
                "achieved": round(r.achieved, 1), "unit": r.achieved_unit,
                "frac_of_measured_peak": round(r.roofline_fraction, 4),
                "rel_err_floored": r.correctness.rel_err_floored if r.correctness else None,
                "rel_err_normwise": r.correctness.rel_err_normwise if r.correctness else None,
                "normwise_bound": NORMWISE_BOUND[cfg["dtype"]],
                "error": r.error[:200]}
        except Exception as e:  # keep the headline line alive
            out[f"{name}{list(shape)}"] = {"status": "error", "error": str(e)[:200]}
        torch.cuda.empty_cache()
    return out


SEARCH_SHAPE = (4096, 4096, 4096)
SEARCH_BATCH = 128


def run_search(world, rank):
    """Search throughput: candidates evaluated per second for ONE batch of the
    B200 matmul space at 4096^3 -- 128 distinct candidates drawn once from a
    fixed seed, the same batch at every GPU count -- partitioned over the
    ranks (optimizer/search/loop.py:138-172 with its batch spread over
    devices).  Each candidate goes through the whole harness path with the
    reference's 20 warm-up + 100 timed launches (benchmarks/harness.py:
    102-106,144-203).  Every rank first caches each dtype's inputs and
    reference (a worker keeps them per (task, shape, dtype, seed)); then the
    ranks pull candidates, longest first, from a counter in the gloo group's
    store until the batch is done.  candidates/s = batch / the slowest rank's
    time from the common start to its last result; per-rank busy times show
    any load imbalance."""
    import random

    from gpu_optimizer_b200 import distributed as D
    from gpu_optimizer_b200.dispatch import longest_first
    from gpu_optimizer_b200.harness import BenchmarkSettings, CudaBenchmarkEngine
    from gpu_optimizer_b200.tasks import get_task

    if world > 1:
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    task = get_task("matmul", "b200")
    space = task.param_space(SEARCH_SHAPE)
    rng = random.Random(2024)
    seen, cands = set(), []
    while len(cands) < SEARCH_BATCH:
        c = task.make_candidate(SEARCH_SHAPE, space.sample(rng), "random")
        if c.candidate_id not in seen:
            seen.add(c.candidate_id)
            cands.append(c)
    eng = CudaBenchmarkEngine(settings=BenchmarkSettings())
    for dt in space["dtype"].choices:
        eng.inputs_and_reference(task, SEARCH_SHAPE, dt)
    torch.cuda.synchronize()
    order = longest_first(cands)
    results, st = D.pull_partition(cands, lambda c: eng.benchmark_candidate(task, c), order)
    ranks = st["ranks"]
    wall = max(r["wall_s"] for r in ranks)
    statuses = [r.status for r in results]
    return {"candidates_per_s": round(len(cands) / wall, 2), "candidates": len(cands),
            "seconds": round(wall, 2), "shape": list(SEARCH_SHAPE), "gpus": world,
            "timing": "20 warm-up + 100 timed launches per candidate",
            "dispatch": "shared counter in the gloo group's store, longest first",
            "statuses": {s: statuses.count(s) for s in sorted(set(statuses))},
            "ranks": [{"rank": r["rank"], "count": r["count"], "busy_s": round(r["busy_s"], 2),
                       "wall_s": round(r["wall_s"], 2)} for r in ranks]}


def main():
    args = parse_args()
    rank, world, local = dist_init(args.gpus)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist

            # no barrier: the other ranks leave at once while rank 0 works
            dist.destroy_process_group()
        return
    line = run_ours(args, rank, world, local)
    if not args.no_extras:
        try:
            line["search"] = run_search(world, rank)
        except Exception as e:
            line["search"] = {"error": str(e)[:200]}
        if world == 1:
            line["tasks"] = run_extras(world)
    if rank == 0 and world == 1 and not args.no_extras:
        line["cpu_baseline"] = cpu_baseline()
        try:
            cpu = cpu_task_baselines()
            for k, v in cpu.items():
                if k in line.get("tasks", {}):
                    line["tasks"][k]["cpu_baseline"] = v
        except Exception as e:  # keep the headline line alive
            line["cpu_task_baselines_error"] = str(e)[:200]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
