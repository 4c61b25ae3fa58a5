"""Benchmark harness: compile, validate and time candidates on a B200.

Mirrors the reference's ``CudaBenchmarkEngine`` (benchmarks/harness.py:133-218):
the same statuses, ``LatencyStats``, ``BenchmarkResult`` and
``BenchmarkSettings``, and the same per-candidate sequence (inputs -> build
-> warm compile -> validate against the task's torch reference -> CUDA-event
timing -> GFLOP/s), with the kernel layer being this package's runner.

Additions for B200 measurement:

* inputs and reference outputs are cached per (task, profile, shape, dtype,
  seed) instead of being regenerated for every candidate (the reference
  regenerates them, harness.py:167);
* an optional L2 flush (write of a buffer larger than the 126 MB L2) between
  timed iterations, outside the timed event pair;
* roofline fields: achieved GB/s or TFLOP/s of the task's algorithmic work
  and its fraction of a peak, plus the device index and worker id.
"""

from __future__ import annotations

import logging
import time
from collections import OrderedDict
from collections.abc import Sequence
from dataclasses import asdict, dataclass, field

import numpy as np
import torch

from .correctness import CorrectnessReport, check_correctness
from .space import Candidate
from .tasks import Task

logger = logging.getLogger(__name__)

STATUS_OK = "ok"
STATUS_COMPILE_ERROR = "compile_error"
STATUS_RUNTIME_ERROR = "runtime_error"
STATUS_INCORRECT = "incorrect"


@dataclass
class LatencyStats:
    mean_ms: float
    median_ms: float
    p50_ms: float
    p90_ms: float
    p99_ms: float
    std_ms: float
    min_ms: float
    iterations: int

    @classmethod
    def from_samples(cls, samples_ms: Sequence[float]) -> LatencyStats:
        arr = np.asarray(samples_ms, dtype=np.float64)
        return cls(
            mean_ms=float(arr.mean()), median_ms=float(np.median(arr)),
            p50_ms=float(np.percentile(arr, 50)), p90_ms=float(np.percentile(arr, 90)),
            p99_ms=float(np.percentile(arr, 99)),
            std_ms=float(arr.std(ddof=1)) if arr.size > 1 else 0.0,
            min_ms=float(arr.min()), iterations=int(arr.size))


@dataclass
class BenchmarkResult:
    candidate_id: str
    task: str
    shape: tuple[int, ...]
    config: dict
    engine: str
    status: str
    gpu_name: str
    correct: bool = False
    correctness_mode: str = "none"
    correctness: CorrectnessReport | None = None
    latency: LatencyStats | None = None
    throughput_gflops: float = 0.0
    memory_bytes: int = 0
    compile_time_s: float = 0.0
    warmup: int = 0
    provenance: str = "manual"
    parent_id: str | None = None
    error: str = ""
    timestamp: float = field(default_factory=time.time)
    # B200 additions
    achieved: float = 0.0           # GB/s (hbm-bound tasks) or TFLOP/s (tensor-bound)
    achieved_unit: str = ""
    roofline_fraction: float = 0.0  # achieved / peak
    kernel: str = ""
    device_index: int = 0
    worker_id: int = 0

    @property
    def ok(self) -> bool:
        return self.status == STATUS_OK

    @property
    def latency_ms(self) -> float:
        return self.latency.median_ms if (self.ok and self.latency) else float("inf")

    def to_dict(self) -> dict:
        d = asdict(self)
        d["shape"] = list(self.shape)
        return d


@dataclass
class BenchmarkSettings:
    warmup: int = 20
    iterations: int = 100
    seed: int = 0
    flush_l2: bool = False
    # input sets (with their reference outputs) kept resident per engine: a
    # search draws every dtype of a task, so keep all of them
    cache_inputs: int = 8
    # time replays of a CUDA graph holding one call instead of the calls
    # themselves: removes host launch overhead from small kernels' numbers
    cuda_graph: bool = False


class L2Flusher:
    """Overwrites a buffer larger than L2 to evict cached operands."""

    def __init__(self, device: torch.device, nbytes: int | None = None) -> None:
        if nbytes is None:
            l2 = int(getattr(torch.cuda.get_device_properties(device), "L2_cache_size",
                             128 << 20))
            nbytes = 2 * l2
        self.buf = torch.empty(nbytes // 4, dtype=torch.int32, device=device)

    def __call__(self) -> None:
        self.buf.fill_(0)


def default_peaks() -> dict:
    """Peak denominators: the pool's measured peaks when present, else fallbacks."""
    import json
    from pathlib import Path

    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                    "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained",
                                                         d["bf16_tflops"])),
                    "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class CudaBenchmarkEngine:
    """Measures candidates on one CUDA device with CUDA-event timing."""

    label = "cuda"

    def __init__(self, hardware=None, settings: BenchmarkSettings | None = None,
                 device: int | None = None, worker_id: int = 0) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("CudaBenchmarkEngine requires a CUDA device")
        self.settings = settings or BenchmarkSettings()
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        torch.cuda.set_device(self.device)
        if hardware is None:
            from .hardware import detect_hardware

            hardware = detect_hardware(self.device.index)
        self.hardware = hardware
        self.worker_id = worker_id
        self.peaks = default_peaks()
        self._cache: OrderedDict = OrderedDict()
        self._flusher: L2Flusher | None = None

    # ------------------------------------------------------------- inputs
    def inputs_and_reference(self, task: Task, shape, dtype: str):
        key = (task.name, getattr(task, "profile", type(task).__module__), tuple(shape), dtype,
               self.settings.seed)
        hit = self._cache.get(key)
        if hit is not None:
            self._cache.move_to_end(key)
            return hit
        while len(self._cache) >= max(1, self.settings.cache_inputs):
            self._cache.popitem(last=False)
            torch.cuda.empty_cache()
        inputs = task.make_inputs(shape, dtype, str(self.device), self.settings.seed)
        ref = task.reference(*inputs)
        self._cache[key] = (inputs, ref)
        return inputs, ref

    # ------------------------------------------------------------- timing
    def _time_callable(self, fn, graph_ok: bool = True) -> LatencyStats:
        s = self.settings
        for _ in range(s.warmup):
            fn()
        torch.cuda.synchronize(self.device)
        if s.cuda_graph and graph_ok:
            # capture one call (every lazy setup already ran in the warm-up)
            # on a side stream, then time graph replays on the current one
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                with torch.cuda.graph(g, stream=side):
                    fn()
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            fn = g.replay
            fn()
            torch.cuda.synchronize(self.device)
        if s.flush_l2 and self._flusher is None:
            self._flusher = L2Flusher(self.device)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(s.iterations)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(s.iterations)]
        for i in range(s.iterations):
            if self._flusher is not None and s.flush_l2:
                self._flusher()
            starts[i].record()
            fn()
            ends[i].record()
        torch.cuda.synchronize(self.device)
        return LatencyStats.from_samples([starts[i].elapsed_time(ends[i])
                                          for i in range(s.iterations)])

    def _roofline(self, task: Task, shape, dtype: str, median_ms: float):
        if not hasattr(task, "roofline_work"):
            # a task object of the reference's own registry: the same task
            # of this package's registry knows the algorithmic work
            from .tasks import get_task

            task = get_task(task.name)
        work = task.roofline_work(shape, dtype)
        if task.roofline_bound == "tensor":
            ach = work / (median_ms * 1e-3) / 1e12
            return ach, "TFLOP/s", ach / self.peaks["bf16_tflops"]
        ach = work / (median_ms * 1e-3) / 1e9
        return ach, "GB/s", ach / self.peaks["hbm_gbs"]

    # --------------------------------------------------------- candidates
    def benchmark_candidate(self, task: Task, candidate: Candidate) -> BenchmarkResult:
        from .runner import KernelBuildError, build_callable, check_device_status, warm_compile

        shape, config = candidate.shape, candidate.config
        base = dict(candidate_id=candidate.candidate_id, task=task.name, shape=shape,
                    config=dict(config), engine=self.label, gpu_name=self.hardware.name,
                    provenance=candidate.provenance, parent_id=candidate.parent_id,
                    warmup=self.settings.warmup, device_index=self.device.index or 0,
                    worker_id=self.worker_id)
        try:
            inputs, ref = self.inputs_and_reference(task, shape, candidate.dtype)
        except Exception as e:
            return BenchmarkResult(**base, status=STATUS_RUNTIME_ERROR,
                                   error=f"input generation failed: {e}")
        try:
            kc = build_callable(task.name, shape, config, inputs)
            compile_time = warm_compile(kc)
        except KernelBuildError as e:
            return BenchmarkResult(**base, status=STATUS_COMPILE_ERROR, error=str(e))
        base["kernel"] = kc.launch.get("kernel", "")
        try:
            out = kc.fn()
            check_device_status()
            rtol, atol = task.tolerance(candidate.dtype)
            report = check_correctness(out, ref, rtol, atol)
        except Exception as e:
            return BenchmarkResult(**base, status=STATUS_RUNTIME_ERROR,
                                   compile_time_s=compile_time, error=str(e))
        if not report.passed:
            return BenchmarkResult(**base, status=STATUS_INCORRECT, correct=False,
                                   correctness_mode="device", correctness=report,
                                   compile_time_s=compile_time,
                                   error=f"correctness: {report.summary()}")
        torch.cuda.reset_peak_memory_stats(self.device)
        try:
            stats = self._time_callable(kc.fn)
            check_device_status()
        except Exception as e:
            return BenchmarkResult(**base, status=STATUS_RUNTIME_ERROR,
                                   compile_time_s=compile_time, error=str(e))
        mem = int(torch.cuda.max_memory_allocated(self.device))
        gflops = task.flops(shape) / (stats.median_ms * 1e-3) / 1e9
        ach, unit, frac = self._roofline(task, shape, candidate.dtype, stats.median_ms)
        return BenchmarkResult(**base, status=STATUS_OK, correct=True,
                               correctness_mode="device", correctness=report, latency=stats,
                               throughput_gflops=gflops, memory_bytes=mem,
                               compile_time_s=compile_time, achieved=ach, achieved_unit=unit,
                               roofline_fraction=frac)

    def benchmark_baseline(self, task: Task, shape: Sequence[int],
                           dtype: str = "float32") -> BenchmarkResult:
        shape = tuple(int(x) for x in shape)
        inputs, _ = self.inputs_and_reference(task, shape, dtype)
        stats = self._time_callable(lambda: task.baseline(*inputs), graph_ok=False)
        gflops = task.flops(shape) / (stats.median_ms * 1e-3) / 1e9
        ach, unit, frac = self._roofline(task, shape, dtype, stats.median_ms)
        return BenchmarkResult(
            candidate_id=f"baseline-torch-{task.name}", task=task.name, shape=shape,
            config={"dtype": dtype, "baseline": "torch"}, engine=self.label,
            gpu_name=self.hardware.name, status=STATUS_OK, correct=True,
            correctness_mode="device", latency=stats, throughput_gflops=gflops,
            warmup=self.settings.warmup, provenance="baseline", achieved=ach,
            achieved_unit=unit, roofline_fraction=frac, device_index=self.device.index or 0,
            worker_id=self.worker_id)
