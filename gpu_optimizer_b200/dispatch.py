"""Candidate evaluation sharded over the GPUs of one box.

Candidate evaluation is embarrassingly parallel, so the search's benchmark
batches are partitioned across devices with no collective and no tensor
crossing NVLink (the reference evaluates one candidate at a time on one
device, optimizer/search/loop.py:138-172).  ``MultiDeviceEvaluator`` runs
one worker process per GPU (``spawn`` start method, the device pinned with
CUDA_VISIBLE_DEVICES before CUDA initialises); the parent hands each idle
worker the next candidate, so faster devices take more work, and results
are returned in proposal order.  Each worker keeps its own engine, so inputs and
reference outputs are generated once per (task, shape, dtype, seed) per
device.

Failure handling (host side only): a per-candidate deadline; a worker that
exceeds it, or whose process dies, is killed and respawned, and its
candidate is recorded as ``runtime_error`` — the search continues.
"""

from __future__ import annotations

import multiprocessing as mp
import multiprocessing.connection as mpc
import os
import time
import traceback
from collections.abc import Callable, Sequence
from dataclasses import dataclass

from .harness import STATUS_RUNTIME_ERROR, BenchmarkResult, BenchmarkSettings
from .space import Candidate

EngineFactory = Callable[[int, BenchmarkSettings, int], object]


def relative_cost(cand: Candidate) -> float:
    """Relative evaluation cost of a candidate, from the host-side plan:
    CUDA-core tiles run longest, tf32 tensor-core tiles next, 16-bit ones
    least; a candidate the planner refuses costs nothing (compile_error).
    A CUDA-core tile of a x b outputs per thread does a*b FMAs per a + b
    operands it reads from shared memory, so its time per FLOP scales as
    (a + b) / (a * b); the register-prefetch form (no cp.async pipeline)
    is slower again.  A tensor-core tile of BLOCK_M 32 runs the M=64 MMA
    with half of its rows unused, so it counts twice."""
    import re

    from .runner import KernelBuildError, compile_module

    try:
        kernel = compile_module(cand.task, cand.shape, cand.config).resources()["kernel"]
    except KernelBuildError:
        return 0.0
    if "simt" in kernel:
        m = re.search(r"<(\d+)x(\d+) per thread>", kernel)
        a, b = (int(m.group(1)), int(m.group(2))) if m else (8, 8)
        cost = 120.0 * (a + b) / (a * b)  # 30 for an 8 x 8 tile
        return cost if "async" in kernel else 1.3 * cost
    cost = 3.0 if cand.config.get("dtype") == "tf32" else 1.0
    return cost * max(1.0, 64.0 / float(cand.config.get("BLOCK_M", 64)))


def longest_first(candidates: Sequence[Candidate]) -> list[int]:
    """Dispatch order for a partitioned batch: most expensive first, so
    that the devices finish together (longest-processing-time order)."""
    costs = [relative_cost(c) for c in candidates]
    return sorted(range(len(candidates)), key=lambda i: -costs[i])


def cuda_engine_factory(device: int, settings: BenchmarkSettings, worker_id: int):
    """Default factory: a CudaBenchmarkEngine on the (only) visible device."""
    from .harness import CudaBenchmarkEngine

    return CudaBenchmarkEngine(settings=settings, device=0, worker_id=worker_id)


def _error_result(cand: Candidate, msg: str, worker_id: int, device: int) -> BenchmarkResult:
    return BenchmarkResult(candidate_id=cand.candidate_id, task=cand.task, shape=cand.shape,
                           config=dict(cand.config), engine="cuda",
                           status=STATUS_RUNTIME_ERROR, gpu_name="", provenance=cand.provenance,
                           parent_id=cand.parent_id, error=msg, worker_id=worker_id,
                           device_index=device)


def _worker_main(worker_id: int, device: int, pin_device: bool, factory: EngineFactory,
                 settings: BenchmarkSettings, profile: str, conn, host_threads: int = 0) -> None:
    if pin_device:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(device)
    if host_threads > 0:
        # the host cores are shared by all workers: input generation and
        # CPU-side reference work must not oversubscribe them
        import torch

        torch.set_num_threads(host_threads)
    from .tasks import get_task

    engine, init_err = None, ""
    try:
        engine = factory(device, settings, worker_id)
    except Exception as e:  # keep serving, report every candidate as failed
        init_err = f"engine init failed: {e}"
    conn.send("ready")
    while True:
        try:
            item = conn.recv()
        except EOFError:
            return
        if item is None:
            return
        task_name, shape, config, provenance, parent = item
        cand = Candidate(task=task_name, shape=tuple(shape), config=dict(config),
                         provenance=provenance, parent_id=parent)
        try:
            if engine is None:
                raise RuntimeError(init_err)
            res = engine.benchmark_candidate(get_task(task_name, profile), cand)
            res.worker_id = worker_id
            res.device_index = device
        except Exception as e:
            res = _error_result(cand, f"worker exception: {e}\n{traceback.format_exc()[-400:]}",
                                worker_id, device)
        conn.send(res)


@dataclass
class _Worker:
    wid: int
    device: int
    proc: mp.Process
    conn: object
    ready: bool = False
    busy_idx: int | None = None
    busy_since: float = 0.0


class MultiDeviceEvaluator:
    """Evaluate candidate batches on N devices, one worker process each.

    Each worker has a private duplex pipe: the parent hands it one candidate
    at a time and therefore always knows which candidate a worker holds, and
    no lock is shared between workers, so one that dies cannot block the
    others.
    """

    def __init__(self, devices: Sequence[int], settings: BenchmarkSettings | None = None,
                 profile: str = "reference", factory: EngineFactory = cuda_engine_factory,
                 pin_devices: bool = True, candidate_timeout_s: float = 300.0) -> None:
        if not devices:
            raise ValueError("need at least one device")
        self.devices = list(devices)
        self.settings = settings or BenchmarkSettings()
        self.profile = profile
        self.factory = factory
        self.pin_devices = pin_devices
        self.timeout = candidate_timeout_s
        self._ctx = mp.get_context("spawn")
        self.respawns = 0
        self._workers: list[_Worker] = [self._spawn(i, d) for i, d in enumerate(self.devices)]

    def _spawn(self, wid: int, device: int) -> _Worker:
        parent, child = self._ctx.Pipe(duplex=True)
        threads = max(1, (os.cpu_count() or 1) // len(self.devices))
        p = self._ctx.Process(target=_worker_main, daemon=True,
                              args=(wid, device, self.pin_devices, self.factory, self.settings,
                                    self.profile, child, threads))
        p.start()
        child.close()
        return _Worker(wid, device, p, parent)

    def _replace(self, w: _Worker) -> None:
        if w.proc.is_alive():
            w.proc.kill()
        w.proc.join(timeout=10)
        try:
            w.conn.close()
        except OSError:
            pass
        self.respawns += 1
        self._workers[w.wid] = self._spawn(w.wid, w.device)

    def wait_ready(self, timeout_s: float = 600.0) -> bool:
        """Block until every worker has built its engine (or the deadline)."""
        t0 = time.time()
        while time.time() - t0 < timeout_s:
            pending = [w for w in self._workers if not w.ready]
            if not pending:
                return True
            for c in mpc.wait([w.conn for w in pending], timeout=0.2):
                w = next(x for x in pending if x.conn is c)
                try:
                    if w.conn.recv() == "ready":
                        w.ready = True
                except (EOFError, OSError):
                    self._replace(w)
            for w in pending:
                if not w.ready and not w.proc.is_alive():
                    self._replace(w)
        return all(w.ready for w in self._workers)

    def evaluate(self, candidates: Sequence[Candidate],
                 order: Sequence[int] | None = None) -> list[BenchmarkResult]:
        """Results in the order of ``candidates``.

        ``order`` is the dispatch order (indices into ``candidates``,
        default the proposal order); handing out the longest candidates
        first lets the devices finish together.  A candidate's deadline
        starts when a ready worker receives it; a worker that exits or
        misses the deadline is replaced and its candidate recorded as
        runtime_error.
        """
        n = len(candidates)
        results: list[BenchmarkResult | None] = [None] * n
        order = list(range(n)) if order is None else list(order)
        if sorted(order) != list(range(n)):
            raise ValueError("order must be a permutation of the candidate indices")
        todo = order[::-1]
        done = 0
        respawn_budget = 10 * len(self._workers) + n

        def assign(w: _Worker) -> None:
            if not todo or not w.ready or w.busy_idx is not None:
                return
            i = todo.pop()
            c = candidates[i]
            try:
                w.conn.send((c.task, list(c.shape), dict(c.config), c.provenance, c.parent_id))
            except OSError:
                todo.append(i)
                fail(w, "worker died")
                return
            w.busy_idx, w.busy_since = i, time.time()

        def fail(w: _Worker, why: str) -> None:
            nonlocal done
            if w.busy_idx is not None and results[w.busy_idx] is None:
                results[w.busy_idx] = _error_result(candidates[w.busy_idx], why, w.wid, w.device)
                done += 1
            w.busy_idx = None
            self._replace(w)

        for w in self._workers:
            assign(w)
        while done < n:
            if self.respawns > respawn_budget:  # the pool cannot start workers
                for i in todo:
                    results[i] = _error_result(candidates[i], "worker pool failing", -1, -1)
                    done += 1
                todo.clear()
                break
            watch = [w for w in self._workers if w.busy_idx is not None or not w.ready]
            ready = mpc.wait([w.conn for w in watch], timeout=0.2) if watch else []
            for w in watch:
                if w.conn in ready:
                    try:
                        msg = w.conn.recv()
                    except (EOFError, OSError):
                        fail(w, "worker died")
                        continue
                    if isinstance(msg, str) and msg == "ready":
                        w.ready = True
                    elif w.busy_idx is not None:
                        if results[w.busy_idx] is None:
                            results[w.busy_idx] = msg
                            done += 1
                        w.busy_idx = None
                elif not w.proc.is_alive():
                    fail(w, "worker died")
                elif w.busy_idx is not None and time.time() - w.busy_since > self.timeout:
                    fail(w, f"timeout after {self.timeout:.0f} s")
            for w in self._workers:
                assign(w)
        return results  # type: ignore[return-value]

    def close(self) -> None:
        for w in self._workers:
            try:
                w.conn.send(None)
            except OSError:
                pass
        for w in self._workers:
            w.proc.join(timeout=10)
            if w.proc.is_alive():
                w.proc.kill()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class SingleDeviceEvaluator:
    """In-process evaluation on one engine (the reference's sequential loop)."""

    def __init__(self, engine, profile: str = "reference") -> None:
        self.engine = engine
        self.profile = profile

    def evaluate(self, candidates: Sequence[Candidate]) -> list[BenchmarkResult]:
        from .tasks import get_task

        return [self.engine.benchmark_candidate(get_task(c.task, self.profile), c)
                for c in candidates]

    def close(self) -> None:
        pass
