"""Host-only stand-in engines for dispatcher tests (no GPU is touched).

The behaviour is chosen by the candidate's config["mode"]:
ok -> a result with latency derived from BLOCK_SIZE; raise -> exception;
crash -> the worker process exits; hang -> the worker sleeps past the deadline.
"""

import os
import time

from gpu_optimizer_b200.harness import BenchmarkResult, LatencyStats


class FakeEngine:
    def __init__(self, device, settings, worker_id):
        self.device, self.worker_id = device, worker_id

    def benchmark_candidate(self, task, cand):
        mode = cand.config.get("mode", "ok")
        if mode == "raise":
            raise ValueError("synthetic failure")
        if mode == "crash":
            os._exit(3)
        if mode == "hang":
            time.sleep(60)
        time.sleep(0.01)
        ms = 1.0 / float(cand.config.get("BLOCK_SIZE", 1))
        return BenchmarkResult(candidate_id=cand.candidate_id, task=cand.task, shape=cand.shape,
                               config=dict(cand.config), engine="fake", status="ok",
                               gpu_name="fake", correct=True,
                               latency=LatencyStats.from_samples([ms, ms]),
                               provenance=cand.provenance)


def factory(device, settings, worker_id):
    return FakeEngine(device, settings, worker_id)
