"""Search loop with batch evaluation sharded over devices.

Keeps the reference's loop semantics (optimizer/search/loop.py:100-197):
dedupe by candidate id, reward per result (optimizer/rewards/reward.py:39-65),
best tracking, observe() after each batch.  The one change is where the
batch goes: the deduped batch is handed to an evaluator (one device
in-process, or ``MultiDeviceEvaluator`` across the box's GPUs) and results
come back in proposal order, so a searcher sees exactly the sequence the
sequential loop would produce.

Random and grid proposers are provided for throughput runs and tests; the
reference's model-based searchers plug in through the same
``propose`` / ``observe`` / ``finalize`` interface.
"""

from __future__ import annotations

import math
import random
import time
from dataclasses import dataclass, field

from .harness import (
    STATUS_COMPILE_ERROR,
    STATUS_INCORRECT,
    STATUS_OK,
    STATUS_RUNTIME_ERROR,
    BenchmarkResult,
)
from .space import Candidate, ParamSpace


@dataclass
class RewardConfig:
    """optimizer/rewards/reward.py:22-36."""

    mode: str = "log_speedup"
    correctness_penalty: float = 1.0
    compile_penalty: float = 0.5
    runtime_penalty: float = 0.8
    memory_limit_bytes: int | None = None
    memory_penalty: float = 0.5
    clip: float | None = 8.0

    def __post_init__(self) -> None:
        if self.mode not in ("speedup", "log_speedup"):
            raise ValueError(f"unknown reward mode {self.mode!r}")


def compute_reward(result: BenchmarkResult, baseline_ms: float,
                   cfg: RewardConfig | None = None) -> float:
    """Status -> penalty, ok -> log2 (or linear) speedup (reward.py:39-65)."""
    cfg = cfg or RewardConfig()
    if baseline_ms <= 0:
        raise ValueError("baseline_ms must be positive")
    if result.status == STATUS_COMPILE_ERROR:
        r = -cfg.compile_penalty
    elif result.status == STATUS_RUNTIME_ERROR:
        r = -cfg.runtime_penalty
    elif result.status == STATUS_INCORRECT:
        r = -cfg.correctness_penalty
    elif result.status == STATUS_OK:
        speedup = baseline_ms / result.latency.median_ms
        r = math.log2(speedup) if cfg.mode == "log_speedup" else speedup - 1.0
        if cfg.memory_limit_bytes is not None and result.memory_bytes > cfg.memory_limit_bytes:
            r -= cfg.memory_penalty
    else:
        raise ValueError(f"unknown result status {result.status!r}")
    if cfg.clip is not None:
        r = max(-cfg.clip, min(cfg.clip, r))
    return float(r)


class RandomSearcher:
    name = "random"

    def __init__(self, task: str, shape, space: ParamSpace, seed: int = 0) -> None:
        self.task, self.shape, self.space = task, tuple(shape), space
        self.rng = random.Random(seed)

    def propose(self, n: int) -> list[Candidate]:
        return [Candidate(self.task, self.shape, self.space.sample(self.rng),
                          provenance="random") for _ in range(n)]

    def observe(self, observations) -> None:
        pass

    def finalize(self) -> None:
        pass


class GridSearcher(RandomSearcher):
    """Shuffled full grid (optimizer/search/grid_search.py:13-28)."""

    name = "grid"

    def __init__(self, task: str, shape, space: ParamSpace, seed: int = 0) -> None:
        super().__init__(task, shape, space, seed)
        self._grid = space.grid()
        self.rng.shuffle(self._grid)
        self._pos = 0

    def propose(self, n: int) -> list[Candidate]:
        out = self._grid[self._pos:self._pos + n]
        self._pos += len(out)
        return [Candidate(self.task, self.shape, c, provenance="grid") for c in out]


@dataclass
class SearchOutcome:
    task: str
    shape: tuple[int, ...]
    best_candidate: Candidate | None
    best_result: BenchmarkResult | None
    baseline_ms: float
    candidates_evaluated: int
    compile_success_rate: float
    duration_s: float
    eval_seconds: float
    history: list[dict] = field(default_factory=list)

    @property
    def candidates_per_s(self) -> float:
        return self.candidates_evaluated / self.eval_seconds if self.eval_seconds else 0.0


class SearchLoop:
    """Propose -> (sharded) benchmark -> reward -> observe."""

    def __init__(self, task: str, shape, searcher, evaluator, baseline_ms: float,
                 max_evaluations: int = 200, batch_size: int = 8,
                 reward_config: RewardConfig | None = None) -> None:
        self.task, self.shape = task, tuple(shape)
        self.searcher, self.evaluator = searcher, evaluator
        self.baseline_ms = baseline_ms
        self.max_evaluations, self.batch_size = max_evaluations, batch_size
        self.reward_config = reward_config or RewardConfig()

    def run(self) -> SearchOutcome:
        t0 = time.time()
        seen: set[str] = set()
        best: tuple[Candidate, BenchmarkResult] | None = None
        evaluated = compiled = 0
        eval_s = 0.0
        history: list[dict] = []
        while evaluated < self.max_evaluations:
            want = min(self.batch_size, self.max_evaluations - evaluated)
            batch = self.searcher.propose(want)
            if not batch:
                break
            fresh = []
            for c in batch:
                if c.candidate_id not in seen:
                    seen.add(c.candidate_id)
                    fresh.append(c)
            if not fresh:
                continue
            te = time.time()
            results = self.evaluator.evaluate(fresh)
            eval_s += time.time() - te
            obs = []
            for cand, res in zip(fresh, results):
                reward = compute_reward(res, self.baseline_ms, self.reward_config)
                evaluated += 1
                compiled += res.status != STATUS_COMPILE_ERROR
                if res.ok and (best is None or res.latency_ms < best[1].latency_ms):
                    best = (cand, res)
                obs.append((cand, res, reward))
                history.append({"iteration": evaluated, "candidate_id": cand.candidate_id,
                                "config": cand.config, "status": res.status,
                                "latency_ms": res.latency_ms if res.ok else None,
                                "reward": reward, "worker": res.worker_id})
            self.searcher.observe(obs)
        self.searcher.finalize()
        return SearchOutcome(self.task, self.shape, best[0] if best else None,
                             best[1] if best else None, self.baseline_ms, evaluated,
                             compiled / evaluated if evaluated else 0.0, time.time() - t0,
                             eval_s, history)
