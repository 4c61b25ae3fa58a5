"""Sharded candidate evaluation: worker pool, failure handling, gloo ranks.

All failures are made on the host (an exception, a worker process that
exits, a worker that sleeps past its deadline); no GPU is used.
"""

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as tmp

import fake_engine
from gpu_optimizer_b200 import distributed as D
from gpu_optimizer_b200.dispatch import MultiDeviceEvaluator
from gpu_optimizer_b200.search import (GridSearcher, RandomSearcher, SearchLoop,
                                       compute_reward)
from gpu_optimizer_b200.space import Candidate, ParamSpace, ParamSpec
from gpu_optimizer_b200.harness import BenchmarkResult, LatencyStats


def cands(modes):
    return [Candidate("vecadd", (1024,), {"BLOCK_SIZE": 2 ** (i % 8 + 1), "mode": m,
                                          "i": i}) for i, m in enumerate(modes)]


def test_results_come_back_in_proposal_order():
    with MultiDeviceEvaluator([0, 1, 2], factory=fake_engine.factory,
                              pin_devices=False) as ev:
        assert ev.wait_ready(120)
        cs = cands(["ok"] * 17)
        res = ev.evaluate(cs)
        # a dispatch order (longest first) changes who runs what, not the
        # order of the results
        res2 = ev.evaluate(cs, order=list(range(17))[::-1])
        with pytest.raises(ValueError):
            ev.evaluate(cs, order=[0, 0])
    assert [r.candidate_id for r in res] == [c.candidate_id for c in cs]
    assert [r.candidate_id for r in res2] == [c.candidate_id for c in cs]
    assert all(r.status == "ok" for r in res)
    assert len({r.worker_id for r in res}) > 1  # work was spread


def test_worker_exception_crash_and_hang_are_contained():
    with MultiDeviceEvaluator([0, 1], factory=fake_engine.factory, pin_devices=False,
                              candidate_timeout_s=3.0) as ev:
        cs = cands(["ok", "raise", "ok", "crash", "ok", "hang", "ok", "ok"])
        res = ev.evaluate(cs)
        statuses = [r.status for r in res]
        assert statuses == ["ok", "runtime_error", "ok", "runtime_error", "ok",
                            "runtime_error", "ok", "ok"]
        assert "synthetic failure" in res[1].error
        assert "died" in res[3].error and "timeout" in res[5].error
        assert ev.respawns >= 2
        # the pool still serves after the failures
        again = ev.evaluate(cands(["ok"] * 4))
        assert all(r.status == "ok" for r in again)


def test_search_loop_dedupes_and_tracks_best():
    space = ParamSpace([ParamSpec("BLOCK_SIZE", (2, 4, 8, 16)), ParamSpec("mode", ("ok",))])
    with MultiDeviceEvaluator([0, 1], factory=fake_engine.factory, pin_devices=False) as ev:
        out = SearchLoop("vecadd", (1024,), GridSearcher("vecadd", (1024,), space), ev,
                         baseline_ms=1.0, max_evaluations=10, batch_size=3).run()
    assert out.candidates_evaluated == 4  # grid exhausted, no duplicates
    assert out.best_candidate.config["BLOCK_SIZE"] == 16
    rs = RandomSearcher("vecadd", (1024,), space, seed=0).propose(3)
    assert len(rs) == 3


def test_reward_matches_reference_rules():
    base = dict(candidate_id="x", task="t", shape=(1,), config={}, engine="cuda",
                gpu_name="g")
    ok = BenchmarkResult(**base, status="ok", latency=LatencyStats.from_samples([0.5, 0.5]))
    assert compute_reward(ok, 1.0) == pytest.approx(1.0)
    assert compute_reward(BenchmarkResult(**base, status="compile_error"), 1.0) == -0.5
    assert compute_reward(BenchmarkResult(**base, status="runtime_error"), 1.0) == -0.8
    assert compute_reward(BenchmarkResult(**base, status="incorrect"), 1.0) == -1.0


def test_shard_unshard_roundtrip():
    items = list(range(23))
    parts = [D.shard(items, r, 4) for r in range(4)]
    assert sorted(sum(parts, [])) == items
    assert D.unshard(parts, len(items)) == items


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        items = list(range(10))
        mine = D.shard(items, rank, world)
        # each rank "evaluates" its shard; time differs per rank
        t = 1.0 + rank
        assert D.reduce_scalar(t, "max") == world
        assert D.reduce_scalar(len(mine), "sum") == len(items)
        parts = D.gather_objects([x * 10 for x in mine])
        assert D.unshard(parts, len(items)) == [x * 10 for x in items]
        D.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_world_size_two_sharding():
    tmp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)


def _slow_square(item):
    import time

    time.sleep(item[1])
    return item[0] * item[0]


def _pull_main(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # one long item and many short ones: the rank that draws the long one
        # takes few others, so both finish near the same time
        items = [(i, 0.6 if i == 3 else 0.05) for i in range(14)]
        order = sorted(range(len(items)), key=lambda i: -items[i][1])  # longest first
        out, st = D.pull_partition(items, _slow_square, order)
        assert out == [i * i for i in range(14)]
        ranks = st["ranks"]
        assert [r["rank"] for r in ranks] == list(range(world))
        assert sum(r["count"] for r in ranks) == len(items)
        assert all(r["count"] >= 1 for r in ranks)
        long_rank = 0 if ranks[0]["busy_s"] > ranks[1]["busy_s"] else 1
        assert ranks[long_rank]["count"] < ranks[1 - long_rank]["count"]
        # a second batch on the same group uses a fresh counter
        out2, _ = D.pull_partition([(i, 0.0) for i in range(5)], _slow_square)
        assert out2 == [i * i for i in range(5)]
        D.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_world_size_two_pull_partition():
    """The search batch is split by a shared counter in the group's store."""
    tmp.spawn(_pull_main, args=(2, _free_port()), nprocs=2, join=True)


def test_pull_partition_without_a_group():
    out, st = D.pull_partition([(2, 0.0), (3, 0.0)], _slow_square, [1, 0])
    assert out == [4, 9] and st["ranks"][0]["count"] == 2


def test_longest_first_order_from_the_plan():
    from gpu_optimizer_b200.dispatch import longest_first, relative_cost

    shape = (4096, 4096, 4096)
    base = {"BLOCK_K": 64, "GROUP_M": 8, "num_warps": 8, "num_stages": 3}
    tc = Candidate("matmul", shape, {**base, "BLOCK_M": 128, "BLOCK_N": 256, "dtype": "bfloat16"})
    refused = Candidate("matmul", shape, {**base, "BLOCK_M": 256, "BLOCK_N": 256,
                                          "BLOCK_K": 128, "num_stages": 6, "dtype": "bfloat16"})
    simt = Candidate("matmul", shape, {**base, "BLOCK_M": 64, "BLOCK_N": 64, "dtype": "float32"})
    tf32 = Candidate("matmul", shape, {**base, "BLOCK_M": 128, "BLOCK_N": 128, "dtype": "tf32"})
    assert relative_cost(refused) == 0.0
    assert longest_first([tc, refused, simt, tf32]) == [2, 3, 0, 1]
    # a BLOCK_M 32 tensor-core tile uses half of each M=64 MMA
    tc32 = Candidate("matmul", shape, {**base, "BLOCK_M": 32, "BLOCK_N": 128,
                                       "dtype": "bfloat16"})
    assert relative_cost(tc32) == 2.0 * relative_cost(tc)
    assert longest_first([tc, tc32]) == [1, 0]
