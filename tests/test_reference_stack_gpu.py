"""The reference's own stack, unchanged, with this backend as its kernel
layer (``compiler.triton.runner`` swapped for ``gpu_optimizer_b200.runner``,
the one-line switch at benchmarks/harness.py:160):

* the reference's real-hardware contract (tests/test_triton_gpu.py:32-70):
  its ``CudaBenchmarkEngine`` on its GPU test shapes, the default config
  and six random configs per task -- every status ``ok`` or
  ``compile_error``, correct on the device;
* the reference's ``SearchLoop`` with its ``RandomSearcher`` and its
  results database: 16 matmul candidates through the reference's engine,
  and 16 through this package's B200 engine with the B200 fields stored in
  the added table.
"""

import random

import pytest

import reference_stack

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not reference_stack.available(),
                                 reason="reference not installed under baseline/_ref")]


@pytest.fixture(scope="module", autouse=True)
def ref():
    reference_stack.activate()


GPU_SHAPES = {  # tests/test_triton_gpu.py:21-29
    "matmul": (384, 320, 288), "vecadd": (1_000_003,), "reduction": (1_000_003,),
    "softmax": (256, 1000), "layernorm": (256, 1000), "fused_elementwise": (1_000_003,),
    "attention": (4, 512, 64),
}


@pytest.fixture(scope="module")
def engine():
    from benchmarks.harness import BenchmarkSettings, CudaBenchmarkEngine
    from hardware.gpu_info import detect_hardware

    return CudaBenchmarkEngine(detect_hardware(), BenchmarkSettings(warmup=3, iterations=10))


@pytest.mark.parametrize("name", sorted(GPU_SHAPES))
def test_reference_engine_default_and_random_configs(engine, name):
    from benchmarks import get_task
    from compiler.triton.runner import GPO_AVAILABLE

    import gpu_optimizer_b200.runner as ours

    assert GPO_AVAILABLE and ours.GPO_AVAILABLE
    task = get_task(name)
    shape = GPU_SHAPES[name]
    res = engine.benchmark_candidate(task, task.make_candidate(shape,
                                                               task.default_config(shape)))
    assert res.status == "ok", f"{name}: {res.error}"
    assert res.correct and res.correctness_mode == "device" and res.engine == "cuda"
    assert res.latency.median_ms > 0
    space = task.param_space(shape)
    rng = random.Random(0)
    ok = 0
    for _ in range(6):
        cand = task.make_candidate(shape, space.sample(rng), provenance="random")
        r = engine.benchmark_candidate(task, cand)
        assert r.status in ("ok", "compile_error"), f"{name} {cand.config}: {r.error}"
        ok += r.status == "ok"
    assert ok >= 1


def _search(ctx_task, engine, db, n=16):
    from hardware.gpu_info import detect_hardware
    from optimizer.search.base import SearchContext
    from optimizer.search.loop import SearchLoop
    from optimizer.search.random_search import RandomSearcher

    ctx = SearchContext(task=ctx_task, shape=GPU_SHAPES["matmul"], hardware=detect_hardware(),
                        seed=5)
    loop = SearchLoop(ctx, RandomSearcher(ctx), engine, db=db, max_evaluations=n,
                      batch_size=8, run_id="b200-dropin")
    return loop.run()


def test_reference_search_loop_with_reference_engine(engine, tmp_path):
    from benchmarks import get_task
    from benchmarks.db import BenchmarkDB

    db = BenchmarkDB(tmp_path / "ref.sqlite")
    out = _search(get_task("matmul"), engine, db)
    assert out.candidates_evaluated == 16
    statuses = [h["status"] for h in out.history]
    assert set(statuses) <= {"ok", "compile_error"}, statuses
    assert out.best_result is not None and out.best_result.ok
    assert all(h["reward"] is not None for h in out.history)
    rows = db.fetch_results(task="matmul", limit=100)
    assert len(rows) >= 16 + 2  # candidates plus the torch and naive baselines


def test_reference_search_loop_with_b200_engine_and_fields(tmp_path):
    from benchmarks import get_task
    from benchmarks.db import BenchmarkDB

    from gpu_optimizer_b200.harness import BenchmarkSettings, CudaBenchmarkEngine
    from gpu_optimizer_b200.results_db import B200ResultsDB

    eng = CudaBenchmarkEngine(settings=BenchmarkSettings(warmup=3, iterations=10))
    db = B200ResultsDB(BenchmarkDB(tmp_path / "b200.sqlite"))
    out = _search(get_task("matmul"), eng, db)
    assert out.candidates_evaluated == 16
    assert {h["status"] for h in out.history} <= {"ok", "compile_error"}
    rows = db.fetch(run_id="b200-dropin")
    ok = [r for r in rows if r["status"] == "ok" and r["provenance"] == "random"]
    assert ok and all(r["achieved"] > 0 and r["achieved_unit"] in ("TFLOP/s", "GB/s")
                      and r["kernel"] for r in ok)
    src = db.candidate_source(ok[0]["candidate_id"])
    assert "__global__" in src["source"]
