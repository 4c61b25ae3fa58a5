"""The reference's real-hardware contract (tests/test_triton_gpu.py:32-70),
run against the B200 backend through the harness."""

import random

import pytest

from gpu_optimizer_b200.harness import BenchmarkSettings, CudaBenchmarkEngine
from gpu_optimizer_b200.tasks import REFERENCE_TASKS, get_task

pytestmark = pytest.mark.gpu

GPU_SHAPES = {  # tests/test_triton_gpu.py:21-29
    "matmul": (384, 320, 288), "vecadd": (1_000_003,), "reduction": (1_000_003,),
    "softmax": (256, 1000), "layernorm": (256, 1000), "fused_elementwise": (1_000_003,),
    "attention": (4, 512, 64), "attention_causal": (4, 512, 64), "fused_gelu": (1_000_003,),
}
ALL = sorted(GPU_SHAPES)


@pytest.fixture(scope="module")
def engine():
    return CudaBenchmarkEngine(settings=BenchmarkSettings(warmup=3, iterations=10))


@pytest.mark.parametrize("name", ALL)
def test_kernel_correct_on_gpu_default_config(engine, name):
    task = get_task(name)
    shape = GPU_SHAPES[name]
    res = engine.benchmark_candidate(task, task.make_candidate(shape, task.default_config(shape)))
    assert res.status == "ok", f"{name}: {res.error}"
    assert res.correct and res.correctness_mode == "device"
    assert res.latency.median_ms > 0 and res.engine == "cuda"


@pytest.mark.parametrize("name", ALL)
def test_kernel_correct_on_gpu_random_configs(engine, name):
    task = get_task(name)
    shape = GPU_SHAPES[name]
    space = task.param_space(shape)
    rng = random.Random(0)
    ok = 0
    for _ in range(6):
        cand = task.make_candidate(shape, space.sample(rng), provenance="random")
        res = engine.benchmark_candidate(task, cand)
        # compile errors are legitimate (resource limits); wrong answers are not
        assert res.status in ("ok", "compile_error"), f"{name} {cand.config}: {res.error}"
        ok += res.status == "ok"
    assert ok >= 1


B200_SMALL = {"matmul": (1024, 1024, 1024), "vecadd": (1 << 20,), "reduction": (1 << 20,),
              "softmax": (512, 8192), "layernorm": (512, 8192), "fused_elementwise": (1 << 20,),
              "fused_gelu": (1 << 20,), "attention": (8, 1024, 128),
              "attention_causal": (8, 1024, 128)}


@pytest.mark.parametrize("name", ALL)
def test_b200_space_random_configs(engine, name):
    task = get_task(name, "b200")
    shape = B200_SMALL[name]
    space = task.param_space(shape)
    rng = random.Random(1)
    statuses = []
    for _ in range(8):
        cand = task.make_candidate(shape, space.sample(rng), provenance="random")
        res = engine.benchmark_candidate(task, cand)
        assert res.status in ("ok", "compile_error"), f"{name} {cand.config}: {res.error}"
        statuses.append(res.status)
    assert "ok" in statuses


def test_baseline_and_roofline_fields(engine):
    task = get_task("vecadd", "b200")
    shape = (1 << 24,)
    base = engine.benchmark_baseline(task, shape, "float32")
    assert base.ok and base.achieved_unit == "GB/s" and base.achieved > 0
    res = engine.benchmark_candidate(task, task.make_candidate(
        shape, {"BLOCK_SIZE": 4096, "num_warps": 8, "dtype": "float32"}))
    assert res.ok and 0 < res.roofline_fraction < 1.5


# one config per family, including launches that zero an output (atomic
# reduction) and multi-launch strategies (unfused elementwise, two_pass)
GRAPH_CFGS = {
    "matmul": {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 64, "GROUP_M": 8, "num_warps": 4,
               "num_stages": 3, "dtype": "bfloat16"},
    "vecadd": {"BLOCK_SIZE": 1024, "num_warps": 4, "dtype": "float32"},
    "reduction": {"BLOCK_SIZE": 1024, "num_warps": 4, "strategy": "atomic", "dtype": "float32"},
    "softmax": {"BLOCK_N": 1024, "num_warps": 4, "num_stages": 2, "dtype": "bfloat16"},
    "layernorm": {"BLOCK_N": 1024, "num_warps": 4, "num_stages": 2, "dtype": "bfloat16"},
    "fused_elementwise": {"BLOCK_SIZE": 1024, "num_warps": 4, "strategy": "unfused",
                          "dtype": "bfloat16"},
    "attention_causal": {"BLOCK_M": 128, "BLOCK_N": 64, "num_warps": 4, "num_stages": 2,
                         "dtype": "bfloat16"},
}


@pytest.mark.parametrize("name", sorted(GRAPH_CFGS))
def test_launches_replay_from_cuda_graph(name):
    """Every family's launch sequence is capturable: a replayed graph gives
    the reference's answer, and the harness times it with cuda_graph=True."""
    import torch

    from gpu_optimizer_b200.correctness import check_correctness
    from gpu_optimizer_b200.runner import build_callable, check_device_status

    task = get_task(name, "b200")
    shape = GPU_SHAPES[name] if name != "matmul" else (512, 512, 256)
    cfg = GRAPH_CFGS[name]
    inputs = task.make_inputs(shape, cfg["dtype"], "cuda", 0)
    ref = task.reference(*inputs)
    kc = build_callable(name, shape, cfg, inputs)
    kc.fn()
    torch.cuda.synchronize()
    out = kc.fn()
    out.zero_()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            kc.fn()
    torch.cuda.current_stream().wait_stream(side)
    g.replay()
    torch.cuda.synchronize()
    check_device_status()
    rtol, atol = task.tolerance(cfg["dtype"])
    assert check_correctness(out, ref, rtol, atol).passed
    eng = CudaBenchmarkEngine(settings=BenchmarkSettings(warmup=3, iterations=10,
                                                         cuda_graph=True))
    res = eng.benchmark_candidate(task, task.make_candidate(shape, cfg))
    assert res.ok and res.latency.median_ms > 0, res.error


def test_multi_device_evaluator_on_gpu():
    """One spawned worker per visible GPU evaluates a small random batch and
    returns the results in proposal order."""
    import torch

    from gpu_optimizer_b200.dispatch import MultiDeviceEvaluator

    task = get_task("matmul", "b200")
    shape = (512, 512, 512)
    space = task.param_space(shape)
    rng = random.Random(3)
    cands = [task.make_candidate(shape, space.sample(rng), "random") for _ in range(6)]
    ev = MultiDeviceEvaluator(devices=list(range(torch.cuda.device_count())), profile="b200",
                              settings=BenchmarkSettings(warmup=2, iterations=5))
    try:
        assert ev.wait_ready(timeout_s=300)
        res = ev.evaluate(cands)
    finally:
        ev.close()
    assert [r.candidate_id for r in res] == [c.candidate_id for c in cands]
    assert all(r.status in ("ok", "compile_error") for r in res), [r.error for r in res]
    assert any(r.status == "ok" for r in res)


def test_device_timeout_on_first_launch_is_a_runtime_error(monkeypatch):
    """GPO_TIMEOUT maps to runtime_error end to end: a first launch whose
    bounded device wait gave up is not a compile failure (the surrogate's
    P(compile) label stays clean), and the candidate's later calls raise."""
    from gpu_optimizer_b200 import _lib

    real = _lib.device_status
    calls = {"n": 0}

    def timed_out_once(stream):
        calls["n"] += 1
        if calls["n"] == 1:
            real(stream)  # synchronise as the real call does
            return _lib.TIMEOUT, 1 << 6
        return real(stream)

    monkeypatch.setattr(_lib, "device_status", timed_out_once)
    eng = CudaBenchmarkEngine(settings=BenchmarkSettings(warmup=1, iterations=2))
    task = get_task("vecadd", "b200")
    cand = task.make_candidate((1 << 16,), {"BLOCK_SIZE": 1024, "num_warps": 4,
                                            "dtype": "float32"})
    res = eng.benchmark_candidate(task, cand)
    assert res.status == "runtime_error", (res.status, res.error)
    assert "timed out" in res.error
    # the next candidate on the same engine is unaffected
    assert eng.benchmark_candidate(task, cand).status == "ok"
