"""This backend against the reference's own Python modules (no GPU).

The reference is installed under ``baseline/_ref`` and imported as it
ships.  Checked here:

* the contracts this package restates so that it also runs without the
  reference -- parameter spaces and ``candidate_id``, the reward, the
  correctness verdict, ``LatencyStats`` / ``BenchmarkResult`` fields, the
  hardware feature vector -- give the reference's answers;
* the reference's simulated engine with ``B200CompileModel`` labels exactly
  the candidates the B200 backend refuses as ``compile_error``, over every
  point of the B200 matmul and attention spaces;
* a B200 result round-trips through the reference's results database with
  the added ``b200_results`` table, and the reference's dashboard route
  serves this backend's CUDA source through the swapped runner import.
"""

import math
import random

import numpy as np
import pytest
import torch

import reference_stack

pytestmark = pytest.mark.skipif(not reference_stack.available(),
                                reason="reference not installed under baseline/_ref")


@pytest.fixture(scope="module", autouse=True)
def ref():
    reference_stack.activate()


REF_SHAPES = {"matmul": (384, 320, 288), "vecadd": (1_000_003,), "reduction": (1_000_003,),
              "softmax": (256, 1000), "layernorm": (256, 1000),
              "fused_elementwise": (1_000_003,), "attention": (4, 512, 64)}


@pytest.mark.parametrize("name", sorted(REF_SHAPES))
def test_spaces_and_candidate_ids_match_reference(name):
    from benchmarks import get_task as ref_task
    from compiler.transformations.space import Candidate as RefCandidate

    from gpu_optimizer_b200.space import Candidate
    from gpu_optimizer_b200.tasks import get_task

    shape = REF_SHAPES[name]
    theirs, ours = ref_task(name), get_task(name)
    ts, os_ = theirs.param_space(shape), ours.param_space(shape)
    assert [(s.name, s.choices) for s in ts] == [(s.name, s.choices) for s in os_]
    assert ts.size() == os_.size()
    assert theirs.default_config(shape) == ours.default_config(shape)
    r1, r2 = random.Random(7), random.Random(7)
    for _ in range(50):
        c1, c2 = ts.sample(r1), os_.sample(r2)
        assert c1 == c2
        assert RefCandidate(name, shape, c1).candidate_id == Candidate(name, shape, c2).candidate_id
        assert ts.neighbors(c1) == os_.neighbors(c2)
    for dtype in [s for s in ts["dtype"].choices]:
        assert tuple(theirs.tolerance(dtype)) == tuple(ours.tolerance(dtype))
    assert theirs.flops(shape) == pytest.approx(ours.flops(shape))


def test_continuous_param_specs_match_reference():
    from compiler.transformations.space import ParamSpace as RP
    from compiler.transformations.space import ParamSpec as RS

    from gpu_optimizer_b200.space import ParamSpace, ParamSpec

    def specs(S):
        return [S("BLOCK_N", choices=(32, 64, 128)), S("scale", low=0.5, high=2.0),
                S("dtype", choices=("float16", "bfloat16"))]

    a, b = RP(specs(RS)), ParamSpace(specs(ParamSpec))
    ra, rb = random.Random(3), random.Random(3)
    for _ in range(20):
        ca, cb = a.sample(ra), b.sample(rb)
        assert ca == cb
        a.validate(ca)
        b.validate(cb)
        assert a.neighbors(ca) == b.neighbors(cb)
    assert a.grid() == b.grid() and a.size() == b.size()
    with pytest.raises(ValueError):
        ParamSpec("x", choices=(1,), low=0.0, high=1.0)
    with pytest.raises(TypeError):
        ParamSpec("x", low=0.0, high=1.0).index_of(0.5)


def _results(make_result, make_stats):
    base = dict(candidate_id="c", task="matmul", shape=(8, 8, 8), config={}, engine="cuda",
                gpu_name="g")
    out = []
    for status in ("ok", "compile_error", "runtime_error", "incorrect"):
        for ms, mem in ((0.5, 0), (2.0, 1 << 30), (1e-4, 0), (1e4, 0)):
            lat = make_stats([ms, ms * 1.1, ms * 0.9]) if status == "ok" else None
            out.append(make_result(**base, status=status, latency=lat, memory_bytes=mem))
    return out


def test_reward_matches_reference():
    from benchmarks.harness import BenchmarkResult as RR
    from benchmarks.harness import LatencyStats as RL
    from optimizer.rewards.reward import RewardConfig as RC
    from optimizer.rewards.reward import compute_reward as ref_reward

    from gpu_optimizer_b200.harness import BenchmarkResult, LatencyStats
    from gpu_optimizer_b200.search import RewardConfig, compute_reward

    cfgs = [{}, {"mode": "speedup"}, {"memory_limit_bytes": 1 << 20}, {"clip": None},
            {"compile_penalty": 0.25, "runtime_penalty": 2.0}]
    for kw in cfgs:
        for theirs, ours in zip(_results(RR, RL.from_samples),
                                _results(BenchmarkResult, LatencyStats.from_samples)):
            for base in (1.0, 0.01):
                assert compute_reward(ours, base, RewardConfig(**kw)) == \
                    ref_reward(theirs, base, RC(**kw))
    with pytest.raises(ValueError):
        RewardConfig(mode="nope")


def test_correctness_verdict_matches_reference():
    from compiler.validation.correctness import check_correctness as ref_check

    from gpu_optimizer_b200.correctness import check_correctness

    g = torch.Generator().manual_seed(0)
    cases = []
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        r = torch.randn(64, 33, generator=g).to(dtype)
        cases += [(r.clone(), r), ((r.float() * 1.01).to(dtype), r),
                  ((r.float() + 0.5).to(dtype), r)]
    bad = torch.randn(5, 5, generator=g)
    bad[2, 2] = math.nan
    cases += [(bad, torch.zeros(5, 5)), (torch.zeros(3), torch.zeros(4)),
              (torch.zeros(0), torch.zeros(0))]
    for c, r in cases:
        for tol in ((1e-4, 1e-5), (2e-2, 1e-2)):
            a, b = check_correctness(c, r, *tol), ref_check(c, r, *tol)
            assert (a.passed, a.max_abs_err, a.max_rel_err, a.rtol, a.atol, a.detail) == \
                (b.passed, b.max_abs_err, b.max_rel_err, b.rtol, b.atol, b.detail)


def test_result_records_and_hardware_vector_match_reference():
    from benchmarks.harness import BenchmarkResult as RR
    from benchmarks.harness import BenchmarkSettings as RSet
    from benchmarks.harness import LatencyStats as RL
    from hardware.gpu_info import HardwareSpec as RH

    from gpu_optimizer_b200.harness import BenchmarkResult, BenchmarkSettings, LatencyStats
    from gpu_optimizer_b200.hardware import B200

    samples = [0.31, 0.29, 0.5, 0.3, 0.33]
    assert vars(LatencyStats.from_samples(samples)) == vars(RL.from_samples(samples))
    base = dict(candidate_id="c", task="t", shape=(1,), config={}, engine="cuda",
                gpu_name="g", status="ok", timestamp=1.0)
    theirs, ours = RR(**base).to_dict(), BenchmarkResult(**base).to_dict()
    assert set(theirs) <= set(ours)
    assert {k: ours[k] for k in theirs} == theirs
    s, t = BenchmarkSettings(), RSet()
    assert (s.warmup, s.iterations, s.seed) == (t.warmup, t.iterations, t.seed)
    fields = {k: v for k, v in B200.to_dict().items() if k in RH.__dataclass_fields__}
    fields["compute_capability"] = tuple(fields["compute_capability"])
    np.testing.assert_array_equal(RH(**fields).feature_vector(), B200.feature_vector())


@pytest.mark.parametrize("name,shape", [("matmul", (4096, 4096, 4096)),
                                        ("attention", (128, 4096, 128)),
                                        ("attention_causal", (128, 4096, 128))])
def test_simulated_engine_compile_labels_agree_with_backend(name, shape):
    from benchmarks.harness import BenchmarkSettings as RSet
    from benchmarks.harness import SimulatedBenchmarkEngine
    from hardware.gpu_info import HardwareSpec as RH

    from gpu_optimizer_b200.compile_model import b200_compiles, use_b200_compile_model
    from gpu_optimizer_b200.hardware import B200
    from gpu_optimizer_b200.tasks import get_task

    fields = {k: v for k, v in B200.to_dict().items() if k in RH.__dataclass_fields__}
    fields["compute_capability"] = tuple(fields["compute_capability"])
    hw = RH(**fields)
    eng = SimulatedBenchmarkEngine(hw, RSet(warmup=1, iterations=2),
                                   check_correctness_emulated=False)
    a100_style = eng.model
    use_b200_compile_model(eng)
    task = get_task(name, "b200")
    grid = task.param_space(shape).grid()
    disagree_before = 0
    refused = 0
    for cfg in grid:
        ok, _ = b200_compiles(name, shape, cfg)
        res = eng.benchmark_candidate(task, task.make_candidate(shape, cfg))
        assert (res.status == "compile_error") == (not ok), (cfg, res.status)
        refused += not ok
        disagree_before += a100_style.compiles(task, shape, cfg)[0] != ok
    # the space has real refusals, and the A100-era estimate mislabels part of it
    assert 0 < refused < len(grid)
    print(f"\n{name}: {len(grid)} configs, {refused} refused by the B200 planner, "
          f"{disagree_before} mislabelled by the reference's A100-era estimate")


def test_results_db_round_trip_and_dashboard_source(tmp_path, monkeypatch):
    from benchmarks.db import BenchmarkDB

    from gpu_optimizer_b200.correctness import CorrectnessReport
    from gpu_optimizer_b200.harness import BenchmarkResult, LatencyStats
    from gpu_optimizer_b200.results_db import B200ResultsDB
    from gpu_optimizer_b200.space import Candidate

    cfg = {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 128, "GROUP_M": 16, "num_warps": 8,
           "num_stages": 3, "dtype": "bfloat16"}
    cand = Candidate("matmul", (4096, 4096, 4096), cfg)
    rep = CorrectnessReport(True, 1e-3, 2e-2, 5e-2, 1e-2, "", 2e-2, 3e-3)
    res = BenchmarkResult(candidate_id=cand.candidate_id, task="matmul",
                          shape=cand.shape, config=cfg, engine="cuda", status="ok",
                          gpu_name="NVIDIA B200", correct=True, correctness_mode="device",
                          correctness=rep, latency=LatencyStats.from_samples([0.1, 0.11]),
                          throughput_gflops=1.3e6, achieved=1300.0, achieved_unit="TFLOP/s",
                          roofline_fraction=0.77,
                          kernel="matmul_tc2_kernel<bf16,256,256,cta_pair_persistent>",
                          device_index=3, worker_id=2)
    base = BenchmarkDB(tmp_path / "results.sqlite")
    db = B200ResultsDB(base)
    db.create_run("run1", "matmul", cand.shape, "random", "cuda", "NVIDIA B200")
    rid = db.insert_result(res, run_id="run1")
    # the reference's own reader sees an unchanged results row
    row = base.fetch_results(task="matmul")[0]
    assert row["candidate_id"] == cand.candidate_id and row["status"] == "ok"
    assert row["latency_median_ms"] == pytest.approx(res.latency.median_ms)
    got = db.fetch(candidate_id=cand.candidate_id)[0]
    assert got["id"] == rid
    assert (got["achieved"], got["achieved_unit"], got["roofline_fraction"], got["kernel"],
            got["device_index"], got["worker_id"]) == (1300.0, "TFLOP/s", 0.77, res.kernel, 3, 2)
    assert got["rel_err_normwise"] == pytest.approx(3e-3)
    src = db.candidate_source(cand.candidate_id)
    assert "__global__" in src["source"] and "BLOCK_M = 256" in src["source"]
    assert src["roofline_fraction"] == 0.77
    # only the coordinator writes
    db._owner = -1
    with pytest.raises(RuntimeError, match="coordinator"):
        db.insert_result(res, run_id="run1")
    # the reference's dashboard route, unchanged, through the swapped import
    import server.api.main as dash

    monkeypatch.setattr(dash, "_db", base)
    out = dash.candidate_source(cand.candidate_id)
    assert "__global__" in out["source"] and "Candidate configuration" in out["source"]
