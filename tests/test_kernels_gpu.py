"""GPU parity: every kernel family, through the C-ABI runner, against the
reference's golden outputs and the CPU oracle on identical seeded inputs.

Bars: bit-exact where the computation is exactly rounded elementwise
(vecadd, fused relu); the reference's per-task (rtol, atol) elsewhere
(benchmarks/*/task.py ``tolerance``), as the reference's own GPU tests
apply (tests/test_triton_gpu.py:32-70 via benchmarks/harness.py:176-189).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_optimizer_b200 import _lib
from gpu_optimizer_b200.runner import KernelBuildError, build_callable, check_device_status
from oracle import reference as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
INDEX = json.loads((GOLDEN / "golden_index.json").read_text())


def golden_ref(name, key, dtype):
    arr = np.load(GOLDEN / f"golden_{name}.npz")[key]
    if dtype == "bfloat16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(arr.copy())


def run(task, shape, cfg, inputs):
    dev = [t.cuda() for t in inputs]
    kc = build_callable(task, shape, cfg, tuple(dev))
    out = kc.fn()
    check_device_status()
    return out.cpu(), kc


def assert_close(task, dtype, out, ref, what=""):
    rtol, atol = O.tolerance(task, dtype)
    v = O.check(out, ref, rtol, atol)
    assert v["passed"], f"{task} {dtype} {what}: {v}"


# --------------------------------------------------------- configurations
MM_TC = [  # tcgen05 family: (BM, BN, BK, GROUP_M, warps, stages)
    (128, 32, 32, 1, 4, 2), (128, 64, 64, 4, 8, 3), (128, 128, 64, 8, 8, 4),
    (128, 256, 64, 8, 8, 4), (128, 256, 128, 1, 4, 2), (256, 128, 64, 4, 8, 3),
    (256, 256, 64, 16, 8, 2), (256, 64, 32, 1, 4, 5), (128, 128, 256, 4, 8, 2),
    # CTA pairs (cta_group::2); 8 warps -> persistent pairs
    (256, 256, 64, 8, 4, 3), (256, 128, 64, 4, 4, 3), (256, 32, 32, 1, 4, 2),
    (256, 256, 128, 8, 4, 2), (256, 256, 64, 8, 8, 6), (256, 128, 64, 16, 8, 8),
    (256, 64, 64, 1, 8, 4),
    # BLOCK_M 64: M=64 MMAs
    (64, 128, 64, 8, 4, 4), (64, 256, 64, 8, 8, 4), (64, 64, 32, 1, 4, 3),
    (64, 32, 128, 4, 8, 2),
    # BLOCK_M 32: M=64 MMAs over 64-row A atoms holding the tile's 32 rows
    (32, 128, 64, 8, 4, 3), (32, 64, 64, 1, 8, 4), (32, 256, 32, 4, 4, 2),
    (32, 32, 128, 1, 8, 2),
]
MM_SIMT = [(16, 16, 16, 1, 2, 2), (32, 32, 16, 1, 4, 2), (64, 128, 32, 4, 8, 3),
           (128, 128, 64, 8, 8, 4)]


def mm_cfg(t, dtype):
    bm, bn, bk, g, w, s = t
    return {"BLOCK_M": bm, "BLOCK_N": bn, "BLOCK_K": bk, "GROUP_M": g, "num_warps": w,
            "num_stages": s, "dtype": dtype}


def task_configs(name, dtype):
    if name == "matmul":
        cfgs = [mm_cfg(t, dtype) for t in MM_SIMT]
        if dtype != "float32":
            cfgs += [mm_cfg(t, dtype) for t in MM_TC]
        return cfgs
    if name == "vecadd":
        return [{"BLOCK_SIZE": b, "num_warps": w, "dtype": dtype}
                for b, w in ((128, 1), (1024, 4), (4096, 8), (256, 8))]
    if name == "reduction":
        return [{"BLOCK_SIZE": b, "num_warps": w, "strategy": s, "dtype": dtype}
                for s in ("loop", "atomic", "two_pass") for b, w in ((256, 1), (8192, 16),
                                                                    (1024, 4))]
    if name in ("softmax", "layernorm"):
        # num_stages >= 2 on single tiles: persistent row ring (shared-memory
        # ring of num_stages rows) or, when the ring does not fit, the
        # register prefetch pipeline
        return [{"BLOCK_N": b, "num_warps": w, "num_stages": s, "dtype": dtype}
                for b, w, s in ((128, 4, 2), (512, 1, 2), (1024, 4, 3), (4096, 16, 4),
                                (16384, 1, 2), (256, 16, 2), (1024, 8, 1), (4096, 8, 4))]
    if name in ("fused_elementwise", "fused_gelu"):
        return [{"BLOCK_SIZE": b, "num_warps": w, "strategy": s, "dtype": dtype}
                for s in ("fused", "unfused") for b, w in ((128, 1), (1024, 4), (4096, 8))]
    if name in ("attention", "attention_causal"):
        cfgs = [{"BLOCK_M": bm, "BLOCK_N": bn, "num_warps": w, "num_stages": s,
                 "dtype": dtype} for bm, bn, w, s in ((32, 32, 4, 1), (16, 64, 2, 2),
                                                      (64, 32, 8, 2))]
        if dtype != "float32":
            cfgs += [{"BLOCK_M": 128, "BLOCK_N": bn, "num_warps": w, "num_stages": s,
                      "dtype": dtype} for bn, s, w in ((32, 1, 4), (64, 2, 4), (128, 2, 4),
                                                       (32, 4, 4), (64, 2, 8), (32, 3, 8),
                                                       (128, 2, 8))]
        return cfgs
    raise KeyError(name)


EXACT = {"vecadd", "fused_elementwise"}


def golden_cases():
    for name in sorted(INDEX["tasks"]):
        for case in INDEX["tasks"][name]["cases"]:
            if case["seed"] == 0:
                yield name, case


@pytest.mark.parametrize("name,case", list(golden_cases()),
                         ids=lambda x: x if isinstance(x, str) else x["dtype"])
def test_parity_with_reference_golden_outputs(name, case):
    """Every family at the reference's odd small shapes vs its own outputs."""
    shape = tuple(INDEX["tasks"][name]["shape"])
    dtype = case["dtype"]
    inputs = O.make_inputs(name, shape, dtype, case["seed"])
    ref = golden_ref(name, case["ref"], dtype)
    for cfg in task_configs(name, dtype):
        try:
            out, kc = run(name, shape, cfg, inputs)
        except KernelBuildError as e:
            # only genuine resource overflow may refuse a config
            assert "GPO_COMPILE_ERROR" in str(e), f"{cfg}: {e}"
            continue
        assert_close(name, dtype, out, ref, f"{cfg} [{kc.launch['kernel']}]")
        emu = O.emulate(name, shape, cfg, inputs)
        if name in EXACT:
            # exactly rounded elementwise work: bit-identical to the
            # reference's algorithm, including the unfused storage roundings
            assert torch.equal(out, emu), f"{name} {cfg} not bit-exact"
        else:
            assert_close(name, dtype, out, emu, f"vs emulate {cfg}")


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("name", ["fused_gelu", "attention_causal"])
def test_parity_new_variants_with_oracle(name, dtype):
    shape = (10_007,) if name == "fused_gelu" else (3, 130, 32)
    inputs = O.make_inputs(name, shape, dtype, 1)
    ref = O.reference(name, inputs)
    for cfg in task_configs(name, dtype):
        try:
            out, kc = run(name, shape, cfg, inputs)
        except KernelBuildError as e:
            assert "GPO_COMPILE_ERROR" in str(e), f"{cfg}: {e}"
            continue
        assert_close(name, dtype, out, ref, f"{cfg} [{kc.launch['kernel']}]")


# (2048, 2560, 256) gives persistent clusters several tiles each
MM_SHAPES = [(384, 320, 288), (1000, 1000, 1000), (257, 512, 136), (128, 256, 64),
             (1024, 2048, 512), (2048, 2560, 256)]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "tf32"])
@pytest.mark.parametrize("shape", MM_SHAPES, ids=str)
def test_tcgen05_matmul_ragged_shapes(shape, dtype):
    inputs = O.make_inputs("matmul", shape, "float32" if dtype == "tf32" else dtype, 0)
    for t in MM_TC:
        cfg = mm_cfg(t, dtype)
        try:
            out, kc = run("matmul", shape, cfg, inputs)
        except KernelBuildError as e:
            assert "GPO_COMPILE_ERROR" in str(e), f"{cfg}: {e}"
            continue
        assert kc.launch["kernel"].startswith("matmul_tc"), kc.launch["kernel"]
        emu = O.emulate("matmul", shape, cfg, inputs)
        assert_close("matmul", dtype, out, emu, f"{shape} {cfg}")


ATT_SHAPES = [(4, 512, 64), (2, 300, 128), (1, 1000, 32), (3, 130, 128), (2, 256, 256)]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("shape", ATT_SHAPES, ids=str)
def test_tcgen05_attention_shapes(shape, dtype, causal):
    name = "attention_causal" if causal else "attention"
    inputs = O.make_inputs(name, shape, dtype, 2)
    ref = O.reference(name, inputs)
    ran = 0
    # BLOCK_M 256: CTA pairs on two query tiles (odd tile counts leave the
    # last pair's second tile partly or wholly past S); BLOCK_M 64: 64-row
    # tiles on M=64 MMAs
    for bm, bn, stages, warps in [(bm, bn, st, w) for bm in (64, 128, 256) for bn in (32, 64, 128)
                                  for st in (1, 2, 3) for w in (4, 8)]:
        cfg = {"BLOCK_M": bm, "BLOCK_N": bn, "num_warps": warps, "num_stages": stages,
               "dtype": dtype}
        try:
            out, kc = run(name, shape, cfg, inputs)
        except KernelBuildError as e:
            assert "GPO_COMPILE_ERROR" in str(e), f"{cfg}: {e}"
            continue
        assert kc.launch["kernel"].startswith(("attn_tc_kernel", "attn_tc_dual_kernel"))
        assert_close(name, dtype, out, ref, f"{shape} {cfg}")
        ran += 1
    assert ran >= 9


def test_edge_cases():
    # n = 0 and n = 1 vectors, single-row softmax, 1x1x1 matmul
    for n in (1, 3, 17):
        ins = O.make_inputs("vecadd", (n,), "float32", 0)
        out, _ = run("vecadd", (n,), {"BLOCK_SIZE": 128, "num_warps": 1, "dtype": "float32"},
                     ins)
        assert torch.equal(out, O.reference("vecadd", ins))
        ins = O.make_inputs("reduction", (n,), "float32", 0)
        for s in ("loop", "atomic", "two_pass"):
            out, _ = run("reduction", (n,), {"BLOCK_SIZE": 256, "num_warps": 2, "strategy": s,
                                            "dtype": "float32"}, ins)
            assert_close("reduction", "float32", out, O.reference("reduction", ins), s)
    ins = O.make_inputs("softmax", (1, 3), "bfloat16", 0)
    out, _ = run("softmax", (1, 3), {"BLOCK_N": 128, "num_warps": 1, "num_stages": 1,
                                     "dtype": "bfloat16"}, ins)
    assert_close("softmax", "bfloat16", out, O.reference("softmax", ins))
    ins = O.make_inputs("matmul", (1, 1, 1), "float32", 0)
    out, _ = run("matmul", (1, 1, 1), mm_cfg((16, 16, 16, 1, 2, 2), "float32"), ins)
    assert_close("matmul", "float32", out, O.reference("matmul", ins))


def test_misaligned_operands_are_rejected_not_launched():
    """A TMA operand that is not 16-byte aligned is refused on the host."""
    a = torch.randn(129 * 64 + 1, device="cuda", dtype=torch.bfloat16)[1:].view(129, 64)
    b = torch.randn(64, 128, device="cuda", dtype=torch.bfloat16)
    kc = build_callable("matmul", (129, 128, 64), mm_cfg((128, 128, 64, 1, 4, 2), "bfloat16"),
                        (a, b))
    with pytest.raises(RuntimeError, match="GPO_BAD_ARGS"):
        kc.fn()


def test_device_timeout_is_reported_not_hung():
    """A bounded device wait on a barrier nobody arrives at reports GPO_TIMEOUT."""
    stream = torch.cuda.current_stream().cuda_stream
    rc, flags = _lib.selftest_timeout(stream, 50)
    assert rc == _lib.TIMEOUT and flags & (1 << 6)
    # the context stays usable and the error word was cleared
    check_device_status()
    ins = O.make_inputs("vecadd", (1000,), "float32", 0)
    out, _ = run("vecadd", (1000,), {"BLOCK_SIZE": 256, "num_warps": 2, "dtype": "float32"},
                 ins)
    assert torch.equal(out, O.reference("vecadd", ins))
