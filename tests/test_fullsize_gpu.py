"""Full-size workloads of the B200 benchmark configurations, checked through
size-independent properties and sampled oracle slices."""

import pytest
import torch

from gpu_optimizer_b200.runner import build_callable, check_device_status
from gpu_optimizer_b200.tasks import get_task
from oracle import reference as O

pytestmark = pytest.mark.gpu

# the headline CTA-pair tile, the persistent CTA pair and the persistent 1-CTA tile
MM_FULL = [
    {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 64, "GROUP_M": 16, "num_warps": 4,
     "num_stages": 3, "dtype": "bfloat16"},
    # the bench headline: persistent pair, 128-deep K stages
    {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 128, "GROUP_M": 16, "num_warps": 8,
     "num_stages": 3, "dtype": "bfloat16"},
    {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K": 64, "GROUP_M": 16, "num_warps": 8,
     "num_stages": 6, "dtype": "bfloat16"},
    {"BLOCK_M": 128, "BLOCK_N": 256, "BLOCK_K": 64, "GROUP_M": 8, "num_warps": 8,
     "num_stages": 4, "dtype": "bfloat16"},
]


@pytest.mark.parametrize("MM_BEST", MM_FULL, ids=lambda c: f"{c['BLOCK_M']}x{c['BLOCK_N']}x{c['BLOCK_K']}w{c['num_warps']}s{c['num_stages']}")
def test_matmul_4096_linearity_and_reference(MM_BEST):
    task = get_task("matmul", "b200")
    shape = (4096, 4096, 4096)
    a, b = task.make_inputs(shape, "bfloat16", "cuda", 0)
    c = build_callable("matmul", shape, MM_BEST, (a, b)).fn().clone()
    c2 = build_callable("matmul", shape, MM_BEST, (a * 2, b)).fn()
    check_device_status()
    # scaling an operand by 2 is exact in bf16, fp32 accumulation and rounding
    assert torch.equal(c2, c * 2)
    ref = task.reference(a, b)
    rtol, atol = O.tolerance("matmul", "bfloat16")
    assert O.check(c, ref, rtol, atol)["passed"]
    # sampled rows against the CPU oracle
    rows = torch.tensor([0, 1, 2047, 4095])
    cpu = O.reference("matmul", (a[rows].cpu(), b.cpu()))
    assert O.check(c[rows].cpu(), cpu, rtol, atol)["passed"]


def test_softmax_layernorm_full_rows():
    for name in ("softmax", "layernorm"):
        task = get_task(name, "b200")
        shape = (16384, 8192)
        ins = task.make_inputs(shape, "bfloat16", "cuda", 0)
        for bn, w in ((8192, 8), (2048, 8), (16384, 4)):
            cfg = {"BLOCK_N": bn, "num_warps": w, "num_stages": 2, "dtype": "bfloat16"}
            out = build_callable(name, shape, cfg, ins).fn()
            check_device_status()
            rtol, atol = O.tolerance(name, "bfloat16")
            assert O.check(out, task.reference(*ins), rtol, atol)["passed"], cfg
            if name == "softmax":
                s = out.float().sum(dim=1)
                assert torch.allclose(s, torch.ones_like(s), atol=2e-2)


def test_reduction_2p28_strategies_agree():
    task = get_task("reduction", "b200")
    shape = (1 << 28,)
    (x,) = task.make_inputs(shape, "float32", "cuda", 0)
    ref = x.double().sum()
    outs = []
    for s in ("loop", "atomic", "two_pass"):
        cfg = {"BLOCK_SIZE": 4096, "num_warps": 8, "strategy": s, "dtype": "float32"}
        outs.append(build_callable("reduction", shape, cfg, (x,)).fn().double().item())
        check_device_status()
    for o in outs:
        assert abs(o - ref.item()) <= 1e-2 + 1e-3 * abs(ref.item())


def test_causal_attention_full_size():
    task = get_task("attention_causal", "b200")
    shape = (128, 4096, 128)
    q, k, v = task.make_inputs(shape, "bfloat16", "cuda", 0)
    cfg = {"BLOCK_M": 128, "BLOCK_N": 128, "num_warps": 4, "num_stages": 2,
           "dtype": "bfloat16"}
    out = build_callable("attention_causal", shape, cfg, (q, k, v)).fn()
    check_device_status()
    # query 0 sees only key 0: its output row is V's row 0, exactly
    assert torch.equal(out[:, 0], v[:, 0])
    rtol, atol = O.tolerance("attention_causal", "bfloat16")
    for h in (0, 77, 127):
        ref = O.reference("attention_causal", (q[h:h + 1].cpu(), k[h:h + 1].cpu(),
                                               v[h:h + 1].cpu()))
        assert O.check(out[h:h + 1].cpu(), ref, rtol, atol)["passed"], h
