"""The persistent two-tile attention kernel (BLOCK_M 256, num_warps 8).

Its CTAs, one per SM, take (256-row span, head) work items from a counter
that each launch borrows from a small pool and the last CTA clears, and
they carry their K/V rings, barrier phases and Q reloads from one item to
the next.  These cases cover what the benchmark shape does not:

* ragged sequence lengths (a partial last span, a partial last K/V block)
  and head counts that leave fewer work items than SMs, full and causal,
  fp16 and bf16, D = 64 and 128, against the CPU reference with the
  reference's own verdict (``check_correctness``) and the normwise bound;
* many launches in a row: more than twice the pool of work counters, so
  every counter is borrowed, cleared and borrowed again; every launch must
  give bit-identical output (an item's result does not depend on which CTA
  takes it), which a counter left non-zero would break by skipping items.
"""

import pytest
import torch

from gpu_optimizer_b200.correctness import NORMWISE_BOUND, rowwise_relative_error
from gpu_optimizer_b200.runner import build_callable, check_device_status
from gpu_optimizer_b200.tasks import get_task
from oracle import reference as O

pytestmark = pytest.mark.gpu

DUAL = {"BLOCK_M": 256, "num_warps": 8}

RAGGED = [
    # (B*H, S, D), BLOCK_N, stages, dtype
    ((3, 1000, 128), 128, 2, "bfloat16"),   # 4 spans, last one 232 rows
    ((5, 130, 64), 64, 3, "float16"),       # one span, 130 rows, 3 K/V blocks
    ((1, 257, 128), 128, 2, "bfloat16"),    # a one-row second span
    ((200, 384, 64), 128, 4, "bfloat16"),   # 400 items, more than the SMs
    ((2, 4096, 128), 32, 2, "float16"),     # BLOCK_N 32
]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("shape,bn,stages,dtype", RAGGED,
                         ids=lambda x: "x".join(map(str, x)) if isinstance(x, tuple) else str(x))
def test_ragged_shapes_match_reference(causal, shape, bn, stages, dtype):
    name = "attention_causal" if causal else "attention"
    task = get_task(name, "b200")
    cfg = {**DUAL, "BLOCK_N": bn, "num_stages": stages, "dtype": dtype}
    q, k, v = task.make_inputs(shape, dtype, "cuda", 3)
    kc = build_callable(name, shape, cfg, (q, k, v))
    assert kc.launch["kernel"].startswith("attn_tc_dual_kernel")
    out = kc.fn()
    check_device_status()
    ref = O.reference(name, (q.cpu(), k.cpu(), v.cpu()))
    rtol, atol = O.tolerance(name, dtype)
    verdict = O.check(out.cpu(), ref, rtol, atol)
    assert verdict["passed"], verdict
    assert rowwise_relative_error(out.cpu(), ref) <= NORMWISE_BOUND[dtype]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_repeated_launches_are_identical(causal):
    name = "attention_causal" if causal else "attention"
    task = get_task(name, "b200")
    shape = (16, 2048, 128)  # 128 items on 148 SMs: every CTA takes at most one
    cfg = {**DUAL, "BLOCK_N": 128, "num_stages": 2, "dtype": "bfloat16"}
    q, k, v = task.make_inputs(shape, "bfloat16", "cuda", 5)
    kc = build_callable(name, shape, cfg, (q, k, v))
    first = kc.fn().clone()
    torch.cuda.synchronize()
    check_device_status()
    big = (64, 2048, 128)  # 512 items: CTAs take several each
    qb, kb, vb = task.make_inputs(big, "bfloat16", "cuda", 6)
    kb_call = build_callable(name, big, cfg, (qb, kb, vb))
    big_first = kb_call.fn().clone()
    for i in range(14):  # 140 launches: more than twice the 64 work counters
        for _ in range(5):
            kc.fn()
            kb_call.fn()
        torch.cuda.synchronize()
        check_device_status()
        assert torch.equal(kc.fn(), first), i
        assert torch.equal(kb_call.fn(), big_first), i
    ref = O.reference(name, (q.cpu()[:2], k.cpu()[:2], v.cpu()[:2]))
    assert rowwise_relative_error(first[:2].cpu(), ref) <= NORMWISE_BOUND["bfloat16"]
