"""The oracle is pinned to the reference's own outputs (tests/golden/).

tests/golden/ was produced by running the reference's ``make_inputs``,
``task.reference`` and ``emulate`` (tests/golden/make_golden.py).  Here the
CPU oracle must reproduce every stored input hash and output bit-for-bit,
and the product's input generators must produce the same inputs.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_optimizer_b200.tasks import get_task
from oracle import reference as O

GOLDEN = Path(__file__).resolve().parent / "golden"
INDEX = json.loads((GOLDEN / "golden_index.json").read_text())
TASKS = sorted(INDEX["tasks"])


def to_np(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def sha(t):
    return hashlib.sha256(to_np(t).tobytes()).hexdigest()


def cases():
    for name in TASKS:
        for c in INDEX["tasks"][name]["cases"]:
            yield name, c


@pytest.mark.parametrize("name,case", list(cases()),
                         ids=lambda x: x if isinstance(x, str) else f"{x['dtype']}-s{x['seed']}")
def test_oracle_matches_reference_bits(name, case):
    shape = tuple(INDEX["tasks"][name]["shape"])
    data = np.load(GOLDEN / f"golden_{name}.npz")
    inputs = O.make_inputs(name, shape, case["dtype"], case["seed"])
    assert [sha(t) for t in inputs] == case["input_sha"]
    np.testing.assert_array_equal(to_np(O.reference(name, inputs)), data[case["ref"]])
    for e in case["emulate"]:
        out = O.emulate(name, shape, e["config"], inputs)
        np.testing.assert_array_equal(to_np(out), data[e["key"]], err_msg=str(e["config"]))


@pytest.mark.parametrize("name", TASKS)
def test_product_inputs_match_reference(name):
    """The harness's seeded inputs equal the reference's (small and GPU shapes)."""
    entry = INDEX["tasks"][name]
    task = get_task(name)
    for case in entry["cases"]:
        ins = task.make_inputs(tuple(entry["shape"]), case["dtype"], "cpu", case["seed"])
        assert [sha(t) for t in ins] == case["input_sha"]
    for dtype, hashes in entry["gpu_input_sha"].items():
        ins = task.make_inputs(tuple(entry["gpu_shape"]), dtype, "cpu", 0)
        assert [sha(t) for t in ins] == hashes


def test_oracle_checker_flags_bad_output():
    """tests/test_tasks_and_emulation.py:94-104 against the oracle's verdict."""
    inputs = O.make_inputs("vecadd", (1024,), "float32", 0)
    ref = O.reference("vecadd", inputs)
    bad = ref.clone()
    bad[100] += 1.0
    rtol, atol = O.tolerance("vecadd", "float32")
    assert not O.check(bad, ref, rtol, atol)["passed"]
    assert not O.check(ref * float("nan"), ref, rtol, atol)["passed"]
    assert O.check(ref.clone(), ref, rtol, atol)["passed"]


def test_oracle_online_softmax_matches_single_tile():
    """tests/test_tasks_and_emulation.py:83-91."""
    inputs = O.make_inputs("softmax", (16, 1000), "float32", 0)
    single = O.emulate("softmax", (16, 1000), {"BLOCK_N": 1024}, inputs)
    online = O.emulate("softmax", (16, 1000), {"BLOCK_N": 128}, inputs)
    assert torch.allclose(single, online, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_oracle_causal_attention_is_masked_softmax(dtype):
    """Causal oracle: the flash restatement equals the masked dense form, and
    the first query row attends only to key 0 (output row 0 == V row 0)."""
    shape = (2, 70, 32)
    ins = O.make_inputs("attention_causal", shape, dtype, 3)
    dense = O.reference("attention_causal", ins)
    flash = O.emulate("attention_causal", shape, {"BLOCK_N": 16}, ins)
    rtol, atol = O.tolerance("attention_causal", dtype)
    assert O.check(flash, dense, rtol, atol)["passed"]
    assert torch.allclose(dense[:, 0].float(), ins[2][:, 0].float(), atol=atol)


def test_oracle_gelu_matches_torch():
    ins = O.make_inputs("fused_gelu", (4096,), "float32", 1)
    ref = O.reference("fused_gelu", ins)
    z = ins[0] * O.FUSED_SCALE + ins[1]
    want = 0.5 * z * (1.0 + torch.erf(z / 2.0 ** 0.5))
    assert torch.allclose(ref, want, rtol=1e-5, atol=1e-6)
