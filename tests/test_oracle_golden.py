"""The oracle is pinned to the reference's own outputs (tests/golden/).

tests/golden/ was produced by running the reference's ``make_inputs``,
``task.reference`` and ``emulate`` (tests/golden/make_golden.py).  Here the
CPU oracle must reproduce every stored input hash and reference output
bit-for-bit, and the product's input generators must produce the same
inputs.  The blocked emulations (online softmax, blocked row statistics)
must match bit-for-bit on the machine that made the fixtures; torch's CPU
kernels for exp and for sums pick their vector code by the host's
instruction set, so on another host their float results may differ in the
last bits, and there each row must agree within a few units of the output
type's precision, relative to the row's largest value.
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
        assert_bits_or_ulps(out, data[e["key"]], case["dtype"], str(e["config"]))


EPS = {"float32": 2.0 ** -23, "float16": 2.0 ** -10, "bfloat16": 2.0 ** -7}
HOST_ULPS = 4  # units of the output type's precision, per row


def as_float(a, dtype):
    if dtype == "bfloat16":  # stored as its 16 raw bits
        return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return a.astype(np.float64)


def assert_bits_or_ulps(out, golden, dtype, msg):
    got = to_np(out)
    if np.array_equal(got, golden):
        return
    g, o = as_float(golden, dtype), as_float(got, dtype)
    scale = np.abs(g).max(axis=-1, keepdims=True)
    err = np.abs(o - g) / np.where(scale > 0, scale, 1.0)
    assert float(err.max()) <= HOST_ULPS * EPS[dtype], (msg, float(err.max()) / EPS[dtype])


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


def _causal_float64(q, k, v):
    """Causal attention in float64 with numpy: an implementation that shares
    no code with torch or with the oracle."""
    qd, kd, vd = (t.double().numpy() for t in (q, k, v))
    bh, s, d = qd.shape
    sc = np.einsum("bqd,bkd->bqk", qd, kd) / np.sqrt(d)
    sc = np.where(np.triu(np.ones((s, s), dtype=bool), 1)[None], -np.inf, sc)
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(axis=-1, keepdims=True)
    return torch.from_numpy(np.einsum("bqk,bkd->bqd", p, vd))


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("shape", [(3, 130, 32), (1, 1024, 128)], ids=str)
def test_causal_oracle_pinned_to_independent_implementations(shape, dtype):
    """The causal attention oracle, on the reference's seeded inputs (the
    inputs the golden index hashes for the attention task), agrees with
    torch's own causal kernel (scaled_dot_product_attention, is_causal=True,
    fp32 math on the CPU) to one rounding of the output, and with a float64
    numpy computation to fp32 accuracy before that rounding."""
    ins = O.make_inputs("attention_causal", shape, dtype, 0)
    if shape == tuple(INDEX["tasks"]["attention"]["shape"]) and dtype != "float16":
        for c in INDEX["tasks"]["attention"]["cases"]:
            if c["dtype"] == dtype and c["seed"] == 0:
                assert [sha(t) for t in ins] == c["input_sha"]
    ref = O.reference("attention_causal", ins)
    q, k, v = (t.float() for t in ins)
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    exact = _causal_float64(*ins)
    ulp = {"float32": 2.0 ** -23, "float16": 2.0 ** -10, "bfloat16": 2.0 ** -7}[dtype]
    mag = exact.abs().clamp_min(1e-3)
    # fp32: two fp32 summation orders (measured 2e-6 relative); 16-bit: one
    # output rounding apart at most
    to_sdpa = (ref.double() - sdpa.to(ref.dtype).double()).abs()
    bound = 1e-5 * mag + 1e-6 if dtype == "float32" else 1.01 * ulp * mag + 1e-6
    assert (to_sdpa <= bound).all(), float(to_sdpa.max())
    # against float64: half an output rounding plus fp32 noise
    assert ((ref.double() - exact).abs() <= 0.51 * ulp * mag + 2e-6).all()


def test_gelu_oracle_pinned_to_math_erf():
    """The fused gelu oracle against Python's math.erf in float64 (no torch
    in the loop), on the reference's seeded inputs of the elementwise task:
    within four fp32 units of the result plus 1e-6 absolute: in fp32 the
    formula 0.5 z (1 + erf(z / sqrt 2)) cancels in the negative tail (at
    z = -2.7, 1 + erf is 0.007 and carries erf's absolute rounding), which
    costs torch's fp32 gelu up to 5e-7 absolute there."""
    import math

    ins = O.make_inputs("fused_gelu", (10007,), "float32", 0)
    ref = O.reference("fused_gelu", ins)
    x, b = ins[0].double().tolist(), ins[1].double().tolist()
    w = float(torch.tensor(O.FUSED_SCALE, dtype=torch.float32))
    want = []
    for xi, bi in zip(x, b):
        z = float(np.float32(np.float32(xi) * np.float32(w)) + np.float32(bi))
        want.append(0.5 * z * (1.0 + math.erf(z / math.sqrt(2.0))))
    want = torch.tensor(want, dtype=torch.float64)
    err = (ref.double() - want).abs()
    assert (err <= 4 * 2.0 ** -23 * want.abs() + 1e-6).all(), float(err.max())
