"""CPU oracle for the gpu-optimizer hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only as the checker (or the timed CPU baseline);
the product kernels never route through it.

It restates, on the CPU with torch in fp32/fp64, what the reference computes
for every task on the hot path:

* ``make_inputs``  — seeded inputs (benchmarks/base.py:112-117 and each
  task's make_inputs), plus the B200 workload distributions;
* ``reference``    — each task's trusted torch reference
  (benchmarks/<task>/task.py ``reference``);
* ``emulate``      — the algorithm-faithful restatement of each candidate
  kernel (compiler/validation/emulation.py:31-159): chunked-K fp32
  accumulation with tf32 mantissa truncation, per-block partial sums,
  online softmax, the per-strategy layernorm variance formula, storage-dtype
  rounding of unfused intermediates, and P cast to V's dtype in attention;
* ``check``        — the allclose-with-NaN-failure verdict
  (compiler/validation/correctness.py:31-50).

Pinning: ``tests/golden/`` holds outputs of the reference's own
``task.reference`` and ``emulate`` on its seeded inputs (generated in the
build container by importing the reference; script committed beside the
fixtures); tests check this oracle against them bit-for-bit.  The causal
attention and gelu variants have no counterpart in the reference: their
oracle (fp32 softmax under a strict upper-triangular -inf mask; erf-form
gelu) is parity unpinned.
"""

from __future__ import annotations

import math

import torch

TORCH_DTYPES = {"float32": torch.float32, "tf32": torch.float32,
                "float16": torch.float16, "bfloat16": torch.bfloat16}
FUSED_SCALE = 0.7071  # benchmarks/fused_elementwise/task.py:19
LN_EPS = 1e-5         # benchmarks/layernorm/task.py:15


# ------------------------------------------------------------------- inputs
def gen(shape, dtype: str, seed: int, scale: float = 1.0, shift: float = 0.0) -> torch.Tensor:
    """benchmarks/base.py:112-117: randn from a seeded CPU generator, scaled, cast."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = torch.randn(*shape, generator=g, dtype=torch.float32) * scale
    if shift:
        t = t + shift
    return t.to(TORCH_DTYPES[dtype])


def uniform(shape, dtype: str, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.rand(*shape, generator=g, dtype=torch.float32) * 2.0 - 1.0).to(
        TORCH_DTYPES[dtype])


def make_inputs(task: str, shape, dtype: str, seed: int = 0, profile: str = "reference"):
    """Per-task seeded inputs (each benchmarks/<task>/task.py make_inputs)."""
    b200 = profile == "b200"
    if task == "matmul":  # matmul/task.py:23-30
        m, n, k = shape
        s = float(k) ** (-0.5 if b200 else -0.25)
        return gen((m, k), dtype, seed, s), gen((k, n), dtype, seed + 1, s)
    if task == "vecadd":  # vecadd/task.py:23-27
        (n,) = shape
        if b200:
            return uniform((n,), dtype, seed), uniform((n,), dtype, seed + 1)
        return gen((n,), dtype, seed), gen((n,), dtype, seed + 1)
    if task == "reduction":  # reduction/task.py:25-29
        (n,) = shape
        return (uniform((n,), dtype, seed) if b200 else gen((n,), dtype, seed),)
    if task == "softmax":  # softmax/task.py:23-26
        m, n = shape
        return (gen((m, n), dtype, seed, math.sqrt(2.0) if b200 else 1.0),)
    if task == "layernorm":  # layernorm/task.py:25-31
        m, n = shape
        if b200:
            return (gen((m, n), dtype, seed, math.sqrt(2.0)),
                    gen((n,), dtype, seed + 1, 0.1, shift=1.0), gen((n,), dtype, seed + 2, 0.1))
        return gen((m, n), dtype, seed), gen((n,), dtype, seed + 1, 0.5), gen((n,), dtype,
                                                                              seed + 2, 0.5)
    if task in ("fused_elementwise", "fused_gelu"):  # fused_elementwise/task.py:29-34
        (n,) = shape
        return gen((n,), dtype, seed), gen((n,), dtype, seed + 1, 0.5)
    if task in ("attention", "attention_causal"):  # attention/task.py:32-38
        bh, s, d = shape
        return gen((bh, s, d), dtype, seed), gen((bh, s, d), dtype, seed + 1), gen(
            (bh, s, d), dtype, seed + 2)
    raise KeyError(task)


# ---------------------------------------------------------------- reference
def _gelu(z: torch.Tensor) -> torch.Tensor:
    """Exact (erf) gelu in fp32, torch's implementation."""
    return torch.nn.functional.gelu(z, approximate="none")


def _attention(q, k, v, causal: bool) -> torch.Tensor:
    """attention/task.py:40-44 in per-head chunks; causal adds a triu(1) -inf mask."""
    bh, s, d = q.shape
    out = torch.empty(bh, s, d, dtype=q.dtype)
    chunk = max(1, (1 << 26) // max(1, s * s))
    mask = torch.ones(s, s, dtype=torch.bool).triu(1) if causal else None
    for h0 in range(0, bh, chunk):
        qf, kf, vf = (t[h0:h0 + chunk].float() for t in (q, k, v))
        scores = qf @ kf.transpose(-2, -1) / math.sqrt(d)
        if mask is not None:
            scores = scores.masked_fill(mask, float("-inf"))
        out[h0:h0 + chunk] = (torch.softmax(scores, dim=-1) @ vf).to(q.dtype)
    return out


def reference(task: str, inputs) -> torch.Tensor:
    """Each task's trusted reference, on CPU."""
    if task == "matmul":  # matmul/task.py:32-34
        a, b = inputs
        return (a.float() @ b.float()).to(a.dtype)
    if task == "vecadd":  # vecadd/task.py:29-31
        a, b = inputs
        return a + b
    if task == "reduction":  # reduction/task.py:31-33
        (x,) = inputs
        return x.double().sum().to(x.dtype).reshape(1)
    if task == "softmax":  # softmax/task.py:28-30
        (x,) = inputs
        return torch.softmax(x.float(), dim=-1).to(x.dtype)
    if task == "layernorm":  # layernorm/task.py:33-36
        x, w, b = inputs
        return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(),
                                              LN_EPS).to(x.dtype)
    if task == "fused_elementwise":  # fused_elementwise/task.py:36-38
        x, bias = inputs
        return torch.relu(x.float() * FUSED_SCALE + bias.float()).to(x.dtype)
    if task == "fused_gelu":
        x, bias = inputs
        return _gelu(x.float() * FUSED_SCALE + bias.float()).to(x.dtype)
    if task == "attention":
        return _attention(*inputs, causal=False)
    if task == "attention_causal":
        return _attention(*inputs, causal=True)
    raise KeyError(task)


# ----------------------------------------------------------------- emulation
def tf32_truncate(x: torch.Tensor) -> torch.Tensor:
    """emulation.py:25-28: clear the 13 low mantissa bits."""
    return (x.float().view(torch.int32) & ~0x1FFF).view(torch.float32)


def emulate(task: str, shape, config: dict, inputs) -> torch.Tensor:
    """Algorithm-faithful CPU run of one candidate (emulation.py:31-159)."""
    if task == "matmul":  # emulation.py:48-59
        a, b = inputs
        bk = int(config["BLOCK_K"])
        if config.get("dtype") == "tf32":
            af, bf = tf32_truncate(a), tf32_truncate(b)
        else:
            af, bf = a.float(), b.float()
        acc = torch.zeros(a.shape[0], b.shape[1], dtype=torch.float32)
        for k0 in range(0, a.shape[1], bk):
            acc += af[:, k0:k0 + bk] @ bf[k0:k0 + bk, :]
        return acc.to(a.dtype)
    if task == "vecadd":  # emulation.py:62-64
        x, y = inputs
        return x + y
    if task == "reduction":  # emulation.py:67-83: per-block fp32 partials, then their sum
        (x,) = inputs
        bs = int(config["BLOCK_SIZE"])
        xf = x.float()
        pad = (-xf.numel()) % bs
        partials = torch.nn.functional.pad(xf, (0, pad)).view(-1, bs).sum(dim=1)
        return partials.sum().to(x.dtype).reshape(1)
    if task == "softmax":  # emulation.py:86-106
        (x,) = inputs
        m, n = shape
        bn = int(config["BLOCK_N"])
        xf = x.float()
        if bn >= n:
            e = torch.exp(xf - xf.max(dim=1, keepdim=True).values)
            return (e / e.sum(dim=1, keepdim=True)).to(x.dtype)
        run_m = torch.full((m,), -float("inf"))
        run_s = torch.zeros(m)
        for i in range(0, n, bn):
            blk = xf[:, i:i + bn]
            nm = torch.maximum(run_m, blk.max(dim=1).values)
            run_s = run_s * torch.exp(run_m - nm) + torch.exp(blk - nm[:, None]).sum(dim=1)
            run_m = nm
        return (torch.exp(xf - run_m[:, None]) / run_s[:, None]).to(x.dtype)
    if task == "layernorm":  # emulation.py:109-124
        x, w, b = inputs
        _m, n = shape
        bn = int(config["BLOCK_N"])
        xf, wf, bf = x.float(), w.float(), b.float()
        if bn >= n:
            mean = xf.mean(dim=1, keepdim=True)
            var = ((xf - mean) ** 2).mean(dim=1, keepdim=True)
        else:
            mean = xf.sum(dim=1, keepdim=True) / n
            var = ((xf * xf).sum(dim=1, keepdim=True) / n - mean * mean).clamp_min(0.0)
        return ((xf - mean) / torch.sqrt(var + LN_EPS) * wf + bf).to(x.dtype)
    if task in ("fused_elementwise", "fused_gelu"):  # emulation.py:127-136
        x, bias = inputs
        act = torch.relu if task == "fused_elementwise" else _gelu
        if config.get("strategy") == "unfused":
            t1 = (x * FUSED_SCALE).to(x.dtype)
            t2 = (t1 + bias).to(x.dtype)
            return act(t2.float()).to(x.dtype) if task == "fused_gelu" else act(t2)
        return act(x.float() * FUSED_SCALE + bias.float()).to(x.dtype)
    if task in ("attention", "attention_causal"):  # emulation.py:139-159
        q, k, v = inputs
        bh, s, d = shape
        bn = int(config["BLOCK_N"])
        scale = 1.0 / math.sqrt(d)
        qf, kf, vf = q.float(), k.float(), v.float()
        acc = torch.zeros(bh, s, d)
        m_i = torch.full((bh, s), -float("inf"))
        l_i = torch.zeros(bh, s)
        rows = torch.arange(s)[:, None]
        for n0 in range(0, s, bn):
            qk = qf @ kf[:, n0:n0 + bn].transpose(-2, -1) * scale
            if task == "attention_causal":
                cols = torch.arange(n0, min(s, n0 + bn))[None, :]
                qk = qk.masked_fill(cols > rows, float("-inf"))
            m_new = torch.maximum(m_i, qk.max(dim=-1).values)
            safe = torch.where(torch.isinf(m_new), torch.zeros_like(m_new), m_new)
            alpha = torch.exp(m_i - safe)
            p = torch.exp(qk - safe[..., None])
            l_i = l_i * alpha + p.sum(dim=-1)
            acc = acc * alpha[..., None] + p.to(v.dtype).float() @ vf[:, n0:n0 + bn]
            m_i = m_new
        return (acc / l_i[..., None]).to(q.dtype)
    raise KeyError(task)


# ------------------------------------------------------------------- verdict
def check(candidate: torch.Tensor, ref: torch.Tensor, rtol: float, atol: float) -> dict:
    """correctness.py:31-50 verdict plus the error figures."""
    c = candidate.detach().float().cpu()
    r = ref.detach().float().cpu()
    if c.shape != r.shape:
        return {"passed": False, "max_abs": float("inf"), "max_rel": float("inf"),
                "detail": "shape mismatch"}
    if not torch.isfinite(c).all():
        return {"passed": False, "max_abs": float("inf"), "max_rel": float("inf"),
                "detail": "non-finite"}
    err = (c - r).abs()
    if err.numel() == 0:
        return {"passed": True, "max_abs": 0.0, "max_rel": 0.0, "detail": ""}
    rel = err / r.abs().clamp_min(1e-12)
    return {"passed": bool((err <= atol + rtol * r.abs()).all()),
            "max_abs": float(err.max()), "max_rel": float(rel.max()), "detail": ""}


# benchmarks/base.py:33-38 and the per-task overrides
def tolerance(task: str, dtype: str) -> tuple[float, float]:
    if task == "matmul":  # matmul/task.py:77-80
        return {"float32": (1e-4, 1e-4), "tf32": (2e-2, 2e-3), "float16": (2e-2, 2e-3),
                "bfloat16": (5e-2, 1e-2)}[dtype]
    if task == "reduction":  # reduction/task.py:75-77
        return (1e-3, 1e-2)
    if task == "layernorm":  # layernorm/task.py:85-87
        return {"float32": (1e-4, 1e-4), "float16": (2e-2, 2e-3), "bfloat16": (5e-2, 1e-2)}[dtype]
    if task in ("attention", "attention_causal"):  # attention/task.py:93-95
        return {"float32": (1e-3, 1e-3), "float16": (2e-2, 2e-3), "bfloat16": (5e-2, 1e-2)}[dtype]
    return {"float32": (1e-4, 1e-5), "tf32": (1e-2, 1e-3), "float16": (1e-2, 1e-3),
            "bfloat16": (2e-2, 1e-2)}[dtype]
