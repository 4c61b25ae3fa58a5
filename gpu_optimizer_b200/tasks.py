"""Benchmark tasks: inputs, on-device validation reference, spaces, analytics.

Mirrors the reference's ``Task`` API (benchmarks/base.py:41-117 and the
per-task modules under benchmarks/) for the hot-path tasks, so the harness
and the search stack see the same methods:

* ``make_inputs``   seeded CPU ``torch.Generator`` per input (seed, seed+1,
                    ...), then moved to the device (benchmarks/base.py:112-117);
* ``reference``     the trusted torch computation the harness compares a
                    candidate against on the device (harness.py:179);
* ``baseline``      the library call whose latency defines speedup;
* ``param_space``   the tunable space; ``default_config`` the naive config;
* ``flops`` / ``bytes_moved`` / ``tolerance`` as in the reference.

Two profiles:

* ``"reference"`` — the reference's spaces and input distributions
  (parity contract, candidate ids identical to the reference's);
* ``"b200"`` — the B200 workload: spaces extended to BLOCK_* up to 256 /
  BLOCK_N up to 16384, and the input distributions of the B200 benchmark
  configurations (matmul N(0,1)/sqrt(K), softmax/layernorm X ~ N(0, var 2),
  layernorm gamma ~ N(1, 0.1) and beta ~ N(0, 0.1), vecadd / reduction
  U[-1, 1]).

Two workload variants are registered as separate tasks so that the
reference tasks' candidate ids stay stable: ``attention_causal`` and
``fused_gelu`` (y = gelu(x*w + b), erf form).
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch
import torch.nn.functional as F

from .space import Config, ParamSpace, ParamSpec

TORCH_DTYPES: dict[str, torch.dtype] = {
    "float32": torch.float32,
    "tf32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
}
DSIZE = {"float32": 4, "tf32": 4, "float16": 2, "bfloat16": 2}

# benchmarks/base.py:33-38
DEFAULT_TOLERANCES: dict[str, tuple[float, float]] = {
    "float32": (1e-4, 1e-5),
    "tf32": (1e-2, 1e-3),
    "float16": (1e-2, 1e-3),
    "bfloat16": (2e-2, 1e-2),
}

FUSED_SCALE = 0.7071  # benchmarks/fused_elementwise/task.py:19
LN_EPS = 1e-5         # benchmarks/layernorm/task.py:15


def _gen(shape: Sequence[int], dtype: str, device: str, seed: int, scale: float = 1.0,
         shift: float = 0.0) -> torch.Tensor:
    """Seeded normal input (benchmarks/base.py:112-117), optional mean shift."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = torch.randn(*shape, generator=g, dtype=torch.float32) * scale
    if shift:
        t = t + shift
    return t.to(device=device, dtype=TORCH_DTYPES[dtype])


def _uniform(shape: Sequence[int], dtype: str, device: str, seed: int) -> torch.Tensor:
    """Seeded U[-1, 1] input."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = torch.rand(*shape, generator=g, dtype=torch.float32) * 2.0 - 1.0
    return t.to(device=device, dtype=TORCH_DTYPES[dtype])


class Task:
    name = "abstract"
    supported_dtypes: tuple[str, ...] = ("float32", "float16", "bfloat16")
    roofline_bound = "hbm"  # "hbm" or "tensor"

    def __init__(self, profile: str = "reference") -> None:
        if profile not in ("reference", "b200"):
            raise ValueError(f"unknown profile {profile!r}")
        self.profile = profile

    # problem ------------------------------------------------------------
    def default_shapes(self) -> list[tuple[int, ...]]:
        raise NotImplementedError

    def make_inputs(self, shape, dtype, device, seed=0) -> tuple[torch.Tensor, ...]:
        raise NotImplementedError

    def reference(self, *inputs: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def baseline(self, *inputs: torch.Tensor) -> torch.Tensor:
        return self.reference(*inputs)

    # search -------------------------------------------------------------
    def param_space(self, shape) -> ParamSpace:
        raise NotImplementedError

    def default_config(self, shape) -> Config:
        raise NotImplementedError

    def make_candidate(self, shape, config: Config, provenance: str = "manual"):
        from .space import Candidate

        self.param_space(shape).validate(config)
        return Candidate(task=self.name, shape=tuple(int(s) for s in shape),
                         config=dict(config), provenance=provenance)

    # analytics ----------------------------------------------------------
    def flops(self, shape) -> float:
        raise NotImplementedError

    def bytes_moved(self, shape, dtype, config: Config | None = None) -> float:
        raise NotImplementedError

    def roofline_work(self, shape, dtype) -> float:
        """Algorithmic work of one call: bytes (hbm-bound) or FLOPs (tensor)."""
        raise NotImplementedError

    def tolerance(self, dtype: str) -> tuple[float, float]:
        return DEFAULT_TOLERANCES[dtype]

    def output_dtype(self, dtype: str) -> torch.dtype:
        return TORCH_DTYPES[dtype]


# --------------------------------------------------------------------- matmul
class MatmulTask(Task):
    """C = A @ B (benchmarks/matmul/task.py:16-80)."""

    name = "matmul"
    supported_dtypes = ("float32", "tf32", "float16", "bfloat16")
    roofline_bound = "tensor"

    def default_shapes(self):
        if self.profile == "b200":
            return [(4096, 4096, 4096), (8192, 8192, 8192)]
        return [(512, 512, 512), (1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)]

    def make_inputs(self, shape, dtype, device, seed=0):
        m, n, k = shape
        s = float(k) ** (-0.5 if self.profile == "b200" else -0.25)
        return _gen((m, k), dtype, device, seed, s), _gen((k, n), dtype, device, seed + 1, s)

    def reference(self, *inputs):
        a, b = inputs
        return (a.float() @ b.float()).to(a.dtype)

    def baseline(self, *inputs):
        a, b = inputs
        return a @ b

    def param_space(self, shape):
        if self.profile == "b200":
            specs = [
                ParamSpec("BLOCK_M", (32, 64, 128, 256)),
                ParamSpec("BLOCK_N", (32, 64, 128, 256)),
                ParamSpec("BLOCK_K", (32, 64, 128, 256)),
                ParamSpec("GROUP_M", (1, 4, 8, 16)),
                ParamSpec("num_warps", (4, 8)),
                ParamSpec("num_stages", (2, 3, 4, 5, 6)),
                ParamSpec("dtype", ("float32", "tf32", "float16", "bfloat16")),
            ]
        else:
            specs = [
                ParamSpec("BLOCK_M", (16, 32, 64, 128)),
                ParamSpec("BLOCK_N", (16, 32, 64, 128)),
                ParamSpec("BLOCK_K", (16, 32, 64)),
                ParamSpec("GROUP_M", (1, 4, 8)),
                ParamSpec("num_warps", (2, 4, 8)),
                ParamSpec("num_stages", (2, 3, 4, 5)),
                ParamSpec("dtype", ("float32", "tf32", "float16", "bfloat16")),
            ]
        return ParamSpace(specs, name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        return {"BLOCK_M": 32, "BLOCK_N": 32, "BLOCK_K": 16 if self.profile != "b200" else 32,
                "GROUP_M": 1, "num_warps": 4, "num_stages": 2, "dtype": "float32"}

    def flops(self, shape):
        m, n, k = shape
        return 2.0 * m * n * k

    def bytes_moved(self, shape, dtype, config=None):
        m, n, k = shape
        return float(DSIZE[dtype]) * (m * k + k * n + m * n)

    def roofline_work(self, shape, dtype):
        return self.flops(shape)

    def tolerance(self, dtype):
        return {"float32": (1e-4, 1e-4), "tf32": (2e-2, 2e-3),
                "float16": (2e-2, 2e-3), "bfloat16": (5e-2, 1e-2)}[dtype]


# --------------------------------------------------------------------- vecadd
class VecAddTask(Task):
    """out = x + y (benchmarks/vecadd/task.py:16-60)."""

    name = "vecadd"

    def default_shapes(self):
        return [(1 << 24,)] if self.profile == "b200" else [(1 << 20,), (1 << 24,), (1 << 26,)]

    def make_inputs(self, shape, dtype, device, seed=0):
        (n,) = shape
        if self.profile == "b200":
            return _uniform((n,), dtype, device, seed), _uniform((n,), dtype, device, seed + 1)
        return _gen((n,), dtype, device, seed), _gen((n,), dtype, device, seed + 1)

    def reference(self, *inputs):
        a, b = inputs
        return a + b

    def param_space(self, shape):
        return ParamSpace([
            ParamSpec("BLOCK_SIZE", (128, 256, 512, 1024, 2048, 4096)),
            ParamSpec("num_warps", (1, 2, 4, 8)),
            ParamSpec("dtype", ("float32", "float16", "bfloat16")),
        ], name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        return {"BLOCK_SIZE": 1024, "num_warps": 4, "dtype": "float32"}

    def flops(self, shape):
        return float(shape[0])

    def bytes_moved(self, shape, dtype, config=None):
        return 3.0 * shape[0] * DSIZE[dtype]

    def roofline_work(self, shape, dtype):
        return 3.0 * shape[0] * DSIZE[dtype]


# ------------------------------------------------------------------ reduction
class ReductionTask(Task):
    """y = sum(x), fp32 (benchmarks/reduction/task.py:18-77)."""

    name = "reduction"
    supported_dtypes = ("float32",)

    def default_shapes(self):
        return [(1 << 28,)] if self.profile == "b200" else [(1 << 20,), (1 << 24,), (1 << 26,)]

    def make_inputs(self, shape, dtype, device, seed=0):
        (n,) = shape
        if self.profile == "b200":
            return (_uniform((n,), dtype, device, seed),)
        return (_gen((n,), dtype, device, seed, 1.0),)

    def reference(self, *inputs):
        (x,) = inputs
        return x.double().sum().to(x.dtype).reshape(1)

    def baseline(self, *inputs):
        (x,) = inputs
        return x.sum().reshape(1)

    def param_space(self, shape):
        return ParamSpace([
            ParamSpec("BLOCK_SIZE", (256, 512, 1024, 2048, 4096, 8192)),
            ParamSpec("num_warps", (1, 2, 4, 8, 16)),
            ParamSpec("strategy", ("loop", "atomic", "two_pass")),
            ParamSpec("dtype", ("float32",)),
        ], name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        return {"BLOCK_SIZE": 1024, "num_warps": 4, "strategy": "two_pass", "dtype": "float32"}

    def flops(self, shape):
        return float(shape[0])

    def bytes_moved(self, shape, dtype, config=None):
        (n,) = shape
        base = 4.0 * n
        if config is not None and config.get("strategy") == "two_pass":
            block = int(config.get("BLOCK_SIZE", 1024))
            base += 2 * 4.0 * max(1, (n + block - 1) // block)
        return base

    def roofline_work(self, shape, dtype):
        return 4.0 * shape[0]

    def tolerance(self, dtype):
        return (1e-3, 1e-2)


# -------------------------------------------------------------------- softmax
class SoftmaxTask(Task):
    """Row softmax (benchmarks/softmax/task.py:16-71)."""

    name = "softmax"

    def default_shapes(self):
        return [(16384, 8192)] if self.profile == "b200" else [(4096, 1024), (8192, 2048),
                                                                (2048, 8192)]

    def make_inputs(self, shape, dtype, device, seed=0):
        m, n = shape
        scale = math.sqrt(2.0) if self.profile == "b200" else 1.0
        return (_gen((m, n), dtype, device, seed, scale),)

    def reference(self, *inputs):
        (x,) = inputs
        return torch.softmax(x.float(), dim=-1).to(x.dtype)

    def baseline(self, *inputs):
        (x,) = inputs
        return torch.softmax(x, dim=-1)

    def param_space(self, shape):
        if self.profile == "b200":
            specs = [ParamSpec("BLOCK_N", (1024, 2048, 4096, 8192, 16384)),
                     ParamSpec("num_warps", (4, 8, 16)),
                     ParamSpec("num_stages", (1, 2, 3, 4)),
                     ParamSpec("dtype", ("float16", "bfloat16"))]
        else:
            specs = [ParamSpec("BLOCK_N", (128, 256, 512, 1024, 2048, 4096)),
                     ParamSpec("num_warps", (1, 2, 4, 8, 16)),
                     ParamSpec("num_stages", (1, 2, 3, 4)),
                     ParamSpec("dtype", ("float32", "float16", "bfloat16"))]
        return ParamSpace(specs, name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        if self.profile == "b200":
            return {"BLOCK_N": 1024, "num_warps": 4, "num_stages": 2, "dtype": "bfloat16"}
        return {"BLOCK_N": 1024, "num_warps": 4, "num_stages": 2, "dtype": "float32"}

    def flops(self, shape):
        m, n = shape
        return 5.0 * m * n

    def bytes_moved(self, shape, dtype, config=None):
        m, n = shape
        passes = 2.0 if (config is not None and int(config.get("BLOCK_N", n)) < n) else 1.0
        return (passes + 1.0) * m * n * DSIZE[dtype]

    def roofline_work(self, shape, dtype):
        m, n = shape
        return 2.0 * m * n * DSIZE[dtype]


# ------------------------------------------------------------------ layernorm
class LayerNormTask(Task):
    """Row layernorm with affine (benchmarks/layernorm/task.py:18-87)."""

    name = "layernorm"

    def default_shapes(self):
        return [(16384, 8192)] if self.profile == "b200" else [(4096, 1024), (8192, 2048),
                                                                (16384, 512)]

    def make_inputs(self, shape, dtype, device, seed=0):
        m, n = shape
        if self.profile == "b200":
            return (_gen((m, n), dtype, device, seed, math.sqrt(2.0)),
                    _gen((n,), dtype, device, seed + 1, 0.1, shift=1.0),
                    _gen((n,), dtype, device, seed + 2, 0.1))
        return (_gen((m, n), dtype, device, seed), _gen((n,), dtype, device, seed + 1, 0.5),
                _gen((n,), dtype, device, seed + 2, 0.5))

    def reference(self, *inputs):
        x, w, b = inputs
        return F.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), LN_EPS).to(x.dtype)

    def baseline(self, *inputs):
        x, w, b = inputs
        return F.layer_norm(x, (x.shape[-1],), w, b, LN_EPS)

    def param_space(self, shape):
        # same spaces as softmax (benchmarks/layernorm/task.py:42-51)
        return ParamSpace(list(SoftmaxTask(self.profile).param_space(shape)),
                          name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        return SoftmaxTask(self.profile).default_config(shape)

    def flops(self, shape):
        m, n = shape
        return 8.0 * m * n

    def bytes_moved(self, shape, dtype, config=None):
        m, n = shape
        passes = 2.0 if (config is not None and int(config.get("BLOCK_N", n)) < n) else 1.0
        return (passes + 1.0) * m * n * DSIZE[dtype] + 2 * n * DSIZE[dtype]

    def roofline_work(self, shape, dtype):
        m, n = shape
        return 2.0 * m * n * DSIZE[dtype] + 2.0 * n * DSIZE[dtype]

    def tolerance(self, dtype):
        return {"float32": (1e-4, 1e-4), "float16": (2e-2, 2e-3),
                "bfloat16": (5e-2, 1e-2)}[dtype]


# ----------------------------------------------------------- fused elementwise
class FusedElementwiseTask(Task):
    """y = relu(x * 0.7071 + bias) (benchmarks/fused_elementwise/task.py:22-84)."""

    name = "fused_elementwise"

    def default_shapes(self):
        return [(1 << 26,)] if self.profile == "b200" else [(1 << 22,), (1 << 24,), (1 << 26,)]

    def make_inputs(self, shape, dtype, device, seed=0):
        (n,) = shape
        return _gen((n,), dtype, device, seed), _gen((n,), dtype, device, seed + 1, 0.5)

    def activation(self, z: torch.Tensor) -> torch.Tensor:
        return torch.relu(z)

    def reference(self, *inputs):
        x, bias = inputs
        return self.activation(x.float() * FUSED_SCALE + bias.float()).to(x.dtype)

    def baseline(self, *inputs):
        x, bias = inputs
        return self.activation(x * FUSED_SCALE + bias)

    def param_space(self, shape):
        return ParamSpace([
            ParamSpec("BLOCK_SIZE", (128, 256, 512, 1024, 2048, 4096)),
            ParamSpec("num_warps", (1, 2, 4, 8)),
            ParamSpec("strategy", ("fused", "unfused")),
            ParamSpec("dtype", ("float32", "float16", "bfloat16")),
        ], name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        return {"BLOCK_SIZE": 1024, "num_warps": 4, "strategy": "unfused", "dtype": "float32"}

    def flops(self, shape):
        return 3.0 * shape[0]

    def bytes_moved(self, shape, dtype, config=None):
        (n,) = shape
        d = DSIZE[dtype]
        if config is not None and config.get("strategy") == "unfused":
            return 7.0 * n * d
        return 3.0 * n * d

    def roofline_work(self, shape, dtype):
        return 3.0 * shape[0] * DSIZE[dtype]


class FusedGeluTask(FusedElementwiseTask):
    """y = gelu(x * w + b), erf form; w = 0.7071, same stream layout."""

    name = "fused_gelu"

    def activation(self, z):
        return F.gelu(z, approximate="none")

    def flops(self, shape):
        return 10.0 * shape[0]


# ------------------------------------------------------------------ attention
class AttentionTask(Task):
    """O = softmax(Q K^T / sqrt(D)) V, non-causal (benchmarks/attention/task.py:24-95)."""

    name = "attention"
    roofline_bound = "tensor"
    causal = False

    def default_shapes(self):
        if self.profile == "b200":
            return [(128, 4096, 128)]
        return [(16, 1024, 64), (32, 2048, 64), (16, 4096, 128)]

    def make_inputs(self, shape, dtype, device, seed=0):
        bh, s, d = shape
        return (_gen((bh, s, d), dtype, device, seed), _gen((bh, s, d), dtype, device, seed + 1),
                _gen((bh, s, d), dtype, device, seed + 2))

    def reference(self, *inputs):
        q, k, v = inputs
        bh, s, d = q.shape
        out = torch.empty_like(q)
        chunk = max(1, (1 << 28) // max(1, s * s))  # bound the fp32 score tensor
        mask = None
        if self.causal:
            mask = torch.ones(s, s, dtype=torch.bool, device=q.device).triu(1)
        for h0 in range(0, bh, chunk):
            qf, kf, vf = (t[h0:h0 + chunk].float() for t in (q, k, v))
            scores = qf @ kf.transpose(-2, -1) / math.sqrt(d)
            if mask is not None:
                scores = scores.masked_fill(mask, float("-inf"))
            out[h0:h0 + chunk] = (torch.softmax(scores, dim=-1) @ vf).to(q.dtype)
        return out

    def baseline(self, *inputs):
        q, k, v = inputs
        return F.scaled_dot_product_attention(q, k, v, is_causal=self.causal)

    def param_space(self, shape):
        if self.profile == "b200":
            specs = [ParamSpec("BLOCK_M", (64, 128, 256)), ParamSpec("BLOCK_N", (32, 64, 128)),
                     ParamSpec("num_warps", (4, 8)), ParamSpec("num_stages", (2, 3, 4)),
                     ParamSpec("dtype", ("float16", "bfloat16"))]
        else:
            specs = [ParamSpec("BLOCK_M", (16, 32, 64, 128)),
                     ParamSpec("BLOCK_N", (16, 32, 64, 128)),
                     ParamSpec("num_warps", (2, 4, 8)), ParamSpec("num_stages", (1, 2, 3)),
                     ParamSpec("dtype", ("float32", "float16", "bfloat16"))]
        return ParamSpace(specs, name=f"{self.name}-{tuple(shape)}")

    def default_config(self, shape):
        if self.profile == "b200":
            return {"BLOCK_M": 64, "BLOCK_N": 32, "num_warps": 4, "num_stages": 2,
                    "dtype": "bfloat16"}
        return {"BLOCK_M": 32, "BLOCK_N": 32, "num_warps": 4, "num_stages": 1,
                "dtype": "float32"}

    def flops(self, shape):
        bh, s, d = shape
        return 4.0 * bh * s * s * d + 5.0 * bh * s * s

    def bytes_moved(self, shape, dtype, config=None):
        bh, s, d = shape
        return 4.0 * bh * s * d * DSIZE[dtype]

    def roofline_work(self, shape, dtype):
        bh, s, d = shape
        return 4.0 * bh * s * s * d

    def tolerance(self, dtype):
        return {"float32": (1e-3, 1e-3), "float16": (2e-2, 2e-3),
                "bfloat16": (5e-2, 1e-2)}[dtype]


class CausalAttentionTask(AttentionTask):
    """Causal variant: key j is visible to query i iff j <= i."""

    name = "attention_causal"
    causal = True

    def flops(self, shape):
        bh, s, d = shape
        return 4.0 * bh * d * s * (s + 1) / 2 + 5.0 * bh * s * (s + 1) / 2

    def roofline_work(self, shape, dtype):
        bh, s, d = shape
        return 4.0 * bh * d * s * (s + 1) / 2


TASK_CLASSES: dict[str, type[Task]] = {
    c.name: c for c in (MatmulTask, VecAddTask, ReductionTask, SoftmaxTask, LayerNormTask,
                        FusedElementwiseTask, AttentionTask, CausalAttentionTask, FusedGeluTask)
}
REFERENCE_TASKS = ("matmul", "vecadd", "reduction", "softmax", "layernorm",
                   "fused_elementwise", "attention")


def get_task(name: str, profile: str = "reference") -> Task:
    if name not in TASK_CLASSES:
        raise KeyError(f"unknown task {name!r}; available: {sorted(TASK_CLASSES)}")
    return TASK_CLASSES[name](profile)
