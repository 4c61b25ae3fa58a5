"""Builds executable callables from candidate configurations (B200 backend).

Drop-in for the reference's ``compiler/triton/runner.py``: the same names
(``KernelBuildError``, ``KernelCallable``, ``build_callable``,
``warm_compile``, ``render_source``) and the same contract, with the Triton
JIT replaced by the sm_100a kernel library ``libgpo.so`` (include/gpo.h):

* ``build_callable`` maps (task, shape, config, inputs) to a zero-argument
  function that launches the configured kernel(s) on torch's current stream
  and returns the output tensor, which is allocated once at build time
  (runner.py:101-113).  Unknown tasks, configs outside every kernel family
  and resource overflow (shared memory, TMEM, register tile) raise
  ``KernelBuildError`` with the library's log (runner.py:52-72), which the
  harness records as ``compile_error``.
* ``warm_compile`` runs the callable once and synchronises; a launch
  failure becomes ``KernelBuildError`` (runner.py:75-89).  A device-side
  wait that timed out is not a compile failure: the callable is marked
  failed and its next call raises ``RuntimeError``, which both harnesses
  record as ``runtime_error`` (harness.py:182-184).
* ``render_source`` returns the CUDA source of the kernel family plus the
  resolved configuration, without a GPU (runner.py:275-297).

There is no fallback: if the library is missing every build raises.
"""

from __future__ import annotations

import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field

import torch

from . import _lib
from .space import Config
from .tasks import TORCH_DTYPES


def _available() -> bool:
    try:
        _lib.load()
    except Exception:
        return False
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(0)[0] == 10


GPO_AVAILABLE = _available()


class KernelBuildError(RuntimeError):
    """Raised when a candidate cannot be compiled/launched; log attached."""

    def __init__(self, message: str, log: str = "") -> None:
        super().__init__(message)
        self.log = log


@dataclass
class KernelCallable:
    """A ready-to-run candidate kernel."""

    fn: Callable[[], torch.Tensor]
    description: str
    launch: dict = field(default_factory=dict)
    module: object = None
    # set by warm_compile when the first run's device wait timed out; fn
    # then raises instead of launching
    state: dict = field(default_factory=dict)


_TASK_INPUTS = {"matmul": 2, "vecadd": 2, "reduction": 1, "softmax": 1, "layernorm": 3,
                "fused_elementwise": 2, "fused_gelu": 2, "attention": 3,
                "attention_causal": 3}


def compile_module(task: str, shape: Sequence[int], config: Config) -> _lib.Module:
    """Compile (plan) one candidate; raises KernelBuildError on failure."""
    if task not in _TASK_INPUTS:
        raise KernelBuildError(f"no B200 kernel family for task {task!r}")
    try:
        mod = _lib.Module(task, shape, config)
    except _lib.LibraryMissing as e:
        raise KernelBuildError(str(e), log=str(e)) from e
    except (KeyError, ValueError) as e:
        raise KernelBuildError(f"bad config: {e}", log=str(e)) from e
    if not mod.ok:
        name = _lib.status_name(mod.status)
        raise KernelBuildError(f"{name}: {mod.log}", log=mod.log)
    return mod


def _output_for(task: str, shape: Sequence[int], inputs, dtype: str) -> torch.Tensor:
    x = inputs[0]
    if task == "matmul":
        m, n, _k = shape
        return torch.empty((m, n), dtype=x.dtype, device=x.device)
    if task == "reduction":
        return torch.empty(1, dtype=torch.float32, device=x.device)
    return torch.empty_like(x)


def build_callable(task: str, shape: Sequence[int], config: Config,
                   inputs: tuple[torch.Tensor, ...]) -> KernelCallable:
    """Construct the launcher for one candidate.  Raises KernelBuildError."""
    shape = tuple(int(s) for s in shape)
    mod = compile_module(task, shape, config)
    want = TORCH_DTYPES[str(config.get("dtype", "float32"))]
    if len(inputs) != _TASK_INPUTS[task]:
        raise KernelBuildError(f"{task} takes {_TASK_INPUTS[task]} inputs, got {len(inputs)}")
    ins = []
    for t in inputs:
        if not t.is_cuda:
            raise KernelBuildError("inputs must be CUDA tensors")
        if t.dtype != want:
            raise KernelBuildError(f"input dtype {t.dtype} does not match config dtype {want}")
        ins.append(t.contiguous())
    res = mod.resources()
    out = _output_for(task, shape, ins, str(config.get("dtype")))
    scratch = [torch.empty(int(b), dtype=torch.uint8, device=ins[0].device) if b else None
               for b in res["scratch_bytes"]]
    args = _lib.GpoArgs()
    for i, t in enumerate(ins):
        args.in_[i] = t.data_ptr()
    args.out = out.data_ptr()
    for i, s in enumerate(scratch):
        args.scratch[i] = s.data_ptr() if s is not None else None
    args.scale = 0.0
    args.eps = 0.0
    keep = (ins, out, scratch)  # keep buffers alive as long as fn
    state: dict = {}

    def fn() -> torch.Tensor:
        _ = keep
        if state.get("failed"):
            raise RuntimeError(state["failed"])
        rc = mod.launch(args, torch.cuda.current_stream().cuda_stream)
        if rc != _lib.OK:
            raise RuntimeError(f"gpo_launch failed: {_lib.status_name(rc)}")
        return out

    launch = {"grid": res["grid"], "kernel": res["kernel"], "smem_bytes": res["smem_bytes"],
              "tmem_cols": res["tmem_cols"], "threads": res["threads_per_cta"],
              "launches_per_call": res["launches_per_call"], **config}
    return KernelCallable(fn, f"b200 {res['kernel']}", launch, mod, state)


def warm_compile(kc: KernelCallable) -> float:
    """Run once and synchronise; returns first-run seconds.

    A launch failure raises KernelBuildError (compile_error).  A device-side
    wait that timed out marks the callable failed instead, so that its next
    call raises RuntimeError (runtime_error in the harness).
    """
    t0 = time.perf_counter()
    try:
        kc.fn()
        rc, flags = _lib.device_status(torch.cuda.current_stream().cuda_stream)
    except Exception as e:
        raise KernelBuildError(f"first launch failed: {e}", log=str(e)) from e
    if rc == _lib.TIMEOUT:
        kc.state["failed"] = (f"device wait timed out on the first launch "
                              f"({_lib.status_name(rc)}, flags {flags:#x})")
    elif rc != _lib.OK:
        raise KernelBuildError(f"first launch failed: {_lib.status_name(rc)} (flags {flags:#x})")
    return time.perf_counter() - t0


def check_device_status() -> None:
    """Raise RuntimeError if a bounded device-side wait gave up since the last check."""
    rc, flags = _lib.device_status(torch.cuda.current_stream().cuda_stream)
    if rc != _lib.OK:
        raise RuntimeError(f"device status {_lib.status_name(rc)} (flags {flags:#x})")


def render_source(task: str, config: Config, shape: Sequence[int] | None = None) -> str:
    """CUDA source of the kernel family + resolved configuration (no GPU needed)."""
    if shape is None:
        shape = {"matmul": (4096, 4096, 4096), "attention": (16, 1024, 64),
                 "attention_causal": (16, 1024, 64), "softmax": (4096, 1024),
                 "layernorm": (4096, 1024)}.get(task, (1 << 20,))
    try:
        mod = compile_module(task, shape, config)
    except KernelBuildError as e:
        return f"// no kernel instantiation for task {task!r}: {e}\n"
    header = "\n".join(f"//   {k} = {v}" for k, v in sorted(config.items()))
    return f"// Candidate configuration:\n{header}\n{mod.source()}"
