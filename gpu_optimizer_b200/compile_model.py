"""The B200 backend's compile verdict as the simulated engine's compile model.

The reference's ``SimulatedBenchmarkEngine`` (benchmarks/harness.py:279)
decides which candidates fail to compile with ``AnalyticGPUModel.compiles``
(optimizer/world_model/analytic.py:44-52): a shared-memory estimate written
for Triton's software pipelining on the A100
(compiler/transformations/constraints.py:21-44) plus a register-pressure
score.  Its verdicts label the surrogate's P(compile) training data
(status ``compile_error`` -> ``compiled=False``).  On the B200 backend the
arbiter is ``gpo_compile``'s plan -- shared memory per CTA, TMEM columns,
register tiles, the kernel families' config rules -- which is pure host
logic and runs without a GPU.  ``B200CompileModel`` puts that verdict into
the simulated engine, so simulated and real runs label the same candidates
as compile failures.
"""

from __future__ import annotations

from collections.abc import Sequence


def b200_compiles(task: str, shape: Sequence[int], config: dict) -> tuple[bool, str]:
    """(True, "") when the B200 backend builds the candidate, else (False, log)."""
    from .runner import KernelBuildError, compile_module

    try:
        compile_module(task, tuple(int(s) for s in shape), config)
    except KernelBuildError as e:
        return False, f"B200 CompilationError: {e}"
    return True, ""


class B200CompileModel:
    """``AnalyticGPUModel``-compatible model whose ``compiles`` is the B200
    backend's verdict; every other method (latency, memory) comes from the
    wrapped model."""

    def __init__(self, base=None, hardware=None) -> None:
        self.base = base
        self.hardware = getattr(base, "hardware", hardware)

    def compiles(self, task, shape, config) -> tuple[bool, str]:
        return b200_compiles(getattr(task, "name", task), shape, config)

    def __getattr__(self, name: str):
        base = self.__dict__.get("base")
        if base is None:
            raise AttributeError(name)
        return getattr(base, name)


def use_b200_compile_model(engine):
    """Give a simulated engine (anything with a ``model`` attribute) the
    B200 compile verdict; returns the engine."""
    engine.model = B200CompileModel(engine.model)
    return engine
