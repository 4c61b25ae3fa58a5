"""Candidate correctness verification (compiler/validation/correctness.py:16-50).

``check_correctness`` keeps the reference's verdict exactly: elementwise
``|c - r| <= atol + rtol * |r|`` (torch.allclose semantics) with any
non-finite candidate value an automatic failure.  It additionally reports
the relative error over elements with ``|r| > atol`` (``rel_err_floored``),
the figure the B200 benchmark configurations bound (fp32 <= 1e-5,
tf32/bf16/fp16 <= 1e-2).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class CorrectnessReport:
    passed: bool
    max_abs_err: float
    max_rel_err: float
    rtol: float
    atol: float
    detail: str = ""
    rel_err_floored: float = 0.0

    def summary(self) -> str:
        status = "PASS" if self.passed else "FAIL"
        return (f"{status} (max_abs={self.max_abs_err:.3e}, max_rel={self.max_rel_err:.3e}, "
                f"rel_floored={self.rel_err_floored:.3e}, rtol={self.rtol:g}, "
                f"atol={self.atol:g})")


def check_correctness(candidate: torch.Tensor, reference: torch.Tensor,
                      rtol: float, atol: float) -> CorrectnessReport:
    if candidate.shape != reference.shape:
        return CorrectnessReport(False, float("inf"), float("inf"), rtol, atol,
                                 f"shape mismatch {tuple(candidate.shape)} vs "
                                 f"{tuple(reference.shape)}", float("inf"))
    c = candidate.detach().float()
    r = reference.detach().float()
    if not torch.isfinite(c).all():
        return CorrectnessReport(False, float("inf"), float("inf"), rtol, atol,
                                 "non-finite values in candidate output", float("inf"))
    if c.numel() == 0:
        return CorrectnessReport(True, 0.0, 0.0, rtol, atol)
    abs_err = (c - r).abs()
    max_abs = float(abs_err.max())
    denom = r.abs().clamp_min(1e-12)
    rel = abs_err / denom
    max_rel = float(rel.max())
    big = r.abs() > atol
    rel_floored = float(rel[big].max()) if bool(big.any()) else 0.0
    ok = bool((abs_err <= atol + rtol * r.abs()).all())
    return CorrectnessReport(ok, max_abs, max_rel, rtol, atol, "", rel_floored)
