"""Candidate correctness verification (compiler/validation/correctness.py:16-50).

``check_correctness`` keeps the reference's verdict exactly: elementwise
``|c - r| <= atol + rtol * |r|`` (torch.allclose semantics) with any
non-finite candidate value an automatic failure.  It additionally reports
two relative errors:

* ``rel_err_normwise``: the largest row-wise relative error
  ``||c - r||_2 / ||r||_2`` over the rows of the last dimension (a 1-D
  output is one row).  This is the figure the B200 benchmark
  configurations bound -- fp32 <= 1e-5, tf32/bf16/fp16 <= 1e-2 -- because
  it stays meaningful where single output elements sit near zero (a
  causal-attention row that averages two value rows of opposite sign);
* ``rel_err_floored``: the largest elementwise relative error over the
  elements with ``|r| > atol``, which such near-cancelling elements
  dominate.
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
    rel_err_normwise: float = 0.0

    def summary(self) -> str:
        status = "PASS" if self.passed else "FAIL"
        return (f"{status} (max_abs={self.max_abs_err:.3e}, max_rel={self.max_rel_err:.3e}, "
                f"rel_floored={self.rel_err_floored:.3e}, "
                f"rel_normwise={self.rel_err_normwise:.3e}, rtol={self.rtol:g}, "
                f"atol={self.atol:g})")


# Bounds of the B200 benchmark configurations on ``rel_err_normwise``.
NORMWISE_BOUND = {"float32": 1e-5, "tf32": 1e-2, "float16": 1e-2, "bfloat16": 1e-2}


def rowwise_relative_error(candidate: torch.Tensor, reference: torch.Tensor) -> float:
    """max over rows of ||c - r||_2 / ||r||_2 (rows of the last dimension).

    A row whose reference norm is zero contributes its absolute error norm.
    """
    c = candidate.detach().double()
    r = reference.detach().double()
    if c.numel() == 0:
        return 0.0
    if c.dim() == 0:
        c, r = c.reshape(1), r.reshape(1)
    c = c.reshape(-1, c.shape[-1])
    r = r.reshape(-1, r.shape[-1])
    num = torch.linalg.vector_norm(c - r, dim=1)
    den = torch.linalg.vector_norm(r, dim=1)
    rel = torch.where(den > 0, num / den.clamp_min(1e-300), num)
    return float(rel.max())


def check_correctness(candidate: torch.Tensor, reference: torch.Tensor,
                      rtol: float, atol: float) -> CorrectnessReport:
    if candidate.shape != reference.shape:
        return CorrectnessReport(False, float("inf"), float("inf"), rtol, atol,
                                 f"shape mismatch {tuple(candidate.shape)} vs "
                                 f"{tuple(reference.shape)}", float("inf"), float("inf"))
    c = candidate.detach().float()
    r = reference.detach().float()
    if not torch.isfinite(c).all():
        return CorrectnessReport(False, float("inf"), float("inf"), rtol, atol,
                                 "non-finite values in candidate output", float("inf"),
                                 float("inf"))
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
    return CorrectnessReport(ok, max_abs, max_rel, rtol, atol, "", rel_floored,
                             rowwise_relative_error(c, r))
