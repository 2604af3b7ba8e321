"""Accuracy assertions for kernels and models (``accuracy/testing.py`` of the Trainium plugin).

* ``assert_close(actual, expected)``: two-way check, errors normalised by the reference's
  absolute maximum (``|a - e| <= atol + rtol * max|e|``), per-dtype default tolerances.
* ``assert_close_three_way(reference, baseline, actual)``: separates error that the low
  precision itself causes from error specific to the code under test.  ``reference`` is a
  high-precision result (fp32), ``baseline`` the same computation in the low dtype by a
  trusted implementation (e.g. PyTorch bf16 on CPU), ``actual`` the kernel under test.  The
  actual error may exceed the baseline's by at most ``slack`` (on the max and the mean);
  beyond that the result is reported as target-specific (a bug), not dtype-inherent.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

# (rtol, atol): rtol is relative to the reference's absolute maximum
DTYPE_TOLERANCE = {
    torch.float32: (1.3e-6, 1e-5),
    torch.float16: (1e-3, 1e-5),
    torch.bfloat16: (1.6e-2, 1e-5),
    torch.float8_e4m3fn: (1.25e-1, 1e-3),
}


@dataclass
class CloseResult:
    name: str
    passed: bool
    max_abs: float
    mean_abs: float
    max_rel: float  # max error / max |expected|
    mismatch_frac: float
    rtol: float
    atol: float

    def summary(self) -> str:
        s = "PASS" if self.passed else "FAIL"
        return (f"[{s}] {self.name}: max_abs={self.max_abs:.3e} mean_abs={self.mean_abs:.3e} "
                f"max_rel={self.max_rel:.3e} mismatched={self.mismatch_frac:.2%} (rtol={self.rtol:g}, "
                f"atol={self.atol:g})")


@dataclass
class ThreeWayResult:
    name: str
    verdict: str  # "ok" | "dtype-inherent" | "target-specific"
    baseline: CloseResult
    actual: CloseResult
    slack: float

    @property
    def passed(self) -> bool:
        return self.verdict != "target-specific"

    def summary(self) -> str:
        return (f"[{self.verdict}] {self.name}: actual max_abs={self.actual.max_abs:.3e} "
                f"(baseline {self.baseline.max_abs:.3e}), mean_abs={self.actual.mean_abs:.3e} "
                f"(baseline {self.baseline.mean_abs:.3e}), slack x{self.slack:g}")


def _tol(dtype, rtol, atol):
    r, a = DTYPE_TOLERANCE.get(dtype, DTYPE_TOLERANCE[torch.float32])
    return (r if rtol is None else rtol), (a if atol is None else atol)


def compare(actual: torch.Tensor, expected: torch.Tensor, rtol: float | None = None, atol: float | None = None,
            name: str = "tensor") -> CloseResult:
    if actual.shape != expected.shape:
        raise ValueError(f"{name}: shape {tuple(actual.shape)} != {tuple(expected.shape)}")
    rtol, atol = _tol(actual.dtype, rtol, atol)
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    err = (a - e).abs()
    emax = e.abs().max().item() if e.numel() else 0.0
    bound = atol + rtol * emax
    nan_mismatch = (torch.isnan(a) != torch.isnan(e)).float().mean().item() if a.numel() else 0.0
    mism = ((err > bound) | torch.isnan(err)).float().mean().item() if a.numel() else 0.0
    return CloseResult(name, mism == 0.0 and nan_mismatch == 0.0, err.max().item() if a.numel() else 0.0,
                       err.mean().item() if a.numel() else 0.0,
                       (err.max().item() / emax) if emax > 0 else 0.0, mism, rtol, atol)


def assert_close(actual, expected, rtol: float | None = None, atol: float | None = None,
                 name: str = "tensor") -> CloseResult:
    """Two-way check; accepts tensors or (nested) lists / tuples of tensors."""
    if isinstance(actual, (list, tuple)):
        res = [assert_close(a, e, rtol, atol, f"{name}[{i}]") for i, (a, e) in enumerate(zip(actual, expected))]
        return res[-1] if res else CloseResult(name, True, 0, 0, 0, 0, 0, 0)
    r = compare(actual, expected, rtol, atol, name)
    if not r.passed:
        raise AssertionError(r.summary())
    return r


def assert_close_three_way(reference: torch.Tensor, baseline: torch.Tensor, actual: torch.Tensor,
                           name: str = "tensor", slack: float = 2.0, floor: float = 0.0) -> ThreeWayResult:
    """reference (high precision), baseline (low precision, trusted), actual (under test)."""
    b = compare(baseline, reference, rtol=float("inf"), atol=0.0, name=f"{name}/baseline")
    a = compare(actual, reference, rtol=float("inf"), atol=0.0, name=f"{name}/actual")
    ok_max = a.max_abs <= slack * b.max_abs + floor
    ok_mean = a.mean_abs <= slack * b.mean_abs + floor
    if ok_max and ok_mean:
        verdict = "ok" if a.max_abs <= b.max_abs + floor else "dtype-inherent"
    else:
        verdict = "target-specific"
    r = ThreeWayResult(name, verdict, b, a, slack)
    if not r.passed:
        raise AssertionError(r.summary())
    return r
