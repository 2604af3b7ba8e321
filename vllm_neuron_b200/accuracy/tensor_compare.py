"""Tensor comparison for accuracy debugging (the reference's ``accuracy/tensor_compare.py``:
``align_shapes`` ``:137``, ``compare_tensors`` ``:195``, ``compare_tensors_three_way`` ``:255``,
Bhattacharyya-coefficient metric ``:176``).

* :func:`compare_tensors` -- error metrics of a target tensor against a reference (max / mean
  absolute error, relative L2, cosine similarity, fraction within tolerance).
* :func:`compare_tensors_three_way` -- judges the target against a high-precision reference
  (fp32) using a same-precision baseline (e.g. HF in bf16) as the yardstick: the target passes
  when its error distribution is no worse than the baseline's by a margin, measured by the
  ratio of mean errors and by the Bhattacharyya coefficient of the two error histograms.
* :func:`compare_captures` -- per-module comparison of two capture directories written by
  :class:`~vllm_neuron_b200.accuracy.tensor_capture.TensorCapture`.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class ComparisonResult:
    name: str
    shape: tuple
    max_abs: float
    mean_abs: float
    rel_l2: float
    cosine: float
    frac_close: float
    passed: bool

    def line(self) -> str:
        mark = "ok  " if self.passed else "FAIL"
        return (f"{mark} {self.name:<40} max {self.max_abs:.3e} mean {self.mean_abs:.3e} "
                f"relL2 {self.rel_l2:.3e} cos {self.cosine:.6f} close {self.frac_close:.4f}")


@dataclass
class ThreeWayResult:
    name: str
    target_mean_err: float
    baseline_mean_err: float
    ratio: float           # target mean error / baseline mean error
    bc: float              # Bhattacharyya coefficient of the two error histograms (1 = same shape)
    passed: bool


@dataclass
class AggregateMetrics:
    n: int = 0
    n_failed: int = 0
    worst: list = field(default_factory=list)  # names, worst relative L2 first

    @property
    def pass_rate(self) -> float:
        return 1.0 - self.n_failed / self.n if self.n else 1.0


def align_shapes(a: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Bring two captures of one tensor to a common shape: squeeze singleton dimensions,
    flatten leading dimensions when the element counts agree, otherwise truncate every
    dimension to the smaller size (padding rows of a bucketed run are dropped)."""
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    if a.shape == b.shape:
        return a, b
    sa, sb = a.squeeze(), b.squeeze()
    if sa.shape == sb.shape:
        return sa, sb
    if sa.numel() == sb.numel():
        return sa.reshape(-1), sb.reshape(-1)
    if sa.dim() == sb.dim():
        idx = tuple(slice(0, min(x, y)) for x, y in zip(sa.shape, sb.shape))
        return sa[idx], sb[idx]
    if sa.shape[-1] == sb.shape[-1]:
        fa, fb = sa.reshape(-1, sa.shape[-1]), sb.reshape(-1, sb.shape[-1])
        n = min(fa.shape[0], fb.shape[0])
        return fa[:n], fb[:n]
    raise ValueError(f"cannot align shapes {tuple(a.shape)} and {tuple(b.shape)}")


def bhattacharyya(errors1: torch.Tensor, errors2: torch.Tensor, bins: int = 100) -> float:
    """Overlap of the histograms of two error samples on a shared range: 1.0 for identical
    distributions, 0.0 for disjoint ones."""
    e1, e2 = errors1.reshape(-1).float(), errors2.reshape(-1).float()
    lo = float(min(e1.min(), e2.min()))
    hi = float(max(e1.max(), e2.max()))
    if hi <= lo:
        return 1.0
    h1 = torch.histc(e1, bins, lo, hi)
    h2 = torch.histc(e2, bins, lo, hi)
    p1, p2 = h1 / h1.sum().clamp_min(1), h2 / h2.sum().clamp_min(1)
    return float(torch.sqrt(p1 * p2).sum())


def compare_tensors(target: torch.Tensor, reference: torch.Tensor, name: str = "tensor", rtol: float = 1e-2,
                    atol: float = 1e-2, min_cosine: float = 0.999) -> ComparisonResult:
    """Error metrics of ``target`` against ``reference`` (shapes aligned first); passes when
    the cosine similarity reaches ``min_cosine`` and every element is within rtol / atol."""
    t, r = align_shapes(target, reference)
    err = (t - r).abs()
    rn = r.norm().item()
    cos = torch.nn.functional.cosine_similarity(t.reshape(1, -1), r.reshape(1, -1)).item() if t.numel() else 1.0
    close = (err <= atol + rtol * r.abs()).float().mean().item() if t.numel() else 1.0
    return ComparisonResult(name, tuple(t.shape), err.max().item() if t.numel() else 0.0,
                            err.mean().item() if t.numel() else 0.0, (t - r).norm().item() / max(rn, 1e-30), cos,
                            close, cos >= min_cosine and close == 1.0)


def compare_tensors_three_way(target: torch.Tensor, baseline: torch.Tensor, reference: torch.Tensor,
                              name: str = "tensor", max_ratio: float = 1.5, min_bc: float = 0.8) -> ThreeWayResult:
    """``reference``: high-precision result (e.g. HF fp32); ``baseline``: the same computation
    at the target's precision (e.g. HF bf16).  The target passes when its mean error is at
    most ``max_ratio`` times the baseline's, or when its error histogram overlaps the
    baseline's by at least ``min_bc`` (Bhattacharyya coefficient)."""
    t, r = align_shapes(target, reference)
    b, r2 = align_shapes(baseline, reference)
    et, eb = (t - r).abs(), (b - r2).abs()
    mt, mb = et.mean().item(), eb.mean().item()
    ratio = mt / mb if mb > 0 else (0.0 if mt == 0 else float("inf"))
    bc = bhattacharyya(et, eb)
    return ThreeWayResult(name, mt, mb, ratio, bc, ratio <= max_ratio or bc >= min_bc)


def compare_captures(target_dir: str, reference_dir: str, rank: int = 0, **tol) -> tuple[list, AggregateMetrics]:
    """Compare every captured module output of two capture directories (same prompts, same
    steps), step by step.  Returns the per-tensor results and aggregate metrics."""
    from .tensor_capture import load_captures

    a, b = load_captures(target_dir, rank), load_captures(reference_dir, rank)
    results = []
    for step, (sa, sb) in enumerate(zip(a, b)):
        ta, tb = sa.get("tensors", sa), sb.get("tensors", sb)
        for key in sorted(set(ta) & set(tb)):
            x, y = ta[key], tb[key]
            if isinstance(x, torch.Tensor) and isinstance(y, torch.Tensor):
                results.append(compare_tensors(x, y, f"step{step}/{key}", **tol))
    agg = AggregateMetrics(len(results), sum(not r.passed for r in results),
                           [r.name for r in sorted(results, key=lambda r: -r.rel_l2)[:10]])
    return results, agg


def report(results: list, agg: AggregateMetrics | None = None) -> str:
    lines = [r.line() for r in results]
    if agg is not None:
        lines.append(f"{agg.n - agg.n_failed}/{agg.n} passed; worst: {', '.join(agg.worst[:5])}")
    return "\n".join(lines)
