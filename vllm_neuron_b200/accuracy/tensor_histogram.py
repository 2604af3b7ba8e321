"""Distribution summaries of tensors (the reference's ``accuracy/tensor_histogram.py``:
``TensorHistogram`` ``:94``, ``BoxTable`` ``:43``): where the magnitudes of an activation, a
weight or an error tensor sit, to spot outliers, saturation (fp8 limits) or dead channels.

``TensorHistogram(t)`` buckets |t| by powers of two (plus zeros, NaN and Inf counts) and keeps
percentiles; ``render()`` draws the buckets as a text bar chart and ``box_table`` lines several
tensors up as box-plot rows (min, p1, p25, median, p75, p99, max)."""

from __future__ import annotations

import math

import torch

_PCTS = (0.0, 0.01, 0.25, 0.5, 0.75, 0.99, 1.0)


class TensorHistogram:
    def __init__(self, t: torch.Tensor, name: str = "tensor", max_samples: int = 1 << 22):
        x = t.detach().float().reshape(-1).cpu()
        self.name = name
        self.numel = x.numel()
        self.nan = int(torch.isnan(x).sum())
        self.inf = int(torch.isinf(x).sum())
        x = x[torch.isfinite(x)]
        self.zeros = int((x == 0).sum())
        if x.numel() > max_samples:  # percentiles from an even subsample
            x = x[:: x.numel() // max_samples + 1]
        self.mean = float(x.mean()) if x.numel() else 0.0
        self.std = float(x.std()) if x.numel() > 1 else 0.0
        q = torch.quantile(x, torch.tensor(_PCTS)) if x.numel() else torch.zeros(len(_PCTS))
        self.percentiles = dict(zip(_PCTS, q.tolist()))
        a = x.abs()
        a = a[a > 0]
        self.buckets: dict[int, int] = {}
        if a.numel():
            e = torch.floor(torch.log2(a)).to(torch.int64)
            vals, cnt = torch.unique(e, return_counts=True)
            self.buckets = {int(v): int(c) for v, c in zip(vals, cnt)}

    def render(self, width: int = 40) -> str:
        """Text bar chart of |x| per power-of-two bucket [2^e, 2^(e+1))."""
        lines = [f"{self.name}: n={self.numel} mean={self.mean:.4g} std={self.std:.4g} zeros={self.zeros} "
                 f"nan={self.nan} inf={self.inf}"]
        if not self.buckets:
            return lines[0]
        top = max(self.buckets.values())
        for e in range(min(self.buckets), max(self.buckets) + 1):
            c = self.buckets.get(e, 0)
            bar = "#" * (math.ceil(width * c / top) if c else 0)
            lines.append(f"  [2^{e:>4}, 2^{e + 1:>4}) {c:>10} {bar}")
        return "\n".join(lines)

    def row(self) -> list[float]:
        return [self.percentiles[p] for p in _PCTS]


def box_table(hists: list[TensorHistogram]) -> str:
    """One box-plot row per tensor: min, p1, p25, median, p75, p99, max."""
    head = f"{'tensor':<32}" + "".join(f"{h:>11}" for h in ("min", "p1", "p25", "p50", "p75", "p99", "max"))
    rows = [head]
    for h in hists:
        rows.append(f"{h.name[:32]:<32}" + "".join(f"{v:>11.4g}" for v in h.row()))
    return "\n".join(rows)
