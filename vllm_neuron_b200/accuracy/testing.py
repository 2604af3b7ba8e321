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


# ---------------------------------------------------------------------------------------
# End-to-end greedy check of an engine against a reference engine (teacher forcing)
# ---------------------------------------------------------------------------------------
TINY_GPT_OSS_D64 = {
    "architectures": ["GptOssForCausalLM"], "model_type": "gpt_oss", "vocab_size": 4096, "hidden_size": 256,
    "num_hidden_layers": 2, "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 64,
    "intermediate_size": 256, "num_local_experts": 8, "num_experts_per_tok": 2, "sliding_window": 128,
    "layer_types": ["sliding_attention", "full_attention"], "rope_theta": 150000.0,
    "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                     "original_max_position_embeddings": 4096},
    "rms_norm_eps": 1e-5, "swiglu_limit": 7.0, "attention_bias": True, "max_position_embeddings": 4096,
}


def write_tiny_gpt_oss_checkpoint(path: str, config: dict | None = None, seed: int = 0) -> dict:
    """A random GPT-OSS-architecture HF checkpoint (safetensors + config.json) for end-to-end
    checks: HF ``GptOssForCausalLM`` initialisation (seed), every bias and sink given a
    non-trivial value.  Returns the config written."""
    from transformers import GptOssConfig, GptOssForCausalLM

    from ..utils.checkpoints import save_state_dict

    cfg_d = dict(config or TINY_GPT_OSS_D64)
    torch.manual_seed(seed)
    hf_cfg = GptOssConfig(**{k: v for k, v in cfg_d.items() if k != "architectures"})
    m = GptOssForCausalLM(hf_cfg).eval().float()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("bias") or "sinks" in n:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    out_cfg = m.config.to_dict()
    out_cfg["architectures"] = ["GptOssForCausalLM"]
    save_state_dict({k: v.detach().clone() for k, v in m.state_dict().items()}, path, out_cfg)
    return out_cfg


@dataclass
class GreedyGapResult:
    n_tokens: int
    n_exact: int
    max_gap: float
    worst: tuple  # (prompt index, position, gap, row std)
    gaps: list  # (gap, row std) per generated position

    @property
    def exact_fraction(self) -> float:
        return self.n_exact / max(1, self.n_tokens)

    def outliers(self, abs_tol: float = 0.05, rel_tol: float = 0.2) -> int:
        """Positions whose gap exceeds max(abs_tol, rel_tol * row std).  A rare isolated
        outlier is a discrete flip (e.g. a router top-k near tie ordered differently in
        bf16 and fp32), not a numerical error of the kernels."""
        return sum(1 for g, sd in self.gaps if g > max(abs_tol, rel_tol * sd))


def greedy_logit_gaps(reference_engine, prompts: list[list[int]], generated: list[list[int]]) -> GreedyGapResult:
    """Teacher-forced check of greedy generations: the reference engine scores prompt +
    generation, and at every generated position the gap between its largest logit and the
    logit of the token the engine under test chose is measured (0 when they agree).  Near
    ties can legitimately flip under a different precision; a wrong kernel gives large gaps."""
    n = exact = 0
    gaps = []
    max_gap, worst = 0.0, (-1, -1, 0.0, 0.0)
    for i, (p, gen) in enumerate(zip(prompts, generated)):
        if not gen:
            continue
        logits = reference_engine.score(list(p) + list(gen[:-1])).float()
        for j, tok in enumerate(gen):
            row = logits[len(p) - 1 + j]
            gap = float(row.max() - row[tok])
            n += 1
            gaps.append((gap, float(row.std())))
            exact += int(int(row.argmax()) == int(tok) or gap == 0.0)
            if gap > max_gap:
                max_gap, worst = gap, (i, j, gap, float(row.std()))
    return GreedyGapResult(n, exact, max_gap, worst, gaps)
