"""Logit validation of the serving engine against a reference model
(``accuracy/logit_validation.py`` of the Trainium plugin).

* ``compare_logits(actual, expected)``: per-position metrics between two [T, V] logit
  tensors: max absolute error, top-1 agreement, top-k overlap, KL(expected || actual) and
  the greedy gap (how far the actual argmax sits below the expected maximum, in logits).
* ``validate_greedy_generation(llm, reference, prompts)``: generates greedily with the engine,
  teacher-forces the reference model (any callable ``ids [1, L] -> logits [1, L, V]``, e.g.
  an HF model) on prompt + generated tokens, and checks that every generated token is the
  reference argmax or within ``gap_tol`` logits of it; reports the first divergence.
* ``validate_prompt_logits(engine, reference, prompts)``: scores prompts with the engine
  (``LLMEngine.score``, all positions) and compares the full logits with ``compare_logits``.
* ``logit_validation(ids, generate_fn, expected)``: teacher-forced comparison with top-k
  tolerance tiers, ULP-aware handling of flipped near-ties and an optional three-way mode
  against fp32 logits; ``multi_prompt_logit_validation`` adds cross-prompt statistics and
  ``make_engine_generate_fn`` drives the engine's real decode path through its logit dumps.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class LogitMetrics:
    max_abs: float
    top1_agree: float
    topk_overlap: float
    kl: float
    max_greedy_gap: float
    per_position: list = field(default_factory=list, repr=False)


def compare_logits(actual: torch.Tensor, expected: torch.Tensor, top_k: int = 5) -> LogitMetrics:
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    if a.shape != e.shape:
        raise ValueError(f"logit shapes differ: {tuple(a.shape)} vs {tuple(e.shape)}")
    err = (a - e).abs().max(-1).values
    a1, e1 = a.argmax(-1), e.argmax(-1)
    ka, ke = a.topk(top_k, -1).indices, e.topk(top_k, -1).indices
    overlap = torch.tensor([len(set(x.tolist()) & set(y.tolist())) / top_k for x, y in zip(ka, ke)])
    lp_e, lp_a = torch.log_softmax(e, -1), torch.log_softmax(a, -1)
    kl = (lp_e.exp() * (lp_e - lp_a)).sum(-1)
    gap = e.max(-1).values - e.gather(-1, a1[:, None]).squeeze(-1)
    per = [{"pos": i, "max_abs": err[i].item(), "top1": bool(a1[i] == e1[i]), "kl": kl[i].item(),
            "gap": gap[i].item()} for i in range(a.shape[0])]
    return LogitMetrics(err.max().item(), (a1 == e1).float().mean().item(), overlap.mean().item(),
                        kl.max().item(), gap.max().item(), per)


@dataclass
class GenerationCheck:
    prompt_index: int
    tokens: list
    gaps: list
    first_divergence: int | None  # index of the first token beyond gap_tol (None = none)

    @property
    def passed(self) -> bool:
        return self.first_divergence is None


def validate_greedy_generation(llm, reference, prompts: list[list[int]], max_new_tokens: int = 16,
                               gap_tol: float = 0.05) -> list[GenerationCheck]:
    from ..engine.sampling_params import SamplingParams

    outs = llm.generate(prompt_token_ids=prompts,
                        sampling_params=SamplingParams(temperature=0, max_tokens=max_new_tokens, ignore_eos=True))
    checks = []
    with torch.no_grad():
        for i, (p, o) in enumerate(zip(prompts, outs)):
            toks = list(o.outputs[0].token_ids)
            full = torch.tensor([p + toks])
            logits = reference(full)
            logits = getattr(logits, "logits", logits)[0, len(p) - 1:len(p) - 1 + len(toks)].float()
            gaps = [(logits[j].max() - logits[j, t]).item() for j, t in enumerate(toks)]
            first = next((j for j, g in enumerate(gaps) if g > gap_tol), None)
            checks.append(GenerationCheck(i, toks, gaps, first))
    return checks


def validate_prompt_logits(engine, reference, prompts: list[list[int]], top_k: int = 5) -> list[LogitMetrics]:
    res = []
    with torch.no_grad():
        for p in prompts:
            got = engine.score(p)
            want = reference(torch.tensor([p]))
            want = getattr(want, "logits", want)[0]
            res.append(compare_logits(got[:, :want.shape[-1]], want, top_k))
    return res


# --------------------------------------------------------------------------------------------
# Teacher-forced logit validation with tolerance tiers, ULP-aware divergence and a three-way
# mode (``logit_validation`` ``accuracy/logit_validation.py:146``, ``multi_prompt_logit_validation``
# ``:1757`` of the Trainium plugin).
#
# generate_fn(ids) continues every sequence of ``ids`` greedily and returns logits [S', B, V]
# (or (logits, sampled ids [B, S'])).  The validator walks the expected sequence: every position
# up to and including the first one where the target's token differs from the teacher token
# (argmax of the fp32 baseline when given, else of the expected logits) is checked, then the
# teacher tokens up to there are appended to ``ids`` and generation restarts.  So every position
# is checked against the same context the reference saw, and one flipped near-tie does not make
# the rest of the sequence incomparable.
#
# Per position: positions that are -inf in either tensor are dropped; a constant offset of the
# target (least-squares fit target ~ a * expected + c) is removed; each tier ``k -> (atol, rtol)``
# of ``tol_map`` checks the expected top-k entries (``"all"``: every entry) with
# ``max(|t - e| - atol) / max|e| <= rtol``.  A divergent position passes when the target's
# logits of the two competing tokens are at most ``divergence_n_ulps`` units in the last place
# (of a float with ``mantissa_bits``; bf16 = 7) apart, or ``divergence_tol`` when n_ulps is None.
# --------------------------------------------------------------------------------------------

# Tiers and the fixed divergence tolerance are the reference's defaults, so verdicts agree.
DEFAULT_TOLERANCE_MAP = {"5": (1e-5, 0.011), "50": (1e-5, 0.02), "1000": (1e-5, 0.03), "all": (1e-5, 0.05)}
DEFAULT_DIVERGENCE_TOL = 1e-3
DEFAULT_AGGREGATE_CONFIG = {
    "pp_static_thresholds": [0.03, 0.05],
    "pp_linf_multipliers": [1.5, 2.0],
    "pp_l2_multipliers": [1.5, 2.0],
    "agg_bc_threshold": 0.99,
    "agg_sigma_ratio_threshold": 1.0,
}


def ulp(value: float, mantissa_bits: int = 7) -> float:
    """Spacing of floats with ``mantissa_bits`` explicit mantissa bits at ``|value|``:
    2^(floor(log2|value|) - mantissa_bits)."""
    a = abs(value)
    if not math.isfinite(a):
        return float("nan")
    if a < 1e-30:
        return 0.0
    return 2.0 ** (math.floor(math.log2(a)) - mantissa_bits)


@dataclass
class TokenCheck:
    batch: int
    index: int
    passed: bool
    tier_errors: dict            # tier -> max relative error
    mean_abs_error: float        # mean |t - e| / max|e|
    shift: float                 # removed constant offset
    divergence: bool
    divergence_gap: float
    divergence_limit: float
    three_way: dict | None = None  # base/tgt linf and l2, bc, passed (informational)


@dataclass
class ValidationResult:
    passed: bool
    tokens: list                 # [batch][position] -> TokenCheck
    label: str = ""

    def __bool__(self) -> bool:
        return self.passed

    def failures(self) -> list:
        return [t for row in self.tokens for t in row if not t.passed]

    def summary(self) -> str:
        n = sum(len(r) for r in self.tokens)
        bad = self.failures()
        div = sum(t.divergence for r in self.tokens for t in r)
        worst = {}
        for r in self.tokens:
            for t in r:
                for k, v in t.tier_errors.items():
                    worst[k] = max(worst.get(k, 0.0), v)
        head = (f"{self.label + ': ' if self.label else ''}{'PASS' if self.passed else 'FAIL'} "
                f"{n - len(bad)}/{n} positions, {div} divergent; worst per tier: "
                + ", ".join(f"top-{k} {v:.3g}" for k, v in worst.items()))
        lines = [head] + [f"  batch {t.batch} pos {t.index}: tiers {({k: round(v, 5) for k, v in t.tier_errors.items()})}"
                          f" divergence gap {t.divergence_gap:.3g} (limit {t.divergence_limit:.3g})" for t in bad[:20]]
        return "\n".join(lines)


def _drop_neg_inf(e: torch.Tensor, a: torch.Tensor, *others):
    keep = ~(torch.isneginf(e) | torch.isneginf(a))
    return keep, e[keep], a[keep], [o[keep] for o in others]


def _remove_shift(e: torch.Tensor, a: torch.Tensor) -> tuple[torch.Tensor, float]:
    """Least-squares fit a ~ s * e + c over the finite entries; returns a - c and c."""
    X = torch.stack([e.double(), torch.ones_like(e, dtype=torch.float64)], 1)
    sol = torch.linalg.lstsq(X, a.double()[:, None], driver="gelsd").solution
    c = float(sol[1, 0])
    return a - c, c


def _tier_error(e: torch.Tensor, a: torch.Tensor, k, atol: float) -> float:
    if k != "all":
        idx = torch.topk(e, min(int(k), e.numel())).indices
        e, a = e[idx], a[idx]
        ok = torch.isfinite(a)
        if not bool(ok.any()):
            return float("inf")
        e, a = e[ok], a[ok]
    m = float(e.abs().max()) if e.numel() else 0.0
    if m == 0.0:
        return 0.0 if bool(torch.equal(a, e)) else float("inf")
    return float(((a - e).abs() - atol).max()) / m


def _three_way(fp32: torch.Tensor, base: torch.Tensor, tgt: torch.Tensor, linf_mult: float, l2_mult: float) -> dict:
    from .tensor_compare import bhattacharyya

    ok = torch.isfinite(fp32) & torch.isfinite(base) & torch.isfinite(tgt)
    if not bool(ok.any()):
        return {"base_linf": float("inf"), "tgt_linf": float("inf"), "base_l2": float("inf"),
                "tgt_l2": float("inf"), "bc": 0.0, "passed": False, "base_errors": None, "tgt_errors": None}
    r, b, t = fp32[ok].float(), base[ok].float(), tgt[ok].float()
    rmax, rn = float(r.abs().max().clamp_min(1e-10)), float(r.norm().clamp_min(1e-10))
    db, dt = b - r, t - r
    m = {"base_linf": float(db.abs().max()) / rmax, "tgt_linf": float(dt.abs().max()) / rmax,
         "base_l2": float(db.norm()) / rn, "tgt_l2": float(dt.norm()) / rn,
         "base_errors": db.abs(), "tgt_errors": dt.abs()}
    m["bc"] = bhattacharyya(m["base_errors"], m["tgt_errors"])
    m["passed"] = m["tgt_linf"] < linf_mult * m["base_linf"] and m["tgt_l2"] < l2_mult * m["base_l2"]
    return m


def check_token_logits(expected: torch.Tensor, actual: torch.Tensor, tol_map: dict | None = None,
                       actual_token: int | None = None, baseline: torch.Tensor | None = None,
                       divergence_n_ulps: int | None = 1, mantissa_bits: int = 7,
                       divergence_tol: float = DEFAULT_DIVERGENCE_TOL, linf_mult: float = 1.5,
                       l2_mult: float = 1.5, batch: int = 0, index: int = 0) -> TokenCheck:
    """One position's check (see the section comment above); ``expected`` / ``actual`` /
    ``baseline`` are [V] logits, ``actual_token`` the target's sampled id (default: argmax)."""
    tol_map = tol_map or DEFAULT_TOLERANCE_MAP
    e, a = expected.detach().float().cpu(), actual.detach().float().cpu()
    if e.shape != a.shape:
        raise ValueError(f"logit shapes differ: {tuple(e.shape)} vs {tuple(a.shape)}")
    others = [baseline.detach().float().cpu()] if baseline is not None else []
    keep, e, a, others = _drop_neg_inf(e, a, *others)
    if actual_token is not None:
        if not bool(keep[actual_token]):
            raise ValueError(f"sampled token {actual_token} has a -inf logit")
        actual_token = int(keep[:actual_token].sum())
    if torch.isnan(a).any() or e.numel() == 0:
        nan = float("nan")
        return TokenCheck(batch, index, False, {k: float("inf") for k in tol_map}, nan, 0.0, True, nan, 0.0)
    a, shift = _remove_shift(e, a)
    a = a.float()
    tiers = {k: _tier_error(e, a, k, atol) for k, (atol, _) in tol_map.items()}
    tiers_ok = all(tiers[k] <= rtol for k, (_, rtol) in tol_map.items())
    emax = float(e.abs().max().clamp_min(1e-30))
    mean_abs = float((a - e).abs().mean()) / emax
    want = int(e.argmax())
    got = int(a.argmax()) if actual_token is None else actual_token
    divergent, gap, limit = want != got, 0.0, divergence_tol
    in_bounds = True
    if divergent:
        gap = abs(float(a[got]) - float(a[want]))
        if divergence_n_ulps is not None:
            limit = divergence_n_ulps * ulp(max(abs(float(a[got])), abs(float(a[want]))), mantissa_bits)
        in_bounds = gap <= limit
    tw = _three_way(others[0], e, a, linf_mult, l2_mult) if others else None
    return TokenCheck(batch, index, tiers_ok and in_bounds, tiers, mean_abs, shift, divergent, gap, limit, tw)


def logit_validation(input_ids: list[list[int]], generate_fn, expected_logits: torch.Tensor,
                     tol_map: dict | None = None, baseline_logits: torch.Tensor | None = None,
                     divergence_n_ulps: int | None = 1, mantissa_bits: int = 7,
                     divergence_tol: float = DEFAULT_DIVERGENCE_TOL, linf_mult: float = 1.5, l2_mult: float = 1.5,
                     label: str = "", verbose: bool = False) -> ValidationResult:
    """Teacher-forced validation of ``generate_fn`` against ``expected_logits`` [S, B, V]
    (see the section comment).  ``baseline_logits`` (fp32, same shape) switches on the
    three-way mode: teacher tokens come from it and every position also records the
    target's and the expected tensor's error against it.  ``input_ids`` is not modified."""
    ids = [list(x) for x in input_ids]
    B = len(ids)
    if expected_logits.dim() != 3 or expected_logits.shape[1] != B:
        raise ValueError(f"expected_logits must be [S, {B}, V], got {tuple(expected_logits.shape)}")
    if baseline_logits is not None and baseline_logits.shape != expected_logits.shape:
        raise ValueError("baseline_logits must have the shape of expected_logits")
    teacher = (baseline_logits if baseline_logits is not None else expected_logits).argmax(-1).T  # [B, S]
    S = teacher.shape[1]
    tokens: list[list[TokenCheck]] = [[] for _ in range(B)]
    passed, start = True, 0
    while start < S:
        out = generate_fn(ids)
        sampled = None
        if isinstance(out, tuple):
            out, sampled = out
            sampled = torch.as_tensor(sampled)
            if tuple(sampled.shape) != (B, out.shape[0]):
                raise ValueError(f"generate_fn returned logits {tuple(out.shape)} and ids {tuple(sampled.shape)}")
        if out.shape[0] == 0:
            raise RuntimeError("generate_fn returned no logits")
        n = min(out.shape[0], S - start)
        got = sampled[:, :n] if sampled is not None else out[:n].argmax(-1).T
        has_nan = bool(torch.isnan(out[:n].float()).any())
        diff = (got.cpu() != teacher[:, start:start + n].cpu()).any(0)
        stop = n if (has_nan or not bool(diff.any())) else int(diff.nonzero()[0]) + 1
        for b in range(B):
            for j in range(stop):
                g = start + j
                t = check_token_logits(expected_logits[g, b], out[j, b], tol_map,
                                       int(sampled[b, j]) if sampled is not None else None,
                                       baseline_logits[g, b] if baseline_logits is not None else None,
                                       divergence_n_ulps, mantissa_bits, divergence_tol, linf_mult, l2_mult, b, g)
                tokens[b].append(t)
                passed &= t.passed
        if has_nan:
            passed = False
            break
        for b in range(B):
            ids[b] += teacher[b, start:start + stop].tolist()
        start += stop
    res = ValidationResult(bool(passed), tokens, label)
    if verbose:
        print(res.summary())
    return res


@dataclass
class MultiPromptResult:
    passed: bool
    per_prompt: list             # ValidationResult per prompt
    aggregate: dict

    def __bool__(self) -> bool:
        return self.passed


def _aggregate(results: list[ValidationResult], cfg: dict) -> dict:
    """Cross-prompt statistics of the three-way metrics: per prompt, how many stay under
    static / relative thresholds; per position index (batch 0), the Bhattacharyya overlap of
    the pooled target and baseline error distributions; and the ratio of the pooled RMS
    errors (target / baseline)."""
    from .tensor_compare import bhattacharyya

    per = [[t.three_way for r in res.tokens for t in r if t.three_way is not None] for res in results]
    per = [p for p in per if p]
    agg: dict = {}
    if not per:
        return agg
    n = len(per)
    for th in cfg.get("pp_static_thresholds", []):
        agg[f"pp_static_{th}"] = f"{sum(max(m['tgt_linf'] for m in p) < th for p in per)}/{n}"
    for key in ("linf", "l2"):
        for mult in cfg.get(f"pp_{key}_multipliers", []):
            ok = sum(max(m[f"tgt_{key}"] for m in p) < mult * max(m[f"base_{key}"] for m in p) for p in per)
            agg[f"pp_max_{key}_{mult}x"] = f"{ok}/{n}"
    first = [[t.three_way for t in res.tokens[0] if t.three_way is not None] for res in results if res.tokens]
    first = [f for f in first if f]
    bcs = []
    for j in range(max((len(f) for f in first), default=0)):
        b = [f[j]["base_errors"] for f in first if len(f) > j and f[j]["base_errors"] is not None]
        t = [f[j]["tgt_errors"] for f in first if len(f) > j and f[j]["tgt_errors"] is not None]
        bcs.append(bhattacharyya(torch.cat(b), torch.cat(t)) if b and t else 0.0)
    agg["per_token_bc"] = bcs
    agg["agg_bc"] = "PASS" if bcs and min(bcs) >= cfg.get("agg_bc_threshold", 0.99) else "FAIL"
    be = [m["base_errors"] for p in per for m in p if m["base_errors"] is not None]
    te = [m["tgt_errors"] for p in per for m in p if m["tgt_errors"] is not None]
    if be and te:
        brms = float(torch.cat(be).square().mean().sqrt())
        trms = float(torch.cat(te).square().mean().sqrt())
        agg["agg_sigma_ratio"] = trms / brms if brms > 0 else float("inf")
    else:
        agg["agg_sigma_ratio"] = float("inf")
    return agg


def multi_prompt_logit_validation(prompts_input_ids: list[list[list[int]]], generate_fn,
                                  prompts_expected_logits: list[torch.Tensor],
                                  prompts_baseline_logits: list[torch.Tensor] | None = None,
                                  aggregate_config: dict | None = None, replicate_to_batch_size: int | None = None,
                                  **kwargs) -> MultiPromptResult:
    """``logit_validation`` per prompt (each prompt a batch [B][L]); with fp32 baselines the
    run also passes when the pooled statistics do (sigma ratio at most the threshold, or
    every position's error overlap at least ``agg_bc_threshold``), so a few borderline
    positions in one prompt do not fail a target whose errors match the dtype's own.
    ``replicate_to_batch_size`` repeats a batch-1 prompt B times (every copy must agree)."""
    cfg = dict(DEFAULT_AGGREGATE_CONFIG, **(aggregate_config or {}))
    results = []
    for i, ids in enumerate(prompts_input_ids):
        exp = prompts_expected_logits[i]
        base = prompts_baseline_logits[i] if prompts_baseline_logits is not None else None
        if replicate_to_batch_size and replicate_to_batch_size > 1:
            if exp.shape[1] != 1 or len(ids) != 1:
                raise ValueError("replicate_to_batch_size needs batch-1 prompts")
            r = replicate_to_batch_size
            ids = [list(ids[0]) for _ in range(r)]
            exp = exp.repeat(1, r, 1)
            base = base.repeat(1, r, 1) if base is not None else None
        results.append(logit_validation(ids, generate_fn, exp, baseline_logits=base,
                                        label=f"prompt {i + 1}/{len(prompts_input_ids)}", **kwargs))
    passed = all(r.passed for r in results)
    agg = {}
    if prompts_baseline_logits is not None:
        agg = _aggregate(results, cfg)
        passed = passed or agg.get("agg_sigma_ratio", float("inf")) <= cfg["agg_sigma_ratio_threshold"] \
            or agg.get("agg_bc") == "PASS"
    return MultiPromptResult(passed, results, agg)


def make_engine_generate_fn(llm, num_new_tokens: int, logits_dir: str):
    """``generate_fn`` for the validators backed by the serving engine's real decode path:
    greedy ``LLM.generate`` of ``num_new_tokens`` tokens per sequence with the engine's
    ``neuron_config.debug_logits_dir`` set to ``logits_dir``; returns (logits [n, B, V],
    ids [B, n]).  Stateless: the validators use only the positions they still need."""
    from ..engine.debug_logits import clear_debug_logits, read_debug_logits
    from ..engine.sampling_params import SamplingParams

    def fn(ids: list[list[int]]):
        n = num_new_tokens
        clear_debug_logits(logits_dir)
        outs = llm.generate(prompt_token_ids=[list(x) for x in ids],
                            sampling_params=SamplingParams(temperature=0, max_tokens=n, ignore_eos=True))
        d = read_debug_logits(logits_dir)
        keys = sorted(d)
        if len(keys) != len(ids):
            raise RuntimeError(f"{len(keys)} logit streams for {len(ids)} prompts")
        rows = [torch.stack([d[k][len(ids[b]) - 1 + j] for j in range(n)]) for b, k in enumerate(keys)]
        toks = torch.tensor([list(o.outputs[0].token_ids)[:n] for o in outs])
        return torch.stack(rows, 1), toks

    return fn
