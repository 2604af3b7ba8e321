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
"""

from __future__ import annotations

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
