"""Speculative-decoding verification with sampling (rejection sampling).

Counterpart of the Trainium plugin's probabilistic path (``vllm/sample/rejection_sampler.py:19``,
arXiv 2211.17192) for drafts proposed greedily by the EAGLE-3 draft model: the draft
distribution q is one-hot at the draft token d, so per verified position j
* the draft is accepted with probability min(1, p_j(d) / q(d)) = p_j(d);
* on rejection the emitted token is drawn from the residual norm(max(0, p_j - q)), i.e. p_j
  with d removed and renormalised, and verification stops;
* when every draft is accepted, a bonus token is drawn from p at the last position.
The emitted sequence is therefore distributed exactly as non-speculative sampling from p.
p_j is the request's sampling distribution (temperature, top-k, top-p) at position j; a
temperature <= 0 makes p one-hot at the argmax, which reduces to greedy accept-until-mismatch.

All randomness comes from host-supplied uniforms (per request and position), so every
tensor-parallel rank emits the same tokens.  Inputs are the candidate logits gathered over
the vocab shards (the same candidates the sampler uses).
"""

from __future__ import annotations

import torch

from ..ops import reference as ref


def rejection_sample(cand_logits: torch.Tensor, cand_ids: torch.Tensor, draft: torch.Tensor,
                     temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor, u_accept: torch.Tensor,
                     u_sample: torch.Tensor, max_top_k: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """Per verified position (rows): returns (token [N] int64, accepted [N] bool).

    cand_logits / cand_ids [N, C]: candidate logits and their vocab ids; draft [N] (-1 at a
    bonus position, which is always "rejected" and samples from p); temperature / top_k /
    top_p / uniforms [N].  ``token`` is the draft where accepted, else the resampled token;
    the caller keeps each sequence's tokens up to and including its first non-accepted row."""
    greedy_pos = cand_logits.float().argmax(-1)
    greedy_tok = cand_ids.gather(1, greedy_pos[:, None]).squeeze(1)
    t = temperature.float().clamp_min(1e-6)
    probs, order = ref.topk_topp_filter(cand_logits.float() / t[:, None], top_k, top_p, max_top_k)
    ids = cand_ids.gather(1, order)  # vocab ids of the filtered candidates
    is_draft = ids == draft[:, None]
    p_draft = (probs * is_draft).sum(-1)
    sampled_greedy = temperature <= 0
    accepted = torch.where(sampled_greedy, draft == greedy_tok, u_accept.float() < p_draft)
    accepted = accepted & (draft >= 0)
    resid = probs.masked_fill(is_draft & (draft[:, None] >= 0), 0.0)
    mass = resid.sum(-1, keepdim=True)
    resid = torch.where(mass > 0, resid / mass.clamp_min(1e-30), probs)
    cdf = resid.cumsum(-1)
    choice = (cdf <= u_sample.float()[:, None]).sum(-1).clamp(max=resid.shape[1] - 1)
    resampled = ids.gather(1, choice[:, None]).squeeze(1)
    resampled = torch.where(sampled_greedy, greedy_tok, resampled)
    token = torch.where(accepted, draft, resampled)
    return token.to(torch.int64), accepted
