"""Mixture-of-experts references.

* router: linear (+bias) -> top-k -> softmax over the selected logits
  (``functional/moe/router.py:300-566``, GPT-OSS order "topk then softmax",
  ``model_mxfp4.py:949-955``); sigmoid / softmax-then-topk orders are provided for
  other models (Qwen3-Next uses softmax over all experts then top-k, renormalised).
* experts: gate/up interleaved along 2I (row 2i = gate_i, row 2i+1 = up_i), clamped
  SwiGLU ``gate.clamp(max=L) * sigmoid(alpha*gate) * (up.clamp(-L, L) + 1)``
  (``model_mxfp4.py:1104,1207-1211``), down projection, scaled by the affinity and
  summed over the top-k (``functional/moe/moe_cte.py:448``).
* blockwise mapping: tokens grouped per local expert in blocks of ``block_size``
  (``functional/moe/moe_blockwise.py:294``).
* all-to-all helpers: dedup per destination rank and 1-indexed token ids with -1
  padding (``functional/moe/permute_routed_tokens.py:32-35``, ``topk_reduce.py:35-39``).
"""

from __future__ import annotations

import torch


def router_topk(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, top_k: int,
                order: str = "topk_softmax", renormalize: bool = True
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (topk_ids [T,k] int32, topk_weights [T,k] fp32, router_logits [T,E] fp32)."""
    logits = x.float() @ weight.float().t()
    if bias is not None:
        logits = logits + bias.float()
    if order == "topk_softmax":
        vals, ids = torch.topk(logits, top_k, dim=-1)
        w = torch.softmax(vals, dim=-1)
    elif order == "softmax_topk":
        probs = torch.softmax(logits, dim=-1)
        w, ids = torch.topk(probs, top_k, dim=-1)
        if renormalize:
            w = w / w.sum(-1, keepdim=True)
    elif order == "sigmoid_topk":
        probs = torch.sigmoid(logits)
        w, ids = torch.topk(probs, top_k, dim=-1)
        if renormalize:
            w = w / w.sum(-1, keepdim=True)
    else:
        raise ValueError(order)
    return ids.to(torch.int32), w, logits


def clamped_swiglu(gate: torch.Tensor, up: torch.Tensor, alpha: float = 1.702, limit: float | None = 7.0
                   ) -> torch.Tensor:
    g, u = gate.float(), up.float()
    if limit is not None:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
        return g * torch.sigmoid(alpha * g) * (u + 1.0)
    return torch.nn.functional.silu(g) * u


def moe_experts(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, w13: torch.Tensor,
                b13: torch.Tensor | None, w2: torch.Tensor, b2: torch.Tensor | None, alpha: float = 1.702,
                limit: float | None = 7.0, interleaved: bool = True, expert_offset: int = 0,
                act: str = "swiglu_clamp") -> torch.Tensor:
    """x [T,H]; w13 [E_local, 2I, H]; w2 [E_local, H, I]; biases [E_local, 2I] / [E_local, H].

    Only routes whose expert falls in ``[expert_offset, expert_offset + E_local)``
    contribute (expert parallelism); the caller all-reduces the partial sums."""
    T, H = x.shape
    E_local = w13.shape[0]
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in range(E_local):
        ge = e + expert_offset
        tok, slot = torch.where(topk_ids == ge)
        if tok.numel() == 0:
            continue
        h = xf[tok] @ w13[e].float().t()
        if b13 is not None:
            h = h + b13[e].float()
        if interleaved:
            gate, up = h[:, 0::2], h[:, 1::2]
        else:
            I = h.shape[1] // 2
            gate, up = h[:, :I], h[:, I:]
        if act == "swiglu_clamp":
            a = clamped_swiglu(gate, up, alpha, limit)
        else:
            a = torch.nn.functional.silu(gate) * up
        y = a @ w2[e].float().t()
        if b2 is not None:
            y = y + b2[e].float()
        out.index_add_(0, tok, y * topk_weights[tok, slot].float()[:, None])
    return out.to(x.dtype)


def build_blockwise_mapping(topk_ids: torch.Tensor, num_local_experts: int, block_size: int,
                            expert_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Group (token, k) routes by local expert into blocks of ``block_size`` rows.

    Returns (token_position_to_id [N*bs] int32 (-1 = padding, else the flat route
    index t*k+j), block_to_expert [N] int32, expert_offsets [E_local+1] int32 (first
    block of each expert))."""
    T, k = topk_ids.shape
    flat = topk_ids.reshape(-1).long() - expert_offset
    routes = []
    block_to_expert = []
    offsets = [0]
    for e in range(num_local_experts):
        idx = torch.nonzero(flat == e).flatten()
        nblk = (idx.numel() + block_size - 1) // block_size
        pad = torch.full((nblk * block_size - idx.numel(),), -1, dtype=torch.long, device=topk_ids.device)
        routes.append(torch.cat([idx, pad]))
        block_to_expert += [e] * nblk
        offsets.append(offsets[-1] + nblk)
    tp = torch.cat(routes) if routes else torch.empty(0, dtype=torch.long)
    return (tp.to(torch.int32), torch.tensor(block_to_expert, dtype=torch.int32, device=topk_ids.device),
            torch.tensor(offsets, dtype=torch.int32, device=topk_ids.device))


def permute_routed_tokens(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                          experts_per_rank: int, world: int) -> tuple[list[torch.Tensor], list[torch.Tensor],
                                                                       list[torch.Tensor]]:
    """For every destination rank: the tokens that route to at least one of its
    experts (each token once), their local affinity rows [n, experts_per_rank] and
    1-indexed token ids.  Returns per-rank lists (rows, affinities, token_ids)."""
    T = x.shape[0]
    rows, affs, ids = [], [], []
    dst = topk_ids.long() // experts_per_rank
    for r in range(world):
        hit = (dst == r).any(-1)
        tok = torch.nonzero(hit).flatten()
        a = torch.zeros(tok.numel(), experts_per_rank, dtype=torch.float32, device=x.device)
        for j in range(topk_ids.shape[1]):
            sel = dst[tok, j] == r
            le = topk_ids[tok, j].long() - r * experts_per_rank
            a[torch.nonzero(sel).flatten(), le[sel]] = topk_weights[tok, j][sel].float()
        rows.append(x[tok])
        affs.append(a)
        ids.append((tok + 1).to(torch.int32))
    return rows, affs, ids


def topk_reduce(rows: torch.Tensor, token_ids: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """Sum combine-phase rows into their tokens: ``token_ids`` are 1-indexed, <=0 = pad."""
    out = torch.zeros(num_tokens, rows.shape[-1], dtype=torch.float32, device=rows.device)
    valid = token_ids > 0
    out.index_add_(0, (token_ids[valid] - 1).long(), rows[valid].float())
    return out.to(rows.dtype)
