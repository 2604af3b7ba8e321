"""Gated DeltaNet (Qwen3-Next linear attention) reference ops, fp32, varlen with state slots.

Semantics follow the public model definition (HF ``transformers`` ``Qwen3NextGatedDeltaNet``,
``modeling_qwen3_next.py``: ``torch_causal_conv1d_update``, ``torch_recurrent_gated_delta_rule``,
``Qwen3NextRMSNormGated``); the Trainium plugin has no such model.  The serving layout is
ours: a flat token batch split by ``query_start_loc`` and one persistent state slot per
running request (conv state ``[slots, C, K-1]``, recurrent state ``[slots, Hv, dk, dv]`` fp32).
``has_init[b]`` = the sequence continues from its slot's state (a later prefill segment or a
decode step); otherwise the state starts from zero.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, conv_state: torch.Tensor, qsl: torch.Tensor,
                  slots: torch.Tensor, has_init: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv (kernel K, no bias) + SiLU over each sequence's tokens.

    x [T, C] (row stride may exceed C); w [C, K]; conv_state [S, C, K-1] holds the last
    K-1 inputs of every slot and is updated in place."""
    T, C = x.shape
    K = w.shape[1]
    out = torch.empty(T, C, dtype=x.dtype, device=x.device)
    q = qsl.tolist()
    for b, s in enumerate(slots.tolist()):
        lo, hi = q[b], q[b + 1]
        if hi <= lo:
            continue
        prev = conv_state[s].float() if bool(has_init[b]) else torch.zeros(C, K - 1, device=x.device)
        xb = torch.cat([prev, x[lo:hi].float().t()], dim=1)  # [C, K-1+L]
        y = F.conv1d(xb[None], w.float()[:, None, :], groups=C)[0]  # [C, L]
        out[lo:hi] = F.silu(y).t().to(x.dtype)
        conv_state[s] = xb[:, -(K - 1):].to(conv_state.dtype)
    return out


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gate_and_beta(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor
                  ) -> tuple[torch.Tensor, torch.Tensor]:
    """Log-decay g = -exp(A_log) * softplus(a + dt_bias) and write strength beta = sigmoid(b)."""
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, b.float().sigmoid()


def gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                     state: torch.Tensor, qsl: torch.Tensor, slots: torch.Tensor, has_init: torch.Tensor,
                     scale: float | None = None) -> torch.Tensor:
    """Recurrent gated delta rule.  q, k [T, Hk, dk] (raw; L2-normalised here), v [T, Hv, dv],
    g, beta [T, Hv] fp32; value head h reads key head h // (Hv // Hk).  For every token:
    S <- exp(g) S;  S <- S + k (beta (v - S^T k))^T;  o = S^T (scale q).
    ``state`` [S, Hv, dk, dv] fp32 updated in place.  Returns o [T, Hv, dv] fp32."""
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    rep = Hv // Hk
    scale = dk ** -0.5 if scale is None else scale
    qn = l2norm(q.float()).repeat_interleave(rep, dim=1) * scale
    kn = l2norm(k.float()).repeat_interleave(rep, dim=1)
    vf = v.float()
    o = torch.zeros(T, Hv, dv, dtype=torch.float32, device=q.device)
    bounds = qsl.tolist()
    for b, s in enumerate(slots.tolist()):
        lo, hi = bounds[b], bounds[b + 1]
        if hi <= lo:
            continue
        S = state[s].clone() if bool(has_init[b]) else torch.zeros(Hv, dk, dv, device=q.device)
        for t in range(lo, hi):
            S = S * g[t].exp()[:, None, None]
            kv = torch.einsum("hkv,hk->hv", S, kn[t])
            delta = (vf[t] - kv) * beta[t][:, None]
            S = S + kn[t][:, :, None] * delta[:, None, :]
            o[t] = torch.einsum("hkv,hk->hv", S, qn[t])
        state[s] = S
    return o


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float, out_dtype=None) -> torch.Tensor:
    """Per-head RMSNorm of x [T, H, d] times weight, gated by silu(z) [T, H, d]."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (w.float() * y.to(out_dtype or x.dtype).float()) * F.silu(z.float())
    return y.to(out_dtype or x.dtype)


def chunked_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                             beta: torch.Tensor, state: torch.Tensor, qsl: torch.Tensor, slots: torch.Tensor,
                             has_init: torch.Tensor, scale: float | None = None, chunk: int = 64) -> torch.Tensor:
    """The chunked form of :func:`gated_delta_rule` that the prefill kernels implement.

    Per chunk of C tokens (G = in-chunk cumulative log decay):
      L_ij = beta_i (k_i . k_j) e^(G_i - G_j) (j < i),  T = (I + L)^-1  (UT transform),
      W = T (beta e^G k),  U = T (beta v),  P_ij = (q_i . k_j) e^(G_i - G_j) (j <= i);
    then, sequentially over chunks with state S [dk, dv]:
      V' = U - W S,  O = (e^G q) S + P V',  S <- e^(G_last) S + (e^(G_last - G) k)^T V'.
    Every exponent is <= 0 (g <= 0), so no term overflows."""
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    rep = Hv // Hk
    scale = dk ** -0.5 if scale is None else scale
    qn = (l2norm(q.float()).repeat_interleave(rep, dim=1) * scale).transpose(0, 1)  # [Hv, T, dk]
    kn = l2norm(k.float()).repeat_interleave(rep, dim=1).transpose(0, 1)
    vf = v.float().transpose(0, 1)  # [Hv, T, dv]
    gt, bt = g.float().t(), beta.float().t()  # [Hv, T]
    o = torch.zeros(Hv, T, dv, dtype=torch.float32, device=q.device)
    bounds = qsl.tolist()
    for b, s in enumerate(slots.tolist()):
        lo, hi = bounds[b], bounds[b + 1]
        S = state[s].clone() if bool(has_init[b]) else torch.zeros(Hv, dk, dv, device=q.device)
        for c0 in range(lo, hi, chunk):
            c1 = min(hi, c0 + chunk)
            C = c1 - c0
            qc, kc, vc = qn[:, c0:c1], kn[:, c0:c1], vf[:, c0:c1]
            G = gt[:, c0:c1].cumsum(-1)  # [Hv, C]
            bc = bt[:, c0:c1]
            dec = torch.exp((G[:, :, None] - G[:, None, :]).tril())  # masked below
            strict = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device), -1)
            causal = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device))
            L = (bc[:, :, None] * (kc @ kc.transpose(-1, -2)) * dec).masked_fill(~strict, 0)
            Tm = torch.linalg.solve_triangular(torch.eye(C, device=q.device) + L,
                                               torch.eye(C, device=q.device).expand(Hv, C, C), upper=False,
                                               unitriangular=True)
            W = Tm @ (bc[:, :, None] * G.exp()[:, :, None] * kc)
            U = Tm @ (bc[:, :, None] * vc)
            P = ((qc @ kc.transpose(-1, -2)) * dec).masked_fill(~causal, 0)
            Vn = U - W @ S
            o[:, c0:c1] = (qc * G.exp()[:, :, None]) @ S + P @ Vn
            Gl = G[:, -1]
            S = Gl.exp()[:, None, None] * S + (kc * (Gl[:, None] - G).exp()[:, :, None]).transpose(-1, -2) @ Vn
        if hi > lo:
            state[s] = S
    return o.transpose(0, 1).contiguous()
