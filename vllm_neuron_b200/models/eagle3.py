"""EAGLE-3 draft model (Llama-style single decoder layer).

Semantics of the Trainium plugin's ``Eagle3LlamaForCausalLM``
(``model/llama3/eagle3_model.py:309-593``) and the public EAGLE-3 design:
* ``fc`` combines the target's three auxiliary hidden states (low / middle / high layer
  inputs, concatenated) into one hidden vector (``combine_hidden_states``, :588);
* the decoder layer normalises the token embedding (``input_layernorm``) and the hidden
  state (``hidden_norm``), concatenates them (2H) as the attention input, keeps the
  hidden state (optionally after its norm) as the residual (:403-447);
* the output hidden state feeds the next recurrent step; logits over the draft
  vocabulary map to target ids through ``d2t`` (target = draft + d2t[draft]).
The draft runs replicated on every TP rank (it is one layer), with its own paged KV
cache addressed by the target's block tables.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable

import torch
import torch.nn as nn

from .. import ops
from ..nn.linear import RMSNorm
from ..ops import reference as ref
from .base import KVSpec, LayerSpec


@dataclass
class Eagle3Config:
    hidden_size: int = 4096
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    vocab_size: int = 128256
    draft_vocab_size: int = 32000
    target_hidden_size: int = 4096
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    norm_before_residual: bool = False
    max_position_embeddings: int = 131072

    @classmethod
    def from_hf(cls, d: dict, quantization: str | None = None) -> "Eagle3Config":
        rope = d.get("rope_scaling") or d.get("rope_parameters")
        theta = d.get("rope_theta") or (rope or {}).get("rope_theta", 10000.0)
        H = d["hidden_size"]
        return cls(hidden_size=H, num_attention_heads=d["num_attention_heads"],
                   num_key_value_heads=d.get("num_key_value_heads", d["num_attention_heads"]),
                   head_dim=d.get("head_dim") or H // d["num_attention_heads"],
                   intermediate_size=d["intermediate_size"], vocab_size=d["vocab_size"],
                   draft_vocab_size=d.get("draft_vocab_size", d["vocab_size"]),
                   target_hidden_size=d.get("target_hidden_size", H), rms_norm_eps=d.get("rms_norm_eps", 1e-5),
                   rope_theta=theta, rope_scaling=rope if rope and rope.get("rope_type") not in (None, "default")
                   else None, norm_before_residual=d.get("norm_before_residual", False),
                   max_position_embeddings=d.get("max_position_embeddings", 8192))


def _p(shape, dtype, device):
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


class Eagle3LlamaForCausalLM(nn.Module):
    config_class = Eagle3Config

    def __init__(self, cfg: Eagle3Config, ps=None, dtype=torch.bfloat16, device="cpu", kv_dtype=None):
        super().__init__()
        self.cfg = cfg
        H, d = cfg.hidden_size, cfg.head_dim
        self.nq, self.nkv, self.d = cfg.num_attention_heads, cfg.num_key_value_heads, d
        self.dtype = dtype
        self.kv_dtype = kv_dtype or dtype
        self.embed_tokens = _p((cfg.vocab_size, H), dtype, device)
        self.fc = _p((H, 3 * cfg.target_hidden_size), dtype, device)
        self.input_layernorm = RMSNorm(H, cfg.rms_norm_eps, device=device)
        self.hidden_norm = RMSNorm(H, cfg.rms_norm_eps, device=device)
        self.qkv = _p(((self.nq + 2 * self.nkv) * d, 2 * H), dtype, device)
        self.o_proj = _p((H, self.nq * d), dtype, device)
        self.post_attention_layernorm = RMSNorm(H, cfg.rms_norm_eps, device=device)
        self.gate_up = _p((2 * cfg.intermediate_size, H), dtype, device)
        self.down = _p((H, cfg.intermediate_size), dtype, device)
        self.norm = RMSNorm(H, cfg.rms_norm_eps, device=device)
        self.lm_head = _p((cfg.draft_vocab_size, H), dtype, device)
        self.register_buffer("d2t", torch.zeros(cfg.draft_vocab_size, dtype=torch.int64, device=device),
                             persistent=False)
        rs = cfg.rope_scaling
        if rs and rs.get("rope_type") == "llama3":
            inv, af = ref.llama3_inv_freq(d, cfg.rope_theta, rs["factor"], rs["low_freq_factor"],
                                          rs["high_freq_factor"], rs["original_max_position_embeddings"]), 1.0
        else:
            inv, af = ref.yarn_inv_freq(d, cfg.rope_theta)
        self.register_buffer("cos_sin", ops.build_cos_sin_cache(inv, min(cfg.max_position_embeddings, 1 << 16), af,
                                                                device=device), persistent=False)
        self.scale = 1.0 / math.sqrt(d)
        self.has_embed = False

    def get_kv_spec(self) -> KVSpec:
        return KVSpec([LayerSpec(self.nkv, self.d, self.kv_dtype)])

    def combine_hidden_states(self, aux: torch.Tensor) -> torch.Tensor:
        return ops.linear(aux, self.fc)

    def step(self, token_ids: torch.Tensor, positions: torch.Tensor, hidden: torch.Tensor, meta, kv) -> torch.Tensor:
        """One draft layer over a token batch.  Returns the new hidden state (pre-norm)."""
        emb = self.embed_tokens[token_ids]
        e = self.input_layernorm(emb)
        if self.cfg.norm_before_residual:
            hn = self.hidden_norm(hidden)
            residual = hn
        else:
            residual = hidden
            hn = self.hidden_norm(hidden)
        x = torch.cat([e, hn], dim=-1)
        qkv = ops.linear(x, self.qkv)
        k_cache, v_cache = kv
        q = ops.rope_and_cache(qkv, positions, self.cos_sin, k_cache, v_cache, meta.slot_mapping, self.nq, self.nkv,
                               self.d)
        o = ops.attention(q, k_cache, v_cache, meta, self.scale)
        a = ops.linear(o.reshape(o.shape[0], -1), self.o_proj)
        x2, residual = ops.fused_add_rms_norm(a, residual.clone(), self.post_attention_layernorm.weight,
                                              self.cfg.rms_norm_eps)
        m = ops.linear(ops.silu_and_mul(ops.linear(x2, self.gate_up)), self.down)
        return m + residual

    def logits_to_target_ids(self, h: torch.Tensor) -> torch.Tensor:
        logits = ops.linear(self.norm(h), self.lm_head)
        _, draft = ops.argmax(logits)
        return draft + self.d2t[draft]

    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        loaded = set()
        H = self.cfg.hidden_size
        I = self.cfg.intermediate_size
        for name, t in weights:
            n = name
            for pre in ("model.", "midlayer.", "layers.0."):
                if n.startswith(pre):
                    n = n[len(pre):]
            if n == "embed_tokens.weight":
                self.embed_tokens.data.copy_(t.to(self.dtype))
                self.has_embed = True
            elif n == "fc.weight":
                self.fc.data.copy_(t.to(self.dtype))
            elif n in ("input_layernorm.weight", "hidden_norm.weight", "post_attention_layernorm.weight",
                       "norm.weight"):
                getattr(self, n.split(".")[0]).weight.data.copy_(t.float())
            elif n.startswith("self_attn.") and n.split(".")[1] in ("q_proj", "k_proj", "v_proj"):
                which = n.split(".")[1][0]
                d = self.d
                off = {"q": 0, "k": self.nq * d, "v": (self.nq + self.nkv) * d}[which]
                self.qkv.data[off:off + t.shape[0]].copy_(t.to(self.dtype))
            elif n == "self_attn.o_proj.weight":
                self.o_proj.data.copy_(t.to(self.dtype))
            elif n == "mlp.gate_proj.weight":
                self.gate_up.data[:I].copy_(t.to(self.dtype))
            elif n == "mlp.up_proj.weight":
                self.gate_up.data[I:].copy_(t.to(self.dtype))
            elif n == "mlp.down_proj.weight":
                self.down.data.copy_(t.to(self.dtype))
            elif n == "lm_head.weight":
                self.lm_head.data.copy_(t.to(self.dtype))
            elif n == "d2t":
                self.d2t.copy_(t.long())
            else:
                continue
            loaded.add(name)
        del H
        return loaded
