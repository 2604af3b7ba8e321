"""Structured outputs: grammar-constrained sampling (JSON schema, JSON object, regex, choice,
EBNF grammar).

The reference takes vLLM's grammar bitmask from the scheduler output and applies it as a logit
mask before on-device sampling (``vllm/worker/neuron_model_runner.py:988-1060``, scheduler
``:884-894``; requests are refused when ``enable_structured_outputs`` is off,
``vllm/platform.py:396-435``).  Here the engine owns the grammar state itself: each constrained
request gets an xgrammar matcher at admission; every step the runner asks the matchers of the
rows it samples for their allowed-token bitmask (packed int32, one bit per vocabulary id), masks
its vocabulary shard of the logits with it, and the scheduler feeds every sampled token back to
the matcher, finishing the request when the grammar has terminated.  Steps with constrained
rows run outside the decode CUDA graphs (the mask is new every step), as the reference's mask
transfer is per step too.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class StructuredOutputsParams:
    """One constraint per request (vLLM's ``StructuredOutputsParams`` field names)."""

    json: Any = None            # JSON schema (dict or string)
    regex: str | None = None
    choice: list[str] | None = None
    grammar: str | None = None  # EBNF
    json_object: bool = False   # any JSON object
    disable_any_whitespace: bool = False  # JSON without free whitespace between tokens (compact)
    extra: dict = field(default_factory=dict)

    @classmethod
    def from_any(cls, obj: Any) -> "StructuredOutputsParams | None":
        if obj is None or isinstance(obj, cls):
            return obj
        get = obj.get if isinstance(obj, dict) else (lambda k, d=None: getattr(obj, k, d))
        p = cls(json=get("json"), regex=get("regex"), choice=get("choice"), grammar=get("grammar"),
                json_object=bool(get("json_object", False)),
                disable_any_whitespace=bool(get("disable_any_whitespace", False)))
        if sum(x is not None and x is not False for x in (p.json, p.regex, p.choice, p.grammar, p.json_object)) != 1:
            raise ValueError("structured outputs need exactly one of json, regex, choice, grammar, json_object")
        return p

    def key(self) -> tuple:
        j = self.json if isinstance(self.json, str) or self.json is None else json.dumps(self.json, sort_keys=True)
        return (j, self.regex, tuple(self.choice) if self.choice else None, self.grammar, self.json_object,
                self.disable_any_whitespace)


class StructuredOutputManager:
    """Compiles constraints (cached per constraint) and fills allowed-token bitmasks."""

    def __init__(self, tokenizer_info):
        import xgrammar as xgr

        self._xgr = xgr
        self.info = tokenizer_info
        self.vocab_size = tokenizer_info.vocab_size
        self.compiler = xgr.GrammarCompiler(tokenizer_info)
        self._cache: dict[tuple, Any] = {}

    @classmethod
    def from_tokenizer(cls, tokenizer, vocab_size: int | None = None) -> "StructuredOutputManager":
        import xgrammar as xgr

        return cls(xgr.TokenizerInfo.from_huggingface(tokenizer, vocab_size=vocab_size))

    def compile(self, p: StructuredOutputsParams):
        k = p.key()
        g = self._cache.get(k)
        if g is None:
            c = self.compiler
            if p.json is not None:
                g = c.compile_json_schema(p.json if isinstance(p.json, str) else json.dumps(p.json),
                                          any_whitespace=not p.disable_any_whitespace)
            elif p.json_object:
                g = c.compile_builtin_json_grammar()
            elif p.regex is not None:
                g = c.compile_regex(p.regex)
            elif p.choice is not None:
                g = c.compile_grammar("root ::= " + " | ".join(json.dumps(str(x)) for x in p.choice))
            else:
                g = c.compile_grammar(p.grammar)
            self._cache[k] = g
        return g

    def matcher(self, p: StructuredOutputsParams):
        return self._xgr.GrammarMatcher(self.compile(p))

    def bitmask(self, matchers: list) -> torch.Tensor:
        return fill_bitmask(matchers, self.vocab_size)


def fill_bitmask(matchers: list, vocab_size: int) -> torch.Tensor:
    """[len(matchers), ceil(vocab_size / 32)] int32 allowed-token bitmask; rows without a
    matcher (unconstrained sequences, padding) allow every token."""
    import xgrammar as xgr

    bm = xgr.allocate_token_bitmask(len(matchers), vocab_size)
    for i, m in enumerate(matchers):
        if m is None or not m.fill_next_token_bitmask(bm, i):
            bm[i].fill_(-1)
    return bm


def mask_logits(logits: torch.Tensor, bitmask: torch.Tensor, vocab_start: int) -> torch.Tensor:
    """Set to -inf every logit of this vocabulary shard ([rows, V_local], first id
    ``vocab_start``) whose bit is clear in the packed ``bitmask`` [rows, words]."""
    V = logits.shape[1]
    ids = torch.arange(vocab_start, vocab_start + V, device=logits.device)
    words = bitmask.shape[1]
    w = (ids // 32).clamp(max=words - 1)
    bits = (bitmask.to(logits.device)[:, w] >> (ids % 32).to(torch.int32)) & 1
    allowed = (bits != 0) & (ids < words * 32)
    return logits.masked_fill(~allowed, float("-inf"))
