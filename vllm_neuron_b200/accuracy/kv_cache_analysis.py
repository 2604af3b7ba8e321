"""KV-cache inspection (``accuracy/kv_cache_analysis.py`` of the Trainium plugin).

* ``gather_request_kv(k_cache, v_cache, block_ids, seq_len)``: a request's keys and values
  [seq_len, kv_heads, head_dim] out of the paged cache (HND blocks);
* ``compare_kv(a, b)``: per-head error statistics between two such gathers (e.g. this
  engine vs a reference run, or before / after a KV transfer);
* ``kv_stats(k, v)``: magnitude statistics per head (fp8 KV scale selection);
* ``KVSnapshot(engine)`` / ``extract_request_kv`` / ``extract_hf_kv``: every attention layer's
  keys and values of a request as ``{layer: (k, v)}`` with k, v [1, kv_heads, seq, head_dim],
  from the engine's paged cache (copied when the request finishes, before its blocks are
  freed) or from an HF model's cache;
* ``compare_kv_caches(expected, actual, baseline=None)``: per token, layer and head: cosine,
  relative L-inf and L2 errors; with an fp32 ``baseline`` the errors are measured against it
  and each (token, layer) also gets the Bhattacharyya overlap of the target's and the
  expected tensor's error distributions; ``aggregate_kv_bc_across_prompts`` and
  ``combined_bc_per_layer`` pool those errors over prompts (reference:
  ``accuracy/kv_cache_analysis.py`` ``compare_kv_caches`` ``:592``,
  ``aggregate_kv_bc_across_prompts`` ``:761``, ``compute_combined_bc_per_layer`` ``:828``).
"""

from __future__ import annotations

import re
from dataclasses import dataclass

import torch


def gather_request_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, block_ids: list[int], seq_len: int,
                      k_scale: float = 1.0, v_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    bs = k_cache.shape[2]
    nb = (seq_len + bs - 1) // bs
    idx = torch.tensor(block_ids[:nb], device=k_cache.device, dtype=torch.long)
    k = k_cache.index_select(0, idx).float() * k_scale  # [nb, H, bs, d]
    v = v_cache.index_select(0, idx).float() * v_scale
    k = k.permute(0, 2, 1, 3).reshape(nb * bs, k.shape[1], k.shape[3])[:seq_len]
    v = v.permute(0, 2, 1, 3).reshape(nb * bs, v.shape[1], v.shape[3])[:seq_len]
    return k, v


def compare_kv(a: torch.Tensor, b: torch.Tensor) -> dict:
    err = (a.float() - b.float()).abs()
    ref = b.float().abs().amax(dim=(0, 2)).clamp_min(1e-12)
    return {"max_abs": err.max().item(), "mean_abs": err.mean().item(),
            "max_rel_per_head": (err.amax(dim=(0, 2)) / ref).tolist(),
            "first_bad_position": int((err.amax(dim=(1, 2)) > 1e-2 * ref.max()).nonzero()[0].item())
            if (err.amax(dim=(1, 2)) > 1e-2 * ref.max()).any() else None}


def kv_stats(k: torch.Tensor, v: torch.Tensor) -> dict:
    return {"k_absmax_per_head": k.abs().amax(dim=(0, 2)).tolist(), "v_absmax_per_head": v.abs().amax(dim=(0, 2)).tolist(),
            "k_rms": k.pow(2).mean().sqrt().item(), "v_rms": v.pow(2).mean().sqrt().item()}


# ------------------------------------------------------------------------- extraction
def _layer_name(i: int) -> str:
    return f"layers.{i}.self_attn"


def _natural(name: str):
    return [int(t) if t.isdigit() else t for t in re.split(r"(\d+)", name)]


def extract_request_kv(engine, block_ids: list[int], seq_len: int) -> dict:
    """{layer: (k, v)} [1, kv_heads, seq_len, head_dim] fp32 of this rank's attention layers
    (its kv-head shard under tensor parallelism; see ``merge_tp_shards``), dequantised with
    the layer's fp8 KV scales."""
    runner = engine.worker.runner
    model = runner.model
    spec = model.get_kv_spec()
    layers = getattr(model, "layers", None)
    out = {}
    for i, (ls, kv) in enumerate(zip(spec.layers, runner.kv_caches)):
        if ls.kind != "attention" or kv is None:
            continue
        attn = getattr(layers[i], "self_attn", None) if layers is not None and i < len(layers) else None
        ks, vs = float(getattr(attn, "k_scale", 1.0)), float(getattr(attn, "v_scale", 1.0))
        k, v = gather_request_kv(kv[0], kv[1], block_ids, seq_len, ks, vs)
        out[_layer_name(i)] = (k.permute(1, 0, 2)[None].cpu(), v.permute(1, 0, 2)[None].cpu())
    return out


def merge_tp_shards(shards: list[dict]) -> dict:
    """Concatenate the kv-head shards of the tensor-parallel ranks (rank order)."""
    return {name: (torch.cat([s[name][0] for s in shards], 1), torch.cat([s[name][1] for s in shards], 1))
            for name in shards[0]}


class KVSnapshot:
    """Keeps the KV of every request that finishes while it is attached:
    ``snapshot.kv[request_id] = {layer: (k, v)}`` covering the tokens whose KV was written
    (prompt + output - 1).  Attach before ``generate``; ``close()`` detaches."""

    def __init__(self, engine):
        self.engine = engine
        self.kv: dict[str, dict] = {}
        engine.scheduler.on_finish.insert(0, self._grab)

    def _grab(self, req_id: str) -> None:
        req = self.engine.scheduler.requests.get(req_id)
        if req is None or not req.block_ids or req.num_computed_tokens == 0:
            return
        self.kv[req_id] = extract_request_kv(self.engine, list(req.block_ids), req.num_computed_tokens)

    def close(self) -> None:
        try:
            self.engine.scheduler.on_finish.remove(self._grab)
        except ValueError:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


@torch.no_grad()
def extract_hf_kv(model, input_ids: list[int]) -> dict:
    """{layer: (k, v)} [1, kv_heads, len, head_dim] fp32 of an HF causal LM run on ``input_ids``
    (keys after rotary embedding, as the paged cache holds them)."""
    out = model(torch.tensor([list(input_ids)]), use_cache=True)
    pkv = out.past_key_values
    res = {}
    n = len(pkv.layers) if hasattr(pkv, "layers") else len(pkv)
    for i in range(n):
        if hasattr(pkv, "layers"):
            k, v = pkv.layers[i].keys, pkv.layers[i].values
        else:
            k, v = pkv[i][0], pkv[i][1]
        res[_layer_name(i)] = (k.float().cpu(), v.float().cpu())
    return res


# ------------------------------------------------------------------------- comparison
@dataclass
class HeadMetrics:
    k_cos: float
    v_cos: float
    k_linf: float       # max|diff| / max|ref|
    v_linf: float
    k_l2: float         # ||diff|| / ||ref||
    v_l2: float
    base_k_linf: float = 0.0  # three-way: expected vs baseline
    base_v_linf: float = 0.0
    base_k_l2: float = 0.0
    base_v_l2: float = 0.0


@dataclass
class TokenKVMetrics:
    k_bc: float = 1.0
    v_bc: float = 1.0


@dataclass
class TokenKVErrors:
    base_k: torch.Tensor
    base_v: torch.Tensor
    tgt_k: torch.Tensor
    tgt_v: torch.Tensor


def _rel(ref: torch.Tensor, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per head (rows of [H, d]): cosine, relative L-inf, relative L2."""
    d = x - ref
    cos = torch.nn.functional.cosine_similarity(ref, x, dim=-1)
    linf = d.abs().amax(-1) / ref.abs().amax(-1).clamp_min(1e-10)
    l2 = d.norm(dim=-1) / ref.norm(dim=-1).clamp_min(1e-10)
    return cos, linf, l2


def compare_kv_caches(expected: dict, actual: dict, layers: list[str] | None = None, baseline: dict | None = None,
                      return_raw_errors: bool = False):
    """``result[token][layer] -> [HeadMetrics per head]`` (plus ``result[token][layer + "._bc"]
    -> TokenKVMetrics`` with a baseline).  Errors are relative to ``baseline`` when given,
    else to ``expected``.  Every tensor is [1, heads, seq, dim] and the sequence lengths must
    agree.  ``return_raw_errors`` also returns ``raw[token][layer] -> TokenKVErrors`` (absolute
    errors, for the cross-prompt aggregates)."""
    ref = baseline if baseline is not None else expected
    if layers is None:
        common = set(expected) & set(actual) & (set(baseline) if baseline is not None else set(expected))
        layers = sorted(common, key=_natural)
    from .tensor_compare import bhattacharyya

    for name in layers:
        for src, what in ((actual, "actual"), (expected, "expected")):
            if src[name][0].shape[2] != ref[name][0].shape[2]:
                raise ValueError(f"{name}: {what} has {src[name][0].shape[2]} positions, "
                                 f"reference {ref[name][0].shape[2]}")
    S = ref[layers[0]][0].shape[2] if layers else 0
    result, raw = [], []
    for t in range(S):
        tok, terr = {}, {}
        for name in layers:
            rk, rv = ref[name][0][0, :, t].float(), ref[name][1][0, :, t].float()
            ak, av = actual[name][0][0, :, t].float(), actual[name][1][0, :, t].float()
            kc, kl, k2 = _rel(rk, ak)
            vc, vl, v2 = _rel(rv, av)
            bk = torch.zeros_like(kl), torch.zeros_like(kl)
            bv = torch.zeros_like(vl), torch.zeros_like(vl)
            if baseline is not None:
                ek, ev = expected[name][0][0, :, t].float(), expected[name][1][0, :, t].float()
                bk = _rel(rk, ek)[1:]
                bv = _rel(rv, ev)[1:]
                e = TokenKVErrors((ek - rk).abs().reshape(-1), (ev - rv).abs().reshape(-1),
                                  (ak - rk).abs().reshape(-1), (av - rv).abs().reshape(-1))
                tok[name + "._bc"] = TokenKVMetrics(bhattacharyya(e.base_k, e.tgt_k), bhattacharyya(e.base_v, e.tgt_v))
                terr[name] = e
            tok[name] = [HeadMetrics(float(kc[h]), float(vc[h]), float(kl[h]), float(vl[h]), float(k2[h]),
                                     float(v2[h]), float(bk[0][h]), float(bv[0][h]), float(bk[1][h]),
                                     float(bv[1][h])) for h in range(kc.shape[0])]
        result.append(tok)
        raw.append(terr)
    return (result, raw) if return_raw_errors else result


def aggregate_kv_bc_across_prompts(all_raw: list, prompt_lens: list[int], layers: list[str] | None = None) -> dict:
    """``{generated token index: {layer: TokenKVMetrics}}``: for each output position (aligned
    at each prompt's end), the overlap of the pooled baseline and target errors over prompts."""
    from .tensor_compare import bhattacharyya

    if not all_raw:
        return {}
    n_gen = min(len(r) - p for r, p in zip(all_raw, prompt_lens))
    if n_gen <= 0:
        return {}
    layers = layers or sorted(all_raw[0][0], key=_natural)
    out = {}
    for g in range(n_gen):
        row = {}
        for name in layers:
            errs = [r[p + g][name] for r, p in zip(all_raw, prompt_lens) if name in r[p + g]]
            if errs:
                row[name] = TokenKVMetrics(
                    bhattacharyya(torch.cat([e.base_k for e in errs]), torch.cat([e.tgt_k for e in errs])),
                    bhattacharyya(torch.cat([e.base_v for e in errs]), torch.cat([e.tgt_v for e in errs])))
        out[g] = row
    return out


def combined_bc_per_layer(all_raw: list, layers: list[str] | None = None) -> dict:
    """``{layer: TokenKVMetrics}`` over every prompt and position."""
    from .tensor_compare import bhattacharyya

    if not all_raw:
        return {}
    layers = layers or sorted(all_raw[0][0], key=_natural)
    out = {}
    for name in layers:
        errs = [tok[name] for r in all_raw for tok in r if name in tok]
        if errs:
            out[name] = TokenKVMetrics(
                bhattacharyya(torch.cat([e.base_k for e in errs]), torch.cat([e.tgt_k for e in errs])),
                bhattacharyya(torch.cat([e.base_v for e in errs]), torch.cat([e.tgt_v for e in errs])))
    return out


def kv_report(result: list, linf_threshold: float = 1e-2) -> str:
    """One line per layer: worst relative L-inf of K and V over tokens and heads (with where),
    lowest cosine, and how many (token, head) pairs exceed ``linf_threshold``."""
    if not result:
        return "no tokens compared"
    names = [n for n in result[0] if not n.endswith("._bc")]
    lines = [f"{'layer':<28}{'k_linf':>10}{'at':>10}{'v_linf':>10}{'at':>10}{'min_cos':>10}{'over':>8}"]
    for n in names:
        wk = wv = (-1.0, (0, 0))
        mc, over = 1.0, 0
        for t, tok in enumerate(result):
            for h, m in enumerate(tok[n]):
                if m.k_linf > wk[0]:
                    wk = (m.k_linf, (t, h))
                if m.v_linf > wv[0]:
                    wv = (m.v_linf, (t, h))
                mc = min(mc, m.k_cos, m.v_cos)
                over += (m.k_linf > linf_threshold) + (m.v_linf > linf_threshold)
        lines.append(f"{n:<28}{wk[0]:>10.3g}{'t%d h%d' % wk[1]:>10}{wv[0]:>10.3g}{'t%d h%d' % wv[1]:>10}"
                     f"{mc:>10.6f}{over:>8}")
    return "\n".join(lines)
