"""Captured forward passes on disk in the layout the reference's capture readers use
(``accuracy/tensor_io.py`` of the Trainium plugin: ``read`` ``:145``, ``write`` ``:180``), so
captures from the two frameworks and from HF go through one set of comparison scripts.

Layout::

    capture_dir/
      dp{replica}/
        prefill_s{tokens}_{n}/            (or decode_b{seqs}_{n})
          {module name}/rank{r}.pt
          prefill_s{tokens}_{n}_meta.json  ({"req_ids", "positions", "dp_rank"})

``from_capture_steps`` converts the per-step files ``TensorCapture`` writes
(``step_<n>_rank<r>.pt``) into this form; ``capture_hf`` records an HF model's module outputs
for a prompt (one prefill pass, then one decode pass per generated token, greedy, with the
HF cache) in the same form, with module names mapped to this framework's names.
"""

from __future__ import annotations

import json
import os
import re
from dataclasses import dataclass, field

import torch


@dataclass
class ForwardPassMetadata:
    req_ids: list
    positions: list
    dp_rank: int = 0


@dataclass
class CapturedForwardPass:
    dir_name: str
    metadata: ForwardPassMetadata
    tensors: dict = field(default_factory=dict)  # {module name: {tp rank: tensor}}

    @property
    def is_prefill(self) -> bool:
        return self.dir_name.startswith("prefill_s")


def write(replica_dir: str, passes: list[CapturedForwardPass]) -> None:
    os.makedirs(replica_dir, exist_ok=True)
    for p in passes:
        d = os.path.join(replica_dir, p.dir_name)
        os.makedirs(d, exist_ok=True)
        for name, ranks in p.tensors.items():
            os.makedirs(os.path.join(d, name), exist_ok=True)
            for r, t in ranks.items():
                torch.save(t.detach().cpu().clone(), os.path.join(d, name, f"rank{r}.pt"))
        with open(os.path.join(d, f"{p.dir_name}_meta.json"), "w") as f:
            json.dump({"req_ids": list(p.metadata.req_ids), "positions": list(p.metadata.positions),
                       "dp_rank": p.metadata.dp_rank}, f, indent=1)


def _pass_order(name: str):
    m = re.match(r"(prefill_s|decode_b)(\d+)_(\d+)$", name)
    return (int(m.group(3)), name) if m else (1 << 30, name)


def read_replica(replica_dir: str) -> list[CapturedForwardPass]:
    if not os.path.isdir(replica_dir):
        raise FileNotFoundError(f"capture directory not found: {replica_dir}")
    out = []
    names = [d for d in os.listdir(replica_dir) if os.path.isdir(os.path.join(replica_dir, d))
             and (d.startswith("prefill_s") or d.startswith("decode_b"))]
    for name in sorted(names, key=_pass_order):
        d = os.path.join(replica_dir, name)
        meta_path = os.path.join(d, f"{name}_meta.json")
        if not os.path.exists(meta_path):
            raise FileNotFoundError(f"metadata missing for {name}: {meta_path}")
        with open(meta_path) as f:
            m = json.load(f)
        tensors = {}
        for mod in sorted(os.listdir(d)):
            md = os.path.join(d, mod)
            if not os.path.isdir(md):
                continue
            ranks = {}
            for fn in os.listdir(md):
                r = re.fullmatch(r"rank(\d+)\.pt", fn)
                if r:
                    ranks[int(r.group(1))] = torch.load(os.path.join(md, fn), weights_only=True)
            if ranks:
                tensors[mod] = dict(sorted(ranks.items()))
        out.append(CapturedForwardPass(name, ForwardPassMetadata(m["req_ids"], m["positions"], m.get("dp_rank", 0)),
                                       tensors))
    return out


def read(capture_dir: str) -> list[CapturedForwardPass]:
    """Every replica's passes (``dp{N}`` subdirectories), replica by replica."""
    if not os.path.isdir(capture_dir):
        raise FileNotFoundError(f"capture directory not found: {capture_dir}")
    reps = sorted((d for d in os.listdir(capture_dir) if re.fullmatch(r"dp\d+", d)), key=lambda d: int(d[2:]))
    if not reps:
        raise FileNotFoundError(f"no dp<N>/ subdirectories in {capture_dir}")
    out = []
    for d in reps:
        out += read_replica(os.path.join(capture_dir, d))
    return out


def from_capture_steps(step_dir: str, ranks: list[int] | None = None, dp_rank: int = 0) -> list[CapturedForwardPass]:
    """Convert ``TensorCapture`` step files (one file per step and rank) into passes; the
    tensors of the listed tensor-parallel ranks (default: every rank found) are kept per rank."""
    files = {}
    for fn in os.listdir(step_dir):
        m = re.fullmatch(r"step_(\d+)_rank(\d+)\.pt", fn)
        if m:
            files.setdefault(int(m.group(1)), {})[int(m.group(2))] = os.path.join(step_dir, fn)
    out = []
    for n, (step, per_rank) in enumerate(sorted(files.items())):
        use = sorted(per_rank) if ranks is None else [r for r in ranks if r in per_rank]
        if not use:
            continue
        data = {r: torch.load(per_rank[r], weights_only=False) for r in use}
        meta = data[use[0]]["meta"]
        pos = [p for s, k in zip(meta.get("start_pos", []), meta.get("num_tokens", [])) for p in range(s, s + k)]
        kind = meta.get("kind", "prefill")
        size = len(pos) if kind == "prefill" else len(meta.get("req_ids", []))
        name = f"{'prefill_s' if kind == 'prefill' else 'decode_b'}{size}_{n}"
        tensors: dict = {}
        for r in use:
            for mod, t in data[r]["tensors"].items():
                tensors.setdefault(mod, {})[r] = t
        out.append(CapturedForwardPass(name, ForwardPassMetadata(list(meta.get("req_ids", [])), pos, dp_rank), tensors))
    return out


@torch.no_grad()
def capture_hf(model, prompt: list[int], modules: dict[str, str], max_new_tokens: int = 0,
               req_id: str = "hf-0") -> list[CapturedForwardPass]:
    """Module outputs of an HF causal LM: ``modules`` maps HF module names to the names used
    in the captures being compared (e.g. ``{"model.layers.0.mlp": "layers.0.mlp"}``).  The
    prompt runs as one prefill pass; each of ``max_new_tokens`` greedy tokens then runs as a
    one-token decode pass on the HF cache.  Tensors are stored as [tokens, hidden] (rank 0)."""
    mods = dict(model.named_modules())
    missing = [n for n in modules if n not in mods]
    if missing:
        raise KeyError(f"no HF module named {missing[:4]}")
    buf: dict = {}

    def hook(name):
        def fn(_m, _i, out):
            t = out[0] if isinstance(out, (tuple, list)) else out
            buf[name] = t.detach().float().cpu().reshape(-1, t.shape[-1])
        return fn

    handles = [mods[h].register_forward_hook(hook(ours)) for h, ours in modules.items()]
    passes = []
    try:
        ids = torch.tensor([list(prompt)])
        out = model(ids, use_cache=True)
        passes.append(CapturedForwardPass(f"prefill_s{len(prompt)}_0",
                                          ForwardPassMetadata([req_id], list(range(len(prompt)))),
                                          {k: {0: v} for k, v in buf.items()}))
        cache, pos = out.past_key_values, len(prompt)
        for j in range(max_new_tokens):
            buf.clear()
            nxt = out.logits[:, -1].argmax(-1, keepdim=True)
            out = model(nxt, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
            passes.append(CapturedForwardPass(f"decode_b1_{j + 1}", ForwardPassMetadata([req_id], [pos]),
                                              {k: {0: v} for k, v in buf.items()}))
            pos += 1
    finally:
        for h in handles:
            h.remove()
    return passes
