"""Qwen3-VL (dense vision-language model).

Semantics of the Trainium plugin's ``model/qwen3_vl`` (``Qwen3VLForConditionalGeneration``
``model_bf16.py:910``, ``Qwen3VLVisionModel`` ``vision_encoder_bf16.py:675``) and HF
``Qwen3VLForConditionalGeneration``:
* vision: a 3-D patch embedding (temporal 2 x 16 x 16 -> linear), a learned position
  table bilinearly interpolated to the image grid, 2-D rotary embeddings (row / column
  halves), LayerNorm ViT blocks with GELU MLPs, a 2x2 spatial merger to the text width
  and "deepstack" mergers whose outputs are added to the text hidden states of the
  first decoder layers at the image positions;
* text: the Qwen3 dense decoder (QK-norm) with interleaved multimodal RoPE (positions
  [t, h, w] per token; text tokens use t = h = w; after the prompt, positions continue
  at ``max + 1`` via a per-request delta, ``utils/mrope.py:79`` of the reference).
Vision attention is non-causal within each image frame (varlen kernel, head dim 72
padded to 80 in the kernel).  The vision tower is tensor-parallel over the vision TP
group (heads and MLP sharded, row-parallel outputs all-reduced).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..nn.linear import ParallelLMHead, RMSNorm, VocabParallelEmbedding, shard_range
from ..ops import reference as ref
from ..parallel.state import GroupCoordinator, ParallelState
from .base import KVSpec, LayerSpec
from .llama import DenseDecoderLayer, LlamaConfig, LlamaForCausalLM


@dataclass
class VisionConfig:
    depth: int = 27
    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 16
    spatial_merge_size: int = 2
    temporal_patch_size: int = 2
    out_hidden_size: int = 5120
    num_position_embeddings: int = 2304
    deepstack_visual_indexes: tuple = (8, 16, 24)


@dataclass
class Qwen3VLConfig:
    text: LlamaConfig
    vision: VisionConfig
    mrope_section: list = field(default_factory=lambda: [24, 20, 20])
    image_token_id: int = 151655
    vision_start_token_id: int = 151652
    vision_end_token_id: int = 151653
    quantization: str = "bf16"

    @property
    def vocab_size(self) -> int:
        return self.text.vocab_size

    @property
    def hidden_size(self) -> int:
        return self.text.hidden_size

    @classmethod
    def from_hf(cls, d: dict, quantization: str | None = None) -> "Qwen3VLConfig":
        td = dict(d.get("text_config", d))
        td.setdefault("model_type", "qwen3")
        td["model_type"] = "qwen3"
        rope = td.get("rope_parameters") or td.get("rope_scaling") or {}
        td["rope_scaling"] = None
        td["rope_parameters"] = None
        td.setdefault("rope_theta", rope.get("rope_theta", 5000000.0))
        text = LlamaConfig.from_hf(td, quantization or "bf16")
        text.qk_norm = True
        text.tie_word_embeddings = d.get("tie_word_embeddings", td.get("tie_word_embeddings", False))
        vd = d.get("vision_config", {})
        vision = VisionConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in vd.items()
                                 if k in VisionConfig.__dataclass_fields__})
        return cls(text=text, vision=vision, mrope_section=list(rope.get("mrope_section", [24, 20, 20])),
                   image_token_id=d.get("image_token_id", 151655),
                   vision_start_token_id=d.get("vision_start_token_id", 151652),
                   vision_end_token_id=d.get("vision_end_token_id", 151653))


def _p(shape, dtype, device):
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


class _LN(nn.Module):
    def __init__(self, n, device, eps=1e-6):
        super().__init__()
        self.weight = _p((n,), torch.float32, device)
        self.bias = _p((n,), torch.float32, device)
        self.eps = eps

    def forward(self, x):
        return F.layer_norm(x.float(), (x.shape[-1],), self.weight, self.bias, self.eps).to(x.dtype)


class VisionBlock(nn.Module):
    def __init__(self, vc: VisionConfig, tp: GroupCoordinator, dtype, device):
        super().__init__()
        self.tp = tp
        H = vc.hidden_size
        self.nh = vc.num_heads // tp.world_size
        self.d = H // vc.num_heads
        self.I_local = vc.intermediate_size // tp.world_size
        self.norm1 = _LN(H, device)
        self.norm2 = _LN(H, device)
        self.qkv_w = _p((3 * self.nh * self.d, H), dtype, device)
        self.qkv_b = _p((3 * self.nh * self.d,), dtype, device)
        self.proj_w = _p((H, self.nh * self.d), dtype, device)
        self.proj_b = _p((H,), dtype, device)
        self.fc1_w = _p((self.I_local, H), dtype, device)
        self.fc1_b = _p((self.I_local,), dtype, device)
        self.fc2_w = _p((H, self.I_local), dtype, device)
        self.fc2_b = _p((H,), dtype, device)

    def forward(self, x, cu_seqlens, cos, sin, max_len):
        T = x.shape[0]
        h = self.norm1(x)
        qkv = ops.linear(h, self.qkv_w, self.qkv_b).view(T, 3, self.nh, self.d)
        q = ref.apply_rope(qkv[:, 0], cos, sin).contiguous()
        k = ref.apply_rope(qkv[:, 1], cos, sin).contiguous()
        v = qkv[:, 2].contiguous()
        o = ops.varlen_attention(q, k, v, cu_seqlens, 1.0 / math.sqrt(self.d), causal=False, max_seqlen=max_len)
        a = ops.linear(o.reshape(T, -1), self.proj_w)
        a = self.tp.all_reduce(a) + self.proj_b
        x = x + a
        m = F.gelu(ops.linear(self.norm2(x), self.fc1_w, self.fc1_b).float(), approximate="tanh").to(x.dtype)
        m = self.tp.all_reduce(ops.linear(m, self.fc2_w)) + self.fc2_b
        return x + m


class PatchMerger(nn.Module):
    def __init__(self, vc: VisionConfig, postshuffle: bool, dtype, device):
        super().__init__()
        self.m = vc.spatial_merge_size ** 2
        self.hs = vc.hidden_size * self.m
        self.post = postshuffle
        self.norm = _LN(self.hs if postshuffle else vc.hidden_size, device)
        self.fc1_w = _p((self.hs, self.hs), dtype, device)
        self.fc1_b = _p((self.hs,), dtype, device)
        self.fc2_w = _p((vc.out_hidden_size, self.hs), dtype, device)
        self.fc2_b = _p((vc.out_hidden_size,), dtype, device)

    def forward(self, x):
        x = self.norm(x.view(-1, self.hs)) if self.post else self.norm(x).view(-1, self.hs)
        return ops.linear(F.gelu(ops.linear(x, self.fc1_w, self.fc1_b).float()).to(x.dtype), self.fc2_w, self.fc2_b)


class Qwen3VLVisionModel(nn.Module):
    def __init__(self, vc: VisionConfig, tp: GroupCoordinator, dtype, device):
        super().__init__()
        self.vc = vc
        H = vc.hidden_size
        self.patch_dim = vc.in_channels * vc.temporal_patch_size * vc.patch_size ** 2
        self.patch_w = _p((H, self.patch_dim), dtype, device)
        self.patch_b = _p((H,), dtype, device)
        self.pos_embed = _p((vc.num_position_embeddings, H), dtype, device)
        self.side = int(vc.num_position_embeddings ** 0.5)
        self.blocks = nn.ModuleList([VisionBlock(vc, tp, dtype, device) for _ in range(vc.depth)])
        self.merger = PatchMerger(vc, False, dtype, device)
        self.deepstack = nn.ModuleList([PatchMerger(vc, True, dtype, device) for _ in vc.deepstack_visual_indexes])
        hd = H // vc.num_heads
        self.register_buffer("inv_freq", 1.0 / (10000.0 ** (torch.arange(0, hd // 2, 2, dtype=torch.float32) /
                                                             (hd // 2))), persistent=False)

    def _pos_embed(self, grids):
        """Bilinear interpolation of the learned position table to each (h, w) grid,
        reordered into 2x2 merge blocks."""
        outs = []
        dev = self.pos_embed.device
        m = self.vc.spatial_merge_size
        n = self.side
        for t, h, w in grids:
            hi = torch.linspace(0, n - 1, h, device=dev)
            wi = torch.linspace(0, n - 1, w, device=dev)
            h0, w0 = hi.long(), wi.long()
            h1, w1 = (h0 + 1).clamp(max=n - 1), (w0 + 1).clamp(max=n - 1)
            dh, dw = (hi - h0)[:, None], (wi - w0)[None, :]
            tab = self.pos_embed.float()
            e = (tab[(h0[:, None] * n + w0[None, :]).flatten()] * ((1 - dh) * (1 - dw)).flatten()[:, None]
                 + tab[(h0[:, None] * n + w1[None, :]).flatten()] * ((1 - dh) * dw).flatten()[:, None]
                 + tab[(h1[:, None] * n + w0[None, :]).flatten()] * (dh * (1 - dw)).flatten()[:, None]
                 + tab[(h1[:, None] * n + w1[None, :]).flatten()] * (dh * dw).flatten()[:, None])
            e = e.to(self.pos_embed.dtype).repeat(t, 1)
            e = e.view(t, h // m, m, w // m, m, -1).permute(0, 1, 3, 2, 4, 5).reshape(t * h * w, -1)
            outs.append(e)
        return torch.cat(outs)

    def _rot(self, grids):
        m = self.vc.spatial_merge_size
        dev = self.inv_freq.device
        rows, cols = [], []
        for t, h, w in grids:
            br = torch.arange(h // m, device=dev)[:, None, None, None] * m + torch.arange(m, device=dev)[None, None, :,
                                                                                                        None]
            bc = torch.arange(w // m, device=dev)[None, :, None, None] * m + torch.arange(m, device=dev)[None, None,
                                                                                                        None, :]
            r = br.expand(h // m, w // m, m, m).reshape(-1)
            c = bc.expand(h // m, w // m, m, m).reshape(-1)
            rows.append(r.repeat(t))
            cols.append(c.repeat(t))
        r, c = torch.cat(rows), torch.cat(cols)
        fr = r[:, None].float() * self.inv_freq[None]
        fc = c[:, None].float() * self.inv_freq[None]
        rot = torch.cat([fr, fc], dim=-1)  # [T, head_dim/2]
        return rot.cos(), rot.sin()

    def forward(self, patches: torch.Tensor, grids: list[tuple[int, int, int]]):
        x = ops.linear(patches.to(self.patch_w.dtype), self.patch_w, self.patch_b)
        x = x + self._pos_embed(grids)
        cos, sin = self._rot(grids)
        lens = []
        for t, h, w in grids:
            lens += [h * w] * t
        cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=x.device)
        deep = []
        for i, blk in enumerate(self.blocks):
            x = blk(x, cu, cos, sin, max(lens))
            if i in self.vc.deepstack_visual_indexes:
                deep.append(self.deepstack[list(self.vc.deepstack_visual_indexes).index(i)](x))
        return self.merger(x), deep


def preprocess_image(img: torch.Tensor, vc: VisionConfig, max_pixels: int = 1 << 22
                     ) -> tuple[torch.Tensor, tuple[int, int, int]]:
    """[C, H, W] pixels (0..255) -> (patches [t*h*w, C*2*p*p], grid (t, h, w)).  The image is
    resized to multiples of patch*merge (at most ``max_pixels``), normalised with mean/std
    0.5, duplicated to the temporal patch size, and patchified in merge-block order."""
    p, m, tp = vc.patch_size, vc.spatial_merge_size, vc.temporal_patch_size
    C, Hh, Ww = img.shape
    f = p * m
    scale = min(1.0, math.sqrt(max_pixels / max(1, Hh * Ww)))
    nh, nw = max(f, round(Hh * scale / f) * f), max(f, round(Ww * scale / f) * f)
    x = F.interpolate(img[None].float(), size=(nh, nw), mode="bilinear", align_corners=False)[0]
    x = (x / 255.0 - 0.5) / 0.5
    x = x[None].expand(tp, C, nh, nw)
    gh, gw = nh // p, nw // p
    x = x.reshape(1, tp, C, gh // m, m, p, gw // m, m, p)
    x = x.permute(0, 3, 6, 4, 7, 2, 1, 5, 8)  # t, bh, bw, mh, mw, C, tp, p, p
    return x.reshape(gh * gw, C * tp * p * p).contiguous(), (1, gh, gw)


class Qwen3VLForConditionalGeneration(LlamaForCausalLM):
    """Qwen3 text decoder + vision tower.  Multimodal inputs arrive through
    ``meta.extras``: ``mm_embeds`` [n, H] and ``mm_index`` [n] (token rows to replace),
    ``deepstack`` (list of [n, H]), ``mrope_positions`` [3, T] (None: text-only step)."""

    config_class = Qwen3VLConfig

    def __init__(self, cfg: Qwen3VLConfig, ps: ParallelState, dtype=torch.bfloat16, device="cpu", kv_dtype=None):
        super().__init__(cfg.text, ps, dtype, device, kv_dtype)
        self.vl_cfg = cfg
        self.visual = Qwen3VLVisionModel(cfg.vision, ps.vision_tp, dtype, device)
        self.vision_dp = ps.vision_dp
        self.vision_block_size = 2048  # patches per packed encoder call (vision_attention_block_size)
        self.inv = cfg.text.inv_freq()[0]
        self.encoder_calls = 0

    # ------------------------------------------------------------ multimodal helpers
    def embed_multimodal(self, pixels: torch.Tensor) -> dict:
        """One image [C, H, W] -> embeddings for its placeholder tokens, deepstack
        features and the grid (``embed_multimodal``, reference ``model_bf16.py:1051``)."""
        patches, grid = preprocess_image(pixels, self.vl_cfg.vision)
        dev = self.visual.patch_w.device
        emb, deep = self.visual(patches.to(dev), [grid])
        return {"embeds": emb, "deepstack": deep, "grid": grid}

    def embed_images(self, pixels: list[torch.Tensor]) -> list[torch.Tensor]:
        """Every image of a step at once (``vision_encoder_bf16.py:806-862`` of the reference:
        block packing, DP scatter, DP gather).  The images' patch sequences are packed first-fit
        decreasing into blocks of at most ``vision_block_size`` patches; one vision-tower call
        per block runs its images as one varlen batch.  With vision data parallelism the blocks
        are dealt to the ranks of the ``vision_dp`` group (largest first, to the least-loaded
        rank), each rank encodes its blocks with its vision-TP peers, and one all-gather of the
        padded results gives every rank every image.  Returns per image the "fat" rows
        [tokens, hidden x (1 + deepstack levels)]."""
        from ..utils.vision_utils import pack_sequences

        vc = self.vl_cfg.vision
        pre = [preprocess_image(px, vc) for px in pixels]
        lens = [p.shape[0] for p, _ in pre]
        m2 = vc.spatial_merge_size ** 2
        blocks = pack_sequences(lens, self.vision_block_size)
        g = self.vision_dp
        dp = g.world_size if g is not None else 1
        me = g.rank_in_group if g is not None else 0
        load = [0] * dp
        owner = []
        for blk in blocks:  # pack_sequences returns the blocks largest first
            r = min(range(dp), key=lambda i: (load[i], i))
            owner.append(r)
            load[r] += sum(lens[i] for i in blk)
        dev = self.visual.patch_w.device
        out: list[torch.Tensor | None] = [None] * len(pixels)
        mine: list[int] = []
        for blk, r in zip(blocks, owner):
            if r != me:
                continue
            patches = torch.cat([pre[i][0] for i in blk]).to(dev)
            emb, deep = self.visual(patches, [pre[i][1] for i in blk])
            self.encoder_calls += 1
            fat = torch.cat([emb] + list(deep), dim=-1)
            off = 0
            for i in blk:
                n = lens[i] // m2
                out[i] = fat[off:off + n]
                off += n
                mine.append(i)
        if dp > 1:
            width = (1 + len(vc.deepstack_visual_indexes)) * vc.out_hidden_size
            per_rank = [[i for blk, r in zip(blocks, owner) if r == q for i in blk] for q in range(dp)]
            rows = [sum(lens[i] // m2 for i in ids) for ids in per_rank]
            buf = torch.zeros(max(rows), width, dtype=self.visual.patch_w.dtype, device=dev)
            if mine:
                local = torch.cat([out[i] for i in mine])
                buf[:local.shape[0]] = local
            allb = g.all_gather(buf[None], dim=0)  # [dp, max_rows, width]
            for q, ids in enumerate(per_rank):
                off = 0
                for i in ids:
                    n = lens[i] // m2
                    out[i] = allb[q, off:off + n]
                    off += n
        return out  # type: ignore[return-value]

    # ------------------------------------------------ capabilities (models/interfaces.py)
    @classmethod
    def get_vision_token_merge_factor(cls, hf_config) -> int:
        """Raw patches per embedding token: spatial_merge_size squared."""
        from .interfaces import _vision_cfg

        m = int(_vision_cfg(hf_config).get("spatial_merge_size", 2))
        return m * m

    @classmethod
    def get_max_pixels_token_count(cls, hf_config, max_pixels: int) -> int:
        """Raw (pre-merge) patches of an image of ``max_pixels`` pixels: one patch per
        patch_size x patch_size pixels."""
        from .interfaces import _vision_cfg

        p = int(_vision_cfg(hf_config).get("patch_size", 16))
        return max(1, int(max_pixels) // (p * p))

    def build_vision_synthetic_inputs(self, bucket: int, vision_neuron_config, device) -> dict:
        """Zero patches of a one-frame grid (merge x bucket*merge patches) that the encoder
        turns into exactly ``bucket`` embedding tokens."""
        vc = self.vl_cfg.vision
        m, p = vc.spatial_merge_size, vc.patch_size
        grid = (1, m, int(bucket) * m)
        dim = vc.in_channels * vc.temporal_patch_size * p * p
        return {"patches": torch.zeros(m * m * int(bucket), dim, dtype=torch.float32, device=device),
                "grids": [grid]}

    def get_mrope_input_positions(self, token_ids: list[int], grids: list) -> tuple[torch.Tensor, int]:
        return self.mrope_positions(token_ids, grids)

    def num_image_tokens(self, grid) -> int:
        t, h, w = grid
        m = self.vl_cfg.vision.spatial_merge_size
        return t * (h // m) * (w // m)

    def mrope_positions(self, token_ids: list[int], grids: list[tuple[int, int, int]]) -> tuple[torch.Tensor, int]:
        """3-D positions of a prompt whose image placeholders are already expanded, and the
        delta that continues positions after it (``get_rope_index`` semantics)."""
        m = self.vl_cfg.vision.spatial_merge_size
        img = self.vl_cfg.image_token_id
        pos = []
        cur = 0
        i = 0
        g = iter(grids)
        n = len(token_ids)
        while i < n:
            if token_ids[i] == img:
                t, h, w = next(g)
                lh, lw = h // m, w // m
                for tt in range(t):
                    for a in range(lh):
                        for b in range(lw):
                            pos.append((cur, cur + a, cur + b))
                i += t * lh * lw
                cur += max(lh, lw)
            else:
                pos.append((cur, cur, cur))
                cur += 1
                i += 1
        P = torch.tensor(pos, dtype=torch.long).t().contiguous()
        return P, int(P.max().item()) + 1 - n

    # ----------------------------------------------------------------- forward
    def forward(self, input_ids, positions, meta, kv_caches, inputs_embeds=None):
        ex = meta.extras or {}
        h = self.embed_tokens(input_ids)
        mm_idx = ex.get("mm_index")
        if mm_idx is not None and mm_idx.numel():
            h = h.clone()
            h[mm_idx] = ex["mm_embeds"].to(h.dtype)
        p3 = ex.get("mrope_positions")
        cos_sin = self.cos_sin
        pos = positions
        if p3 is not None:
            cos, sin = ref.mrope_cos_sin(p3, self.inv.to(h.device), self.vl_cfg.mrope_section, interleaved=True)
            cos_sin = torch.cat([cos, sin], dim=-1).contiguous()
            pos = torch.arange(h.shape[0], device=h.device)
        deep = ex.get("deepstack") or []
        residual = None
        prev_bias = None
        for i, layer in enumerate(self.layers):
            h, residual = layer(pos, h, residual, meta, kv_caches[i], cos_sin, prev_bias)
            prev_bias = layer.mlp.down.bias
            if i < len(deep) and mm_idx is not None and mm_idx.numel():
                # deepstack: the hidden state after layer i is reduce(h) + residual, so adding
                # the visual features to the (replicated) residual stream adds them to it
                residual = residual.clone()
                residual[mm_idx] += deep[i].to(residual.dtype)
        h, _ = self.ps.tp.all_reduce_add_rmsnorm(h, residual, self.norm.weight, self.cfg.rms_norm_eps, prev_bias)
        return h

    # ----------------------------------------------------------------- loading
    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        rest = []
        loaded = set()
        for name, t in weights:
            if name.startswith("model.visual."):
                self._load_visual(name[len("model.visual."):], t)
                loaded.add(name)
            elif name.startswith("model.language_model."):
                rest.append(("model." + name[len("model.language_model."):], t))
            else:
                rest.append((name, t))
        return loaded | super().load_weights(rest)

    def _load_visual(self, n: str, t: torch.Tensor) -> None:
        v = self.visual
        if n == "patch_embed.proj.weight":
            v.patch_w.data.copy_(t.reshape(t.shape[0], -1).to(v.patch_w.dtype))
        elif n == "patch_embed.proj.bias":
            v.patch_b.data.copy_(t.to(v.patch_b.dtype))
        elif n == "pos_embed.weight":
            v.pos_embed.data.copy_(t.to(v.pos_embed.dtype))
        elif n.startswith("blocks."):
            parts = n.split(".")
            blk = v.blocks[int(parts[1])]
            key = ".".join(parts[2:])
            tp, r = blk.tp.world_size, blk.tp.rank_in_group
            if key in ("norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias"):
                getattr(getattr(blk, key.split(".")[0]), key.split(".")[1]).data.copy_(t.float())
            elif key in ("attn.qkv.weight", "attn.qkv.bias"):
                H = blk.qkv_w.shape[1]
                full = t.view(3, -1, *t.shape[1:])  # [3, H(heads*d), ...]
                s, e = shard_range(full.shape[1], r, tp)
                dst = blk.qkv_w if key.endswith("weight") else blk.qkv_b
                dst.data.copy_(full[:, s:e].reshape(dst.shape).to(dst.dtype))
                del H
            elif key == "attn.proj.weight":
                s, e = shard_range(t.shape[1], r, tp)
                blk.proj_w.data.copy_(t[:, s:e].to(blk.proj_w.dtype))
            elif key == "attn.proj.bias":
                blk.proj_b.data.copy_(t.to(blk.proj_b.dtype))
            elif key in ("mlp.linear_fc1.weight", "mlp.linear_fc1.bias"):
                s, e = shard_range(t.shape[0], r, tp)
                dst = blk.fc1_w if key.endswith("weight") else blk.fc1_b
                dst.data.copy_(t[s:e].to(dst.dtype))
            elif key == "mlp.linear_fc2.weight":
                s, e = shard_range(t.shape[1], r, tp)
                blk.fc2_w.data.copy_(t[:, s:e].to(blk.fc2_w.dtype))
            elif key == "mlp.linear_fc2.bias":
                blk.fc2_b.data.copy_(t.to(blk.fc2_b.dtype))
        else:
            parts = n.split(".")
            if parts[0] == "merger":
                mod = v.merger
                key = ".".join(parts[1:])
            elif parts[0] == "deepstack_merger_list":
                mod = v.deepstack[int(parts[1])]
                key = ".".join(parts[2:])
            else:
                return
            if key.startswith("norm."):
                getattr(mod.norm, key.split(".")[1]).data.copy_(t.float())
            else:
                attr = {"linear_fc1.weight": "fc1_w", "linear_fc1.bias": "fc1_b", "linear_fc2.weight": "fc2_w",
                        "linear_fc2.bias": "fc2_b"}[key]
                getattr(mod, attr).data.copy_(t.to(getattr(mod, attr).dtype))
