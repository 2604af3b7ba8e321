"""Vision-encoder cache inspection (the reference's ``accuracy/encoder_cache_analysis.py``:
``compare_encoder_caches`` ``:211``, ``compare_encoder_caches_by_index`` ``:262``,
``EncoderCacheMetrics`` ``:42``).

The engine keeps each image's encoder output in its on-device encoder cache: per image token
the merged embedding followed by the deepstack features (``fat`` rows).  ``EncoderSnapshot``
copies every image of a request when it finishes (before the cache blocks are released), keyed
``(request_id, image index)``; ``extract_hf_encoder_outputs`` builds the same ``fat`` rows
from an HF Qwen3-VL vision tower, so the two compare row for row.  Metrics per image: relative
L-inf and L2 over the whole tensor and the mean per-token cosine."""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class EncoderCacheMetrics:
    linf: float          # max|diff| / max|ref|
    l2: float            # ||diff|| / ||ref||
    cos_sim: float       # mean cosine over tokens
    num_tokens: int
    embedding_dim: int


def encoder_metrics(ref: torch.Tensor, actual: torch.Tensor) -> EncoderCacheMetrics:
    r, a = ref.detach().float().cpu(), actual.detach().float().cpu()
    n = min(r.shape[0], a.shape[0])
    r, a = r[:n], a[:n]
    d = a - r
    return EncoderCacheMetrics(float(d.abs().max() / r.abs().max().clamp_min(1e-10)) if n else 0.0,
                               float(d.norm() / r.norm().clamp_min(1e-10)) if n else 0.0,
                               float(torch.nn.functional.cosine_similarity(r, a, dim=-1).mean()) if n else 1.0,
                               n, r.shape[-1])


class EncoderSnapshot:
    """``snapshot.items[(request_id, image index)] = fat rows [tokens, hidden * (1 + deepstack)]``
    for every request that finishes while attached."""

    def __init__(self, engine):
        self.engine = engine
        self.cache = engine.worker.runner.encoder_cache
        if self.cache is None:
            raise ValueError("the engine's model has no vision encoder cache")
        self.items: dict[tuple[str, int], torch.Tensor] = {}
        engine.scheduler.on_finish.insert(0, self._grab)

    def _grab(self, req_id: str) -> None:
        for (rid, it), (_, n) in list(self.cache.items.items()):
            if rid == req_id:
                rows = torch.arange(n, device=self.cache.buf.device)
                self.items[(rid, it)] = self.cache.gather(rid, it, rows).float().cpu()

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
def extract_hf_encoder_outputs(hf_model, images: list[torch.Tensor], vision_config) -> list[torch.Tensor]:
    """Fat rows (merged embedding, then each deepstack feature) per image from an HF Qwen3-VL
    model, with this framework's image preprocessing."""
    from ..engine.llm_engine import torch_image
    from ..models.qwen3_vl import preprocess_image

    outs = []
    for img in images:
        patches, grid = preprocess_image(torch_image(img), vision_config)
        o = hf_model.model.visual(patches, grid_thw=torch.tensor([grid]))
        emb = getattr(o, "pooler_output", None)
        deep = getattr(o, "deepstack_features", None)
        if emb is None:
            emb, deep = o[0], o[1]
        outs.append(torch.cat([emb] + list(deep), dim=-1).float())
    return outs


def compare_encoder_caches(expected: dict, actual: dict, baseline: dict | None = None) -> dict:
    """Per key present on both sides: metrics of ``actual`` against ``baseline`` when given,
    else against ``expected`` (keys are e.g. (request_id, image index))."""
    ref = baseline if baseline is not None else expected
    return {k: encoder_metrics(ref[k], actual[k]) for k in sorted(set(ref) & set(actual), key=str)}


def compare_encoder_caches_by_index(expected: list[torch.Tensor], actual: list[torch.Tensor],
                                    baseline: list[torch.Tensor] | None = None) -> list[EncoderCacheMetrics]:
    """Positional comparison (image i against image i), e.g. HF outputs against a snapshot's
    items in request order."""
    ref = baseline if baseline is not None else expected
    return [encoder_metrics(r, a) for r, a in zip(ref, actual)]


def encoder_report(results) -> str:
    items = results.items() if isinstance(results, dict) else enumerate(results)
    lines = [f"{'image':<24}{'tokens':>8}{'dim':>7}{'linf':>11}{'l2':>11}{'cos':>11}"]
    for k, m in items:
        lines.append(f"{str(k):<24}{m.num_tokens:>8}{m.embedding_dim:>7}{m.linf:>11.3g}{m.l2:>11.3g}{m.cos_sim:>11.6f}")
    return "\n".join(lines)
