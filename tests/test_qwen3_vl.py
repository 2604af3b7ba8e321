"""Qwen3-VL: vision tower and full multimodal forward vs HF transformers (fp32, CPU)."""

import pytest
import torch

HF_KW = dict(
    text_config=dict(vocab_size=1024, hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                     rope_parameters={"rope_type": "default", "rope_theta": 1e6, "mrope_section": [4, 6, 6],
                                      "mrope_interleaved": True}, tie_word_embeddings=False),
    vision_config=dict(depth=3, hidden_size=64, intermediate_size=128, num_heads=4, patch_size=16,
                       spatial_merge_size=2, temporal_patch_size=2, out_hidden_size=128, num_position_embeddings=64,
                       deepstack_visual_indexes=[0, 1]),
    image_token_id=1000, vision_start_token_id=1001, vision_end_token_id=1002)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    from vllm_neuron_b200.models.qwen3_vl import Qwen3VLConfig as Cfg
    from vllm_neuron_b200.models.qwen3_vl import Qwen3VLForConditionalGeneration as Ours
    from vllm_neuron_b200.parallel.state import initialize_parallel_state

    torch.manual_seed(0)
    hcfg = Qwen3VLConfig(**HF_KW)
    hcfg._attn_implementation = "eager"
    hcfg.text_config._attn_implementation = "eager"
    hcfg.vision_config._attn_implementation = "eager"
    hf = Qwen3VLForConditionalGeneration(hcfg).eval().float()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if n.endswith("bias") or "norm" in n:
                p.add_(0.05 * torch.randn_like(p))
    d = hcfg.to_dict()
    d["architectures"] = ["Qwen3VLForConditionalGeneration"]
    ps = initialize_parallel_state()
    ours = Ours(Cfg.from_hf(d), ps, dtype=torch.float32, device="cpu")
    ours.load_weights(hf.state_dict().items())
    return hf, ours


def test_vision_tower_matches_hf(models):
    from vllm_neuron_b200.models.qwen3_vl import preprocess_image

    hf, ours = models
    img = torch.rand(3, 100, 130) * 255
    patches, grid = preprocess_image(img, ours.vl_cfg.vision)
    with torch.no_grad():
        out = hf.model.visual(patches, grid_thw=torch.tensor([grid]))
        emb, deep = ours.visual(patches, [grid])
    assert torch.allclose(emb, out.pooler_output, atol=1e-4, rtol=1e-4)
    for a, b in zip(deep, out.deepstack_features):
        assert torch.allclose(a, b, atol=1e-4, rtol=1e-4)


def test_multimodal_logits_match_hf(models):
    from vllm_neuron_b200.models.qwen3_vl import preprocess_image
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    hf, ours = models
    img = torch.rand(3, 64, 96) * 255
    patches, grid = preprocess_image(img, ours.vl_cfg.vision)
    n_img = ours.num_image_tokens(grid)
    ids = [5, 6, 1001] + [1000] * n_img + [1002, 7, 8, 9]
    T = len(ids)
    with torch.no_grad():
        want = hf(input_ids=torch.tensor([ids]), pixel_values=patches, image_grid_thw=torch.tensor([grid]),
                  mm_token_type_ids=torch.tensor([[1 if t == 1000 else 0 for t in ids]])).logits[0]
        mm = ours.embed_multimodal(img)
        p3, delta = ours.mrope_positions(ids, [grid])
        bs = 16
        nb = T // bs + 2
        kv = [(torch.zeros(nb, 2, bs, 32), torch.zeros(nb, 2, bs, 32)) for _ in ours.layers]
        mm_idx = torch.tensor([i for i, t in enumerate(ids) if t == 1000])
        meta = AttentionMetadata(T, 1, False, torch.tensor([0, T], dtype=torch.int32),
                                 torch.tensor([T], dtype=torch.int32),
                                 torch.arange(1, nb, dtype=torch.int32)[None], torch.arange(T) + bs, None, T, T,
                                 extras={"mm_embeds": mm["embeds"], "mm_index": mm_idx, "deepstack": mm["deepstack"],
                                         "mrope_positions": p3})
        h = ours(torch.tensor(ids), torch.arange(T), meta, kv)
        got = ours.compute_logits(h)
    assert delta == int(p3.max()) + 1 - T
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-3), (got - want).abs().max()


def test_vl_generation_through_engine():
    """Image + text prompt through LLM.generate (CPU): placeholder expansion, encoder
    cache, segmented prefill across the image, decode with the M-RoPE position delta.
    Greedy tokens must match a single-segment prefill of the same prompt."""
    from vllm_neuron_b200 import LLM, SamplingParams

    cfg = dict(HF_KW)
    cfg["architectures"] = ["Qwen3VLForConditionalGeneration"]
    img = torch.rand(3, 128, 160) * 255  # grid 8 x 10 patches: 20 merged tokens at prompt rows 3..22
    prompt = [5, 6, 1001, 1000, 1002, 7, 8, 9]
    outs = []
    for chunk in (16, 256):  # 16: the image tokens span two prefill segments
        llm = LLM(hf_config=cfg, load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=2,
                  max_num_batched_tokens=chunk, block_size=16, device="cpu", seed=1)
        o = llm.generate([{"prompt_token_ids": prompt, "multi_modal_data": {"image": img}}],
                         SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
        outs.append(o[0].outputs[0].token_ids)
        assert llm.engine.worker.runner.encoder_cache.num_free == llm.engine.worker.runner.encoder_cache.buf.shape[0]
        llm.shutdown()
    assert outs[0] == outs[1] and len(outs[0]) == 6


def test_vl_oversized_image_refused_at_request_time():
    """An image with more vision tokens than the configured maximum (largest
    num_vision_tokens_buckets entry) is refused by add_request with a ValueError before any
    scheduling; a smaller image on the same engine still runs and frees its cache blocks."""
    import pytest

    from vllm_neuron_b200 import LLM, SamplingParams

    cfg = dict(HF_KW)
    cfg["architectures"] = ["Qwen3VLForConditionalGeneration"]
    llm = LLM(hf_config=cfg, load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=2,
              max_num_batched_tokens=256, block_size=16, device="cpu", seed=1,
              additional_config={"vision_neuron_config": {"num_vision_tokens_buckets": [4]}})
    assert llm.engine.max_embeds_per_image() == 4
    prompt = [5, 6, 1001, 1000, 1002, 7, 8, 9]
    big = torch.rand(3, 64, 96) * 255  # grid 4 x 6 patches: 6 merged tokens
    with pytest.raises(ValueError, match="exceeds the maximum"):
        llm.generate([{"prompt_token_ids": prompt, "multi_modal_data": {"image": big}}],
                     SamplingParams(temperature=0, max_tokens=2))
    assert not llm.engine.has_unfinished_requests()
    small = torch.rand(3, 64, 64) * 255  # grid 4 x 4 patches: 4 merged tokens
    o = llm.generate([{"prompt_token_ids": prompt, "multi_modal_data": {"image": small}}],
                     SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    assert len(o[0].outputs[0].token_ids) == 2
    llm.shutdown()


def test_encoder_cache_snapshot_matches_hf(models, tmp_path):
    """The engine's cached vision-encoder rows of each image (embedding + deepstack features)
    equal HF's vision tower outputs for the same preprocessing."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.encoder_cache_analysis import (EncoderSnapshot, compare_encoder_caches_by_index,
                                                                  encoder_report, extract_hf_encoder_outputs)

    hf, ours = models
    cfg = dict(HF_KW)
    cfg["architectures"] = ["Qwen3VLForConditionalGeneration"]
    llm = LLM(hf_config=cfg, load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=2,
              max_num_batched_tokens=256, block_size=16, device="cpu", seed=1)
    try:
        model = llm.engine.worker.model
        model.load_state_dict(ours.state_dict(), strict=False)
        imgs = [torch.rand(3, 64, 96) * 255, torch.rand(3, 96, 64) * 255]
        prompt = [5, 1001, 1000, 1002, 1001, 1000, 1002, 7]
        with EncoderSnapshot(llm.engine) as snap:
            o = llm.generate([{"prompt_token_ids": prompt, "multi_modal_data": {"image": imgs}}],
                             SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
        rid = o[0].request_id
        got = [snap.items[(rid, 0)], snap.items[(rid, 1)]]
        want = extract_hf_encoder_outputs(hf, imgs, ours.vl_cfg.vision)
        res = compare_encoder_caches_by_index(want, got)
        assert all(m.linf < 1e-4 and m.cos_sim > 0.99999 for m in res), encoder_report(res)
        assert [m.num_tokens for m in res] == [6, 6]
    finally:
        llm.shutdown()


def test_vl_interfaces_and_vision_warmup():
    """Qwen3-VL declares the optional capabilities (spatial merge, pixel budget, M-RoPE,
    vision warm-up); with num_vision_tokens_buckets set, start-up runs the encoder once per
    bucket on synthetic inputs that produce exactly that many tokens."""
    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.models.interfaces import (SupportsMaxPixels, SupportsMRoPE, SupportsSpatialMerge,
                                                    SupportsVisionWarmup)
    from vllm_neuron_b200.models.qwen3_vl import Qwen3VLForConditionalGeneration as VL

    cfg = dict(HF_KW)
    cfg["architectures"] = ["Qwen3VLForConditionalGeneration"]
    assert VL.get_vision_token_merge_factor(cfg) == 4
    assert VL.get_max_pixels_token_count(cfg, 64 * 96) == 24
    llm = LLM(hf_config=cfg, load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=2,
              max_num_batched_tokens=256, block_size=16, device="cpu", seed=1,
              additional_config={"vision_neuron_config": {"num_vision_tokens_buckets": [4, 8]}})
    try:
        model = llm.engine.worker.model
        for proto in (SupportsVisionWarmup, SupportsSpatialMerge, SupportsMaxPixels, SupportsMRoPE):
            assert isinstance(model, proto)
        assert llm.engine.worker.vision_warmups == 2
        inp = model.build_vision_synthetic_inputs(8, None, torch.device("cpu"))
        with torch.no_grad():
            emb, deep = model.visual(inp["patches"], inp["grids"])
        assert emb.shape[0] == 8 and len(deep) == 2
        ids = [5, 1000, 1000, 1000, 1000, 7]
        p, delta = model.get_mrope_input_positions(ids, [(1, 4, 4)])
        assert p.shape == (3, 6) and delta == int(p.max()) + 1 - 6
    finally:
        llm.shutdown()


def test_embed_images_block_packing_matches_single_image_calls(models):
    """Several images encoded together (first-fit-decreasing blocks of at most
    vision_block_size patches, one varlen vision-tower call per block) give each image the
    same rows as encoding it alone."""
    hf, ours = models
    g = torch.Generator().manual_seed(3)
    imgs = [torch.rand(3, h, w, generator=g) * 255 for h, w in ((64, 96), (128, 160), (64, 64), (96, 64))]
    want = []
    with torch.no_grad():
        for im in imgs:
            mm = ours.embed_multimodal(im)
            want.append(torch.cat([mm["embeds"]] + list(mm["deepstack"]), dim=-1))
        old = ours.vision_block_size
        ours.vision_block_size = 96  # patches: 24, 80, 16, 24 -> blocks [80, 16], [24, 24]
        try:
            n0 = ours.encoder_calls
            got = ours.embed_images(imgs)
            calls = ours.encoder_calls - n0
        finally:
            ours.vision_block_size = old
    assert calls == 2
    for a, b in zip(got, want):
        assert a.shape == b.shape and torch.allclose(a, b, atol=1e-4, rtol=1e-4)


def test_vision_data_parallel_generation_matches_single_rank(models, tmp_path):
    """Vision DP = 2 over gloo (vision TP 1, text TP 2): each rank encodes its share of the
    packed blocks and one all-gather gives both ranks every image; greedy tokens of a prompt
    with three images equal the single-rank engine's."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    hf, ours = models
    cfg = hf.config.to_dict()
    cfg["architectures"] = ["Qwen3VLForConditionalGeneration"]
    path = str(tmp_path / "vl")
    save_state_dict({k: v.detach().clone().contiguous() for k, v in hf.state_dict().items()}, path, cfg)
    g = torch.Generator().manual_seed(5)
    imgs = [torch.rand(3, h, w, generator=g) * 255 for h, w in ((64, 96), (96, 64), (64, 64))]
    prompt = [5, 1001, 1000, 1002, 6, 1001, 1000, 1002, 1001, 1000, 1002, 7]
    outs = []
    for extra in ({}, {"tensor_parallel_size": 2,
                       "additional_config": {"vision_neuron_config": {"tp_size": 1, "dp_size": 2,
                                                                      "vision_attention_block_size": 32}}}):
        llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=2, max_num_batched_tokens=256,
                  block_size=16, device="cpu", **extra)
        try:
            o = llm.generate([{"prompt_token_ids": prompt, "multi_modal_data": {"image": imgs}}],
                             SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
            outs.append(list(o[0].outputs[0].token_ids))
        finally:
            llm.shutdown()
    assert outs[0] == outs[1] and len(outs[0]) == 6
