"""Tiny model configurations used across tests (config 1 of the benchmark plan)."""

TINY_GPT_OSS = {
    "architectures": ["GptOssForCausalLM"], "model_type": "gpt_oss", "vocab_size": 4096, "hidden_size": 256,
    "num_hidden_layers": 2, "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 32,
    "intermediate_size": 256, "num_local_experts": 8, "num_experts_per_tok": 2, "sliding_window": 128,
    "layer_types": ["sliding_attention", "full_attention"], "rope_theta": 150000.0, "rms_norm_eps": 1e-5,
    "swiglu_limit": 7.0, "attention_bias": True, "max_position_embeddings": 4096, "initializer_range": 0.02,
    "tie_word_embeddings": False, "hidden_act": "silu", "pad_token_id": None, "eos_token_id": None,
    "bos_token_id": None, "rope_scaling": None, "router_aux_loss_coef": 0.0, "output_router_logits": False,
}


def workload(n=16, lo=32, hi=128, vocab=4096, seed=0):
    import torch

    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        L = int(torch.randint(lo, hi + 1, (1,), generator=g))
        out.append(torch.randint(0, vocab, (L,), generator=g).tolist())
    return out


def hf_torch_path(model) -> None:
    """Make an HF Qwen3-Next model use its PyTorch gated-DeltaNet path (no Triton kernels
    from optional packages), so it runs on the CPU as the fp32 oracle."""
    import torch
    from transformers.models.qwen3_next import modeling_qwen3_next as mq

    for m in model.modules():
        if isinstance(m, mq.Qwen3NextGatedDeltaNet):
            m.causal_conv1d_fn = None
            m.causal_conv1d_update = mq.torch_causal_conv1d_update
            m.chunk_gated_delta_rule = mq.torch_chunk_gated_delta_rule
            m.recurrent_gated_delta_rule = mq.torch_recurrent_gated_delta_rule
            if not isinstance(m.norm, mq.Qwen3NextRMSNormGated):
                w = m.norm.weight.detach().float().cpu()
                m.norm = mq.Qwen3NextRMSNormGated(w.numel(), eps=m.layer_norm_epsilon)
                with torch.no_grad():
                    m.norm.weight.copy_(w)
