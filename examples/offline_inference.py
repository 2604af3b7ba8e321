"""Offline batch generation with the LLM API.

    python examples/offline_inference.py --model /models/gpt-oss-120b --tp 8
    python examples/offline_inference.py --dummy gpt-oss-20b --tp 1        # random weights, no checkpoint

With ``--dummy`` the architecture comes from a built-in config and weights are random
(useful for smoke tests and benchmarking without a checkpoint).
"""

import argparse
import time

from vllm_neuron_b200 import LLM, SamplingParams

DUMMY = {
    "gpt-oss-20b": {
        "architectures": ["GptOssForCausalLM"], "model_type": "gpt_oss", "vocab_size": 201088, "hidden_size": 2880,
        "num_hidden_layers": 24, "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 64,
        "intermediate_size": 2880, "num_local_experts": 32, "num_experts_per_tok": 4, "sliding_window": 128,
        "layer_types": ["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(24)],
        "rope_theta": 150000.0, "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0,
                                                 "beta_slow": 1.0, "original_max_position_embeddings": 4096},
        "rms_norm_eps": 1e-5, "swiglu_limit": 7.0, "attention_bias": True, "max_position_embeddings": 131072,
        "quantization_config": {"quant_method": "mxfp4"}, "eos_token_id": 200002},
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    ap.add_argument("--dummy", choices=sorted(DUMMY), default=None)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=0.0)
    a = ap.parse_args()
    kw = dict(tensor_parallel_size=a.tp, max_model_len=4096, max_num_seqs=32, max_num_batched_tokens=4096)
    if a.dummy:
        llm = LLM(hf_config=DUMMY[a.dummy], load_format="dummy", **kw)
        token_prompts = [list(range(100 + i, 164 + i)) for i in range(8)]
        t0 = time.time()
        outs = llm.generate(prompt_token_ids=token_prompts,
                            sampling_params=SamplingParams(temperature=a.temperature, max_tokens=a.max_tokens,
                                                           ignore_eos=True))
    else:
        llm = LLM(model=a.model, **kw)
        t0 = time.time()
        outs = llm.generate(["The capital of France is", "Write a haiku about GPUs:"],
                            SamplingParams(temperature=a.temperature, max_tokens=a.max_tokens))
    dt = time.time() - t0
    n = sum(len(o.outputs[0].token_ids) for o in outs)
    for o in outs[:4]:
        print(repr(o.outputs[0].text or o.outputs[0].token_ids[:16]))
    print(f"{n} tokens in {dt:.2f}s ({n / dt:.1f} tok/s)")
    llm.shutdown()


if __name__ == "__main__":
    main()
