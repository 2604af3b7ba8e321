"""Teacher-forced logit validation and KV-cache comparison of the engine against HF
transformers on the same checkpoint.

    python examples/logit_and_kv_validation.py --model /models/Llama-3.2-1B --device cuda --tokens 32

1. HF fp32 greedy logits for each prompt are the expected values (``--baseline-fp64`` also
   computes float64 logits for the three-way statistics).
2. The engine runs with ``neuron_config.debug_logits_dir``, so its decode-path logits are
   dumped every step; ``multi_prompt_logit_validation`` checks them position by position with
   teacher forcing (tolerance tiers, ULP-aware handling of flipped near-ties).
3. ``KVSnapshot`` keeps the KV of each finished request; ``compare_kv_caches`` compares it per
   token, layer and head against HF's cache of the same tokens.
"""

import argparse
import tempfile

import torch


@torch.no_grad()
def hf_greedy_logits(m, prompt, n, dtype=torch.float32):
    out = m(torch.tensor([prompt]), use_cache=True)
    rows = [out.logits[0, -1].to(dtype)]
    for _ in range(n - 1):
        out = m(rows[-1].argmax().view(1, 1), past_key_values=out.past_key_values, use_cache=True)
        rows.append(out.logits[0, -1].to(dtype))
    return torch.stack(rows)[:, None]  # [n, 1, V]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--baseline-fp64", action="store_true")
    a = ap.parse_args()
    import copy

    from transformers import AutoModelForCausalLM

    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy import make_engine_generate_fn, multi_prompt_logit_validation
    from vllm_neuron_b200.accuracy.kv_cache_analysis import KVSnapshot, compare_kv_caches, extract_hf_kv, kv_report

    hf = AutoModelForCausalLM.from_pretrained(a.model, torch_dtype=torch.float32).eval()
    V = hf.config.vocab_size
    prompts = [[(1000 + i) % V for i in range(32)], [(2000 + 7 * i) % V for i in range(100)]]
    expected = [hf_greedy_logits(hf, p, a.tokens) for p in prompts]
    baseline = None
    if a.baseline_fp64:
        hf64 = copy.deepcopy(hf).double()
        baseline = [hf_greedy_logits(hf64, p, a.tokens).float() for p in prompts]
    d = tempfile.mkdtemp(prefix="b200_logits_", dir="/dev/shm" if a.device == "cuda" else None)
    llm = LLM(model=a.model, device=a.device, dtype=a.dtype, max_model_len=1024, max_num_seqs=4,
              additional_config={"neuron_config": {"debug_logits_dir": d}})
    try:
        res = multi_prompt_logit_validation([[p] for p in prompts], make_engine_generate_fn(llm, a.tokens, d),
                                            expected, prompts_baseline_logits=baseline)
        for r in res.per_prompt:
            print(r.summary())
        if res.aggregate:
            print({k: v for k, v in res.aggregate.items() if k != "per_token_bc"})
        print("logit validation:", "PASS" if res.passed else "FAIL")
        with KVSnapshot(llm.engine) as snap:
            outs = llm.generate(prompt_token_ids=prompts,
                                sampling_params=SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
        for p, o in zip(prompts, outs):
            seq = p + list(o.outputs[0].token_ids)[:-1]
            print(kv_report(compare_kv_caches(extract_hf_kv(hf, seq), snap.kv[o.request_id])))
    finally:
        llm.shutdown()


if __name__ == "__main__":
    main()
