"""Check the engine against the HF transformers implementation of the same checkpoint:
greedy generations (every token within a small logit gap of the reference argmax) and
teacher-forced prompt logits (top-1 agreement, top-5 overlap, KL).

    python examples/accuracy_check.py --model /models/Llama-3.2-1B --device cuda
"""

import argparse

import torch

from vllm_neuron_b200 import LLM
from vllm_neuron_b200.accuracy import validate_greedy_generation, validate_prompt_logits


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--device", default="cuda")
    a = ap.parse_args()
    from transformers import AutoModelForCausalLM

    ref = AutoModelForCausalLM.from_pretrained(a.model, torch_dtype=torch.float32).eval()
    llm = LLM(model=a.model, device=a.device, max_model_len=2048, max_num_seqs=4)
    prompts = [list(range(1000, 1032)), list(range(2000, 2100))]
    for c in validate_greedy_generation(llm, ref, prompts, max_new_tokens=16, gap_tol=0.5):
        print(f"prompt {c.prompt_index}: {'ok' if c.passed else f'diverges at {c.first_divergence}'}, "
              f"max gap {max(c.gaps):.3f}")
    for m in validate_prompt_logits(llm.engine, ref, prompts):
        print(f"top1 {m.top1_agree:.3f} top5 {m.topk_overlap:.3f} max KL {m.kl:.4f}")
    llm.shutdown()


if __name__ == "__main__":
    main()
