"""EAGLE-3 speculative decoding: a one-layer draft model proposes k tokens per step, the
target verifies them in one forward pass (greedy: lossless; sampled requests: rejection
sampling keeps the output distribution).

    python examples/eagle3_speculative.py --model /models/Llama-3.1-8B-Instruct \
        --draft /models/EAGLE3-LLaMA3.1-Instruct-8B --k 4
"""

import argparse

from vllm_neuron_b200 import LLM, SamplingParams


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--draft", required=True)
    ap.add_argument("--k", type=int, default=4)
    a = ap.parse_args()
    llm = LLM(model=a.model, max_model_len=4096, max_num_seqs=16,
              speculative_config={"method": "eagle3", "model": a.draft, "num_speculative_tokens": a.k})
    outs = llm.generate(["Summarise the history of the transistor."] * 4,
                        SamplingParams(temperature=0, max_tokens=128))
    print(outs[0].outputs[0].text)
    print("acceptance rate", llm.engine.proposer.acceptance_rate())
    llm.shutdown()


if __name__ == "__main__":
    main()
