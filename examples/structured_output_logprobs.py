"""Grammar-constrained generation and logprobs with the LLM API.

    python examples/structured_output_logprobs.py --model /models/gpt-oss-120b --tp 8

Structured outputs must be switched on (``neuron_config.enable_structured_outputs``); the
tokenizer is read from the model directory.  Each request carries one constraint: a JSON schema,
any JSON object, a regex, a list of choices or an EBNF grammar.  ``logprobs=N`` returns, per
generated token, the N most likely tokens and the sampled one with their log-probabilities.
"""

import argparse
import json

from vllm_neuron_b200 import LLM, SamplingParams

SCHEMA = {"type": "object", "properties": {"city": {"type": "string"}, "population": {"type": "integer"}},
          "required": ["city", "population"], "additionalProperties": False}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--tp", type=int, default=1)
    a = ap.parse_args()
    llm = LLM(model=a.model, tensor_parallel_size=a.tp, max_model_len=4096,
              additional_config={"neuron_config": {"enable_structured_outputs": True}})
    tok = llm.get_tokenizer()
    jobs = [("Describe the largest city of France as JSON.", {"json": SCHEMA}),
            ("Is the sky blue? Answer yes or no.", {"choice": ["yes", "no"]}),
            ("Give a date.", {"regex": r"\d{4}-\d{2}-\d{2}"})]
    try:
        outs = llm.generate(prompt_token_ids=[tok.encode(p) for p, _ in jobs],
                            sampling_params=[SamplingParams(temperature=0.0, max_tokens=128, structured_outputs=so,
                                                            logprobs=2) for _, so in jobs])
    finally:
        llm.shutdown()
    for (prompt, so), o in zip(jobs, outs):
        c = o.outputs[0]
        text = tok.decode(c.token_ids, skip_special_tokens=True)
        print(f"{prompt!r} [{json.dumps(so)[:40]}] -> {text!r} ({c.finish_reason})")
        for t, entry in list(zip(c.token_ids, c.logprobs))[:3]:
            print("   ", repr(tok.decode([t])), {repr(tok.decode([i])): round(v, 3) for i, v in entry.items()})


if __name__ == "__main__":
    main()
