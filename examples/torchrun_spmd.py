"""SPMD launch: one process per GPU started by torchrun; every rank builds the engine and
submits the same requests (the schedulers stay in lockstep), rank 0 prints.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/torchrun_spmd.py \
        --model /models/gpt-oss-120b --tp 8
"""

import argparse
import os

from vllm_neuron_b200 import LLM, SamplingParams


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--tp", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--dp", type=int, default=1)
    a = ap.parse_args()
    llm = LLM(model=a.model, spmd=True, tensor_parallel_size=a.tp // a.dp, data_parallel_size=a.dp,
              max_model_len=8192, max_num_seqs=64)
    outs = llm.generate(["Explain NVLink in one sentence."] * 4, SamplingParams(temperature=0, max_tokens=48))
    if int(os.environ.get("RANK", "0")) == 0:
        for o in outs:
            print(o.outputs[0].text)
    llm.shutdown()


if __name__ == "__main__":
    main()
