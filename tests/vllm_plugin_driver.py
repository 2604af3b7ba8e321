"""Runs vLLM's own ``LLM`` with this framework's platform, worker and scheduler (used by
``test_vllm_integration.py`` in a child process, so vLLM's process-wide state stays out of
the test session).  Prints one JSON line: generated tokens, the classes vLLM used."""

import json
import os
import sys


def main() -> None:
    args = json.loads(sys.argv[1])
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"  # engine core in this process
    import vllm.platforms as vp

    from vllm_neuron_b200.platform import B200Platform

    vp._current_platform = B200Platform()  # what the plugin entry point selects when installed
    import vllm
    from vllm import SamplingParams
    from vllm.inputs import TokensPrompt

    kw = dict(model=args["model"], skip_tokenizer_init=True, max_model_len=args.get("max_model_len", 256), max_num_seqs=args.get("max_num_seqs", 4),
              max_num_batched_tokens=args.get("max_num_batched_tokens", 128), block_size=args.get("block_size", 16),
              dtype=args.get("dtype", "float32"), enforce_eager=args.get("enforce_eager", True), gpu_memory_utilization=0.5, enable_prefix_caching=args.get("prefix", False),
              seed=0)
    if args.get("additional_config"):
        kw["additional_config"] = args["additional_config"]
    if args.get("num_gpu_blocks_override"):
        kw["num_gpu_blocks_override"] = args["num_gpu_blocks_override"]
    llm = vllm.LLM(**kw)
    sp = SamplingParams(temperature=0, max_tokens=args["max_tokens"], ignore_eos=True, detokenize=False)
    prompts = [TokensPrompt(prompt_token_ids=p) for p in args["prompts"]]
    outs = llm.generate(prompts, sp, use_tqdm=False)
    res = {"tokens": [list(o.outputs[0].token_ids) for o in outs],
           "cached": [o.num_cached_tokens or 0 for o in outs]}
    if args.get("repeat"):
        again = llm.generate(prompts, sp, use_tqdm=False)
        res["tokens_again"] = [list(o.outputs[0].token_ids) for o in again]
        res["cached_again"] = [o.num_cached_tokens or 0 for o in again]
    vc = llm.llm_engine.vllm_config
    res["worker_cls"] = vc.parallel_config.worker_cls
    res["scheduler_cls"] = str(vc.scheduler_config.scheduler_cls)
    core = llm.llm_engine.engine_core.engine_core
    res["scheduler_type"] = type(core.scheduler).__name__
    print("RESULT " + json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
