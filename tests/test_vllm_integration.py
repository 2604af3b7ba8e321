"""``vllm serve`` / ``vllm.LLM`` with this plugin: vLLM's engine (request queue, KV block
manager, prefix caching, preemption) drives this framework's worker and scheduler.  On the
CPU the platform's base is vLLM's CPU platform and the worker runs this framework's CPU
path; greedy tokens must equal this framework's own engine on the same checkpoint."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytest.importorskip("vllm")

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=1024,
                      tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).eval()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    path = tmp_path_factory.mktemp("llama_vllm")
    save_state_dict({k: v.detach().clone().contiguous() for k, v in m.state_dict().items()}, str(path), d)
    return str(path)


def _prompts():
    g = torch.Generator().manual_seed(1)
    return [torch.randint(1, 2000, (n,), generator=g).tolist() for n in (5, 30, 70, 150)]


def _run_vllm(args: dict) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    env["CUDA_VISIBLE_DEVICES"] = ""
    p = subprocess.run([sys.executable, os.path.join(HERE, "vllm_plugin_driver.py"), json.dumps(args)],
                       capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    lines = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")]
    assert p.returncode == 0 and lines, f"vLLM run failed (rc {p.returncode}):\n{p.stderr[-4000:]}"
    return json.loads(lines[-1][len("RESULT "):])


def _ours(path: str, prompts, max_tokens: int):
    from vllm_neuron_b200 import LLM, SamplingParams

    llm = LLM(model=path, dtype="float32", device="cpu", max_model_len=256, max_num_seqs=4,
              max_num_batched_tokens=128, block_size=16)
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=max_tokens, ignore_eos=True))
        return [list(o.outputs[0].token_ids) for o in outs]
    finally:
        llm.shutdown()


def test_vllm_engine_runs_b200_worker_and_scheduler(ckpt):
    """The plugin's classes are the ones vLLM uses; greedy tokens equal this framework's
    engine; prefix-cache hits (the second pass over the same prompts reuses the first pass's
    blocks) arrive as computed tokens and leave the tokens unchanged."""
    prompts = _prompts()
    want = _ours(ckpt, prompts, 12)
    res = _run_vllm({"model": ckpt, "prompts": prompts, "max_tokens": 12, "prefix": True, "repeat": True})
    assert res["worker_cls"] == "vllm_neuron_b200.vllm_integration.worker.B200VllmWorker"
    assert res["scheduler_type"] in ("B200VllmScheduler", "B200VllmAsyncScheduler"), res["scheduler_type"]
    assert res["tokens"] == want and res["tokens_again"] == want
    assert sum(res["cached_again"]) > 0, res["cached_again"]


def test_vllm_small_kv_pool(ckpt):
    """A KV pool too small for all four requests at once (vLLM queues or preempts and
    recomputes) and 64-token prefill chunks must not change greedy tokens."""
    prompts = _prompts()
    want = _ours(ckpt, prompts, 12)
    small = _run_vllm({"model": ckpt, "prompts": prompts, "max_tokens": 12, "num_gpu_blocks_override": 18,
                       "max_num_batched_tokens": 64})
    assert small["tokens"] == want
