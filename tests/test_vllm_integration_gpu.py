"""vLLM's ``LLM`` on a B200 with this plugin: vLLM's CUDA platform underneath, this
framework's worker (tcgen05 GEMMs, MXFP4 grouped GEMM, paged attention kernels, decode CUDA
graphs) and scheduler.  The tiny GPT-OSS checkpoint's greedy tokens are scored against this
framework's CPU fp32 engine with teacher forcing (as the engine's own GPU end-to-end test)."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
pytest.importorskip("vllm")

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_vllm_llm_with_b200_worker_on_gpu(tmp_path):
    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.accuracy.testing import greedy_logit_gaps, write_tiny_gpt_oss_checkpoint

    path = str(tmp_path / "tiny_gpt_oss")
    write_tiny_gpt_oss_checkpoint(path)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(1, 4000, (n,), generator=g).tolist() for n in (9, 40, 150, 300)]
    nc = {"neuron_config": {"quantization": "mxfp4"}}
    args = {"model": path, "prompts": prompts, "max_tokens": 12, "dtype": "bfloat16", "block_size": 32,
            "additional_config": nc, "enforce_eager": False, "max_num_batched_tokens": 512,
            "max_model_len": 512}
    env = dict(os.environ)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    p = subprocess.run([sys.executable, os.path.join(HERE, "vllm_plugin_driver.py"), json.dumps(args)],
                       capture_output=True, text=True, timeout=900, env=env, cwd=ROOT)
    lines = [l for l in p.stdout.splitlines() if l.startswith("RESULT ")]
    assert p.returncode == 0 and lines, f"vLLM run failed (rc {p.returncode}):\n{p.stderr[-6000:]}"
    res = json.loads(lines[-1][len("RESULT "):])
    assert res["worker_cls"].endswith("B200VllmWorker")
    assert res["scheduler_type"].startswith("B200Vllm")
    gen = res["tokens"]
    assert all(len(t) == 12 for t in gen)
    cpu = LLM(model=path, dtype="float32", device="cpu", max_model_len=512, max_num_seqs=4,
              max_num_batched_tokens=512, block_size=32, additional_config=nc)
    try:
        r = greedy_logit_gaps(cpu.engine, prompts, gen)
    finally:
        cpu.shutdown()
    assert r.outliers() <= r.n_tokens // 24, f"vLLM-driven GPU tokens far from the CPU argmax: {r}"
    assert r.exact_fraction >= 0.75, f"too few exact matches: {r}"
