"""End-to-end logit tests (the reference's test level 4): the engine's decode-path logits,
read from its ``debug_logits_dir`` dumps, validated with teacher forcing by
``multi_prompt_logit_validation`` against HF fp32 goldens (kept in the golden cache) over a grid
of tensor-parallel degrees, prompt lengths and batch sizes, on the tiny GPT-OSS configuration
(CPU, gloo ranks for TP=2)."""

import pytest
import torch

from test_gpt_oss_golden import _hf_model
from tiny_configs import workload

N_NEW = 8


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    m, _ = _hf_model()
    path = tmp_path_factory.mktemp("grid_gpt_oss")
    d = m.config.to_dict()
    d["architectures"] = ["GptOssForCausalLM"]
    save_state_dict({k: v.detach().clone() for k, v in m.state_dict().items()}, str(path), d)
    return str(path), m


@torch.no_grad()
def _hf_logits(m, batch: list[list[int]], n: int) -> torch.Tensor:
    """Greedy continuation logits [n, B, V] (fp32)."""
    cols = []
    for p in batch:
        out = m(torch.tensor([p]), use_cache=True)
        rows = [out.logits[0, -1].float()]
        for _ in range(n - 1):
            out = m(rows[-1].argmax().view(1, 1), past_key_values=out.past_key_values, use_cache=True)
            rows.append(out.logits[0, -1].float())
        cols.append(torch.stack(rows))
    return torch.stack(cols, 1)


@pytest.mark.parametrize("tp", [1, 2])
def test_logit_grid_matches_hf(ckpt, tp, tmp_path, monkeypatch):
    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.accuracy import make_engine_generate_fn, multi_prompt_logit_validation
    from vllm_neuron_b200.utils.golden_cache import get_or_compute, golden_key

    monkeypatch.setenv("VLLM_B200_GOLDEN_CACHE_DIR", str(tmp_path / "goldens"))
    path, hf = ckpt
    grid = []  # (prompt length, batch size) -> one batch of prompts
    for L in (16, 40):
        for B in (1, 3):
            grid.append(workload(n=B, lo=L, hi=L + 1, seed=100 * L + B))
    expected = [get_or_compute(golden_key(model="tiny_gpt_oss", prompts=b, n=N_NEW), lambda b=b: _hf_logits(hf, b, N_NEW))
                for b in grid]
    d = str(tmp_path / "logits")
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=64,
              block_size=16, device="cpu", tensor_parallel_size=tp,
              additional_config={"neuron_config": {"quantization": "bf16", "debug_logits_dir": d}})
    try:
        res = multi_prompt_logit_validation(grid, make_engine_generate_fn(llm, N_NEW, d), expected)
    finally:
        llm.shutdown()
    assert res.passed, "\n".join(r.summary() for r in res.per_prompt)
    assert [len(r.tokens) for r in res.per_prompt] == [1, 3, 1, 3]
    assert all(len(row) == N_NEW for r in res.per_prompt for row in r.tokens)
