"""Disaggregated prefill/decode on one GPU with the device transport (B200IpcConnector):
the prefill engine (its own process, kept alive while the decode engine reads its pool)
exports every request's KV into a CUDA-IPC device pool, and the decode engine copies it into
its blocks with one kernel.  The synthetic KV-verifying model must find every prompt
position's KV exactly as the prefill engine wrote it, with different block sizes on the two
sides."""

import multiprocessing as mp
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

SYN = {"architectures": ["SyntheticModel"], "num_hidden_layers": 3, "num_key_value_heads": 4, "head_dim": 16,
       "vocab_size": 32, "max_position_embeddings": 1024}
PROMPTS = [list(range(1, 40)), list(range(3, 100)), [9, 8, 7]]


def _llm(role, store, block_size):
    from vllm_neuron_b200 import LLM

    return LLM(hf_config=dict(SYN), load_format="dummy", dtype="bfloat16", max_model_len=256, max_num_seqs=4,
               max_num_batched_tokens=256, block_size=block_size, device="cuda", enforce_eager=True,
               gpu_memory_utilization=0.2,
               kv_transfer_config={"kv_connector": "B200IpcConnector", "kv_role": role,
                                   "kv_connector_extra_config": {"store_path": store, "timeout_s": 60,
                                                                 "pool_mb": 64, "engine_id": f"{role}-eng"}})


def _producer(store, q, done):
    try:
        os.environ["VLLM_B200_SYNTHETIC_MODEL"] = "1"
        from vllm_neuron_b200 import SamplingParams

        llm = _llm("kv_producer", store, 16)
        outs = llm.generate([{"prompt_token_ids": p, "kv_transfer_params": {"do_remote_decode": True}}
                             for p in PROMPTS], SamplingParams(temperature=0, max_tokens=1, ignore_eos=True))
        q.put(([o.kv_transfer_params for o in outs], [o.outputs[0].token_ids for o in outs], None))
        done.wait(300)  # the pool must outlive the decode engine's reads
        llm.shutdown()
    except Exception:  # noqa: BLE001
        import traceback

        q.put((None, None, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_ipc_transfer_one_gpu(tmp_path, monkeypatch):
    monkeypatch.setenv("VLLM_B200_SYNTHETIC_MODEL", "1")
    from vllm_neuron_b200 import SamplingParams
    from vllm_neuron_b200.models.synthetic import TOKEN_EMPTY, TOKEN_SUCCESS

    store = str(tmp_path / "kv")
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    p = ctx.Process(target=_producer, args=(store, q, done))
    p.start()
    try:
        params, first, tb = q.get(timeout=300)
        assert tb is None, tb
        assert first == [[TOKEN_EMPTY]] * 3
        assert all(kp["transport"] == "ipc" for kp in params), params
        decode = _llm("kv_consumer", store, 32)
        try:
            outs = decode.generate([{"prompt_token_ids": pr, "kv_transfer_params": kp}
                                    for pr, kp in zip(PROMPTS, params)],
                                   SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
            st = dict(decode.engine.connector.stats)
            status = int(decode.engine.connector.status[0].item())
        finally:
            decode.shutdown()
    finally:
        done.set()
        p.join(timeout=120)
    for o, pr in zip(outs, PROMPTS):
        assert o.outputs[0].token_ids == [TOKEN_SUCCESS] * 4, o.outputs[0].token_ids
        assert o.num_cached_tokens == len(pr) - 1
    assert st["loaded"] == 3 and status == 0
