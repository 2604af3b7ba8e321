"""Tiny GPT-OSS (MXFP4 experts) through the public ``LLM`` API on the GPU, with CUDA graphs
and asynchronous scheduling, checked against the CPU reference path (fp32, PyTorch ops) on
the same checkpoint.  The CPU engine scores every GPU generation with teacher forcing: at
each generated position the GPU's token must be the CPU's argmax or within a small logit gap
of it (near ties may flip between bf16 / MXFP8 and fp32; a rare isolated larger gap is a
router top-k near tie ordered differently, which the test allows once per 24 tokens)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(1, 4000, (n,), generator=g).tolist() for n in (9, 40, 150, 300)]


def test_gpt_oss_mxfp4_graphs_async_matches_cpu_reference(tmp_path):
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.testing import greedy_logit_gaps, write_tiny_gpt_oss_checkpoint

    path = str(tmp_path / "tiny_gpt_oss")
    write_tiny_gpt_oss_checkpoint(path)
    prompts = _prompts()
    nc = {"neuron_config": {"quantization": "mxfp4"}}
    kw = dict(model=path, max_model_len=512, max_num_seqs=4, max_num_batched_tokens=512, block_size=32,
              additional_config=nc)
    gpu = LLM(dtype="bfloat16", device="cuda", async_scheduling=True, **kw)
    try:
        outs = gpu.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
        gen = [list(o.outputs[0].token_ids) for o in outs]
        assert all(len(t) == 12 for t in gen)
        assert gpu.engine.worker.runner.graphs, "decode did not run through CUDA graphs"
        assert gpu.engine.async_stats["lookahead"] > 0, "no asynchronous decode step"
    finally:
        gpu.shutdown()
    cpu = LLM(dtype="float32", device="cpu", **kw)
    try:
        res = greedy_logit_gaps(cpu.engine, prompts, gen)
    finally:
        cpu.shutdown()
    # at most one position in 24 may be a discrete flip (router near tie); every other
    # generated token is the CPU argmax or within the logit-noise band of bf16 / MXFP8
    assert res.outliers() <= res.n_tokens // 24, f"GPU tokens far from the CPU argmax: {res}"
    assert res.exact_fraction >= 0.75, f"too few exact matches: {res}"


def _tp2_worker(rank, port, path, prompts, q):
    import os

    try:
        os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        from vllm_neuron_b200 import LLM, SamplingParams

        nc = {"neuron_config": {"quantization": "mxfp4", "ep_degree": 2}}
        llm = LLM(model=path, dtype="bfloat16", tensor_parallel_size=2, spmd=True, max_model_len=512,
                  max_num_seqs=4, max_num_batched_tokens=512, block_size=32, async_scheduling=True,
                  additional_config=nc)
        try:
            outs = llm.generate(prompt_token_ids=prompts,
                                sampling_params=SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
            gen = [list(o.outputs[0].token_ids) for o in outs]
            tp = llm.engine.worker.ps.tp
            sp_calls = tp.sp_comm.calls if tp.sp_comm is not None else 0
            ok = tp.sp_comm.check_canaries() if tp.sp_comm is not None else False
        finally:
            llm.shutdown()
        q.put((rank, gen, sp_calls, ok, None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, None, 0, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gpt_oss_tp2_ep2_matches_cpu_reference(tmp_path):
    """The same tiny model at TP = 2 x EP = 2 on two GPUs (one process each, as under
    torchrun): prefill steps take the sequence-parallel path (even token counts), whose layer
    boundaries are the scatter GEMM + the NVLink boundary kernel; decode steps the fused
    all-reduce with the MoE route sum.  Rank 0's tokens are scored by the CPU fp32 engine."""
    import socket

    import torch.multiprocessing as mp

    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.accuracy.testing import greedy_logit_gaps, write_tiny_gpt_oss_checkpoint

    path = str(tmp_path / "tiny_gpt_oss")
    write_tiny_gpt_oss_checkpoint(path)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(1, 4000, (n,), generator=g).tolist() for n in (10, 40, 150, 300)]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp2_worker, args=(r, port, path, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, gen, sp_calls, ok, tb in res:
        assert tb is None, tb
        assert sp_calls > 0, f"rank {rank}: no prefill boundary took the fused SP kernel"
        assert ok, f"rank {rank}: SP communicator guard bytes overwritten"
    gen = res[0][1]
    assert gen == res[1][1], "the ranks disagree"
    assert all(len(t) == 12 for t in gen)
    kw = dict(model=path, max_model_len=512, max_num_seqs=4, max_num_batched_tokens=512, block_size=32,
              additional_config={"neuron_config": {"quantization": "mxfp4"}})
    cpu = LLM(dtype="float32", device="cpu", **kw)
    try:
        r = greedy_logit_gaps(cpu.engine, prompts, gen)
    finally:
        cpu.shutdown()
    assert r.outliers() <= r.n_tokens // 24, f"TP2 GPU tokens far from the CPU argmax: {r}"
    assert r.exact_fraction >= 0.75, f"too few exact matches: {r}"
