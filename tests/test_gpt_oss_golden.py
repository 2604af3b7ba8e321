"""Config 1: tiny GPT-OSS-architecture MoE, greedy outputs vs HF transformers fp32.

The HF model (eager attention with sinks + sliding window, dense experts) is the
oracle; our engine loads the same weights from a safetensors checkpoint and must
produce the same greedy tokens with TP=1 and TP=2 (gloo ranks on CPU)."""

import copy

import pytest
import torch

from tiny_configs import TINY_GPT_OSS, workload


def _hf_model():
    from transformers import GptOssConfig, GptOssForCausalLM

    torch.manual_seed(0)
    cfg = GptOssConfig(**{k: v for k, v in TINY_GPT_OSS.items() if k not in ("architectures",)})
    cfg._attn_implementation = "eager"
    m = GptOssForCausalLM(cfg).eval().float()
    # HF zero-initialises expert biases and the router bias is small; give every
    # parameter a non-trivial value so the test exercises them.
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("bias") or "sinks" in n:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    return m, cfg


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    m, cfg = _hf_model()
    path = tmp_path_factory.mktemp("tiny_gpt_oss")
    hf_cfg = m.config.to_dict()
    hf_cfg["architectures"] = ["GptOssForCausalLM"]
    save_state_dict({k: v.detach().clone() for k, v in m.state_dict().items()}, str(path), hf_cfg)
    return str(path), m


def _hf_greedy(m, prompts, n_new):
    outs = []
    with torch.no_grad():
        for p in prompts:
            ids = torch.tensor([p])
            g = m.generate(ids, max_new_tokens=n_new, do_sample=False, eos_token_id=None, pad_token_id=0)
            outs.append(g[0, len(p):].tolist())
    return outs


@pytest.mark.parametrize("tp,dp,a2a,adp,dcp,ep", [(1, 1, None, 1, 1, None), (2, 1, None, 1, 1, None),
                                                  (1, 2, None, 1, 1, None), (1, 2, "naive", 1, 1, "all"),
                                                  (2, 1, "naive", 1, 1, "all"), (1, 2, None, 2, 1, None),
                                                  (2, 2, None, 2, 1, None), (4, 1, None, 1, 2, None),
                                                  (2, 1, None, 1, 1, "all"), (4, 1, None, 1, 1, 2)])
def test_greedy_matches_hf(ckpt, tp, dp, a2a, adp, dcp, ep, monkeypatch):
    """dp=2: two data-parallel replicas in lockstep with the experts shared across them
    (tokens all-gathered / reduce-scattered over DP around the MoE); 5 prompts so one
    replica runs padding steps while the other still works.  a2a: the EP all-to-all
    (each token sent only to the ranks owning its experts; under TP each rank sends a
    slice and the outputs are partial sums).  adp: attention DP (the model runs on every
    replica's tokens over the TP x DP supergroup; attention per replica after a batch <-> heads
    all-to-all).  dcp: decode context parallelism (the two TP ranks that replicate a kv head
    split its tokens; sinks join the LSE merge once, windows are in global positions).
    ep: None = MoE tensor parallelism (every rank holds every expert, the intermediate
    dimension split over the ranks), "all" = expert parallelism over every rank, an int =
    variable EP (that many expert partitions, each split over world / ep ranks)."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.parallel import all2all

    calls = {"n": 0}
    orig = all2all.EpAll2All.dispatch

    def spy(self, *a, **k):
        calls["n"] += 1
        return orig(self, *a, **k)

    monkeypatch.setattr(all2all.EpAll2All, "dispatch", spy)
    from vllm_neuron_b200.parallel import state as pstate

    a2a_calls = {"n": 0}
    orig_a2a = pstate.GroupCoordinator.all_to_all

    def spy_a2a(self, *a, **k):
        a2a_calls["n"] += 1
        return orig_a2a(self, *a, **k)

    monkeypatch.setattr(pstate.GroupCoordinator, "all_to_all", spy_a2a)
    path, hf = ckpt
    prompts = workload(n=4 if tp >= 2 else (5 if dp == 2 else 6))
    n_new = 16
    want = _hf_greedy(hf, prompts, n_new)
    llm = LLM(model=path, dtype="float32", max_model_len=512, max_num_seqs=16, max_num_batched_tokens=256,
              block_size=16, device="cpu", tensor_parallel_size=tp, data_parallel_size=dp,
              all2all_backend=a2a or "allgather_reducescatter", decode_context_parallel_size=dcp,
              enable_expert_parallel=ep == "all",
              additional_config={"neuron_config": {"quantization": "bf16", "attention_dp_size": adp,
                                                   "ep_degree": ep if isinstance(ep, int) else 1}})
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=n_new, ignore_eos=True))
    finally:
        llm.shutdown()
    got = [o.outputs[0].token_ids for o in outs]
    assert got == want
    assert (calls["n"] > 0) == bool(a2a)
    assert (a2a_calls["n"] > 0) == (adp > 1)  # batch <-> heads exchange around attention


def test_moe_tp_mxfp4_pads_intermediate():
    """MoE tensor parallelism with MXFP4 experts whose intermediate size does not split into
    whole 32-element scale blocks per rank (I = 96 over 2 ranks: 48 each): I is padded to 128
    with zero channels, and the partial sums of the two slices equal the unsharded experts."""
    from vllm_neuron_b200.models.gpt_oss import GptOssConfig, GptOssExperts, GptOssForCausalLM
    from vllm_neuron_b200.ops import reference as ref

    torch.manual_seed(0)
    E, H, I = 4, 64, 96
    cfg = GptOssConfig(hidden_size=H, intermediate_size=I, num_local_experts=E, num_experts_per_tok=2,
                       quantization="mxfp4")
    w13 = torch.randn(E, H, 2 * I) * 0.05  # HF layout [E, H, 2I], gate/up interleaved
    w2 = torch.randn(E, I, H) * 0.05
    b13, b2 = torch.randn(E, 2 * I) * 0.02, torch.randn(E, H) * 0.02
    x = torch.randn(5, H)
    ids = torch.stack([torch.randperm(E)[:2] for _ in range(5)]).to(torch.int32)
    wts = torch.softmax(torch.randn(5, 2), -1)

    def build(rank, size):
        ex = GptOssExperts(cfg, 0, 1, torch.float32, "cpu", rank, size)
        for name, t in (("gate_up_proj", w13), ("down_proj", w2)):
            which = "13" if name == "gate_up_proj" else "2"
            sl = ex.slice_13(t.transpose(1, 2), 1) if which == "13" else ex.slice_2(t.transpose(1, 2), 2)
            GptOssForCausalLM._load_dense(ex, which, sl)
        ex.b13.data.copy_(ex.slice_13(b13, 1))
        ex.b2.data.copy_(b2 if rank == 0 else torch.zeros_like(b2))
        return ex

    full = build(0, 1)
    parts = [build(r, 2) for r in range(2)]
    assert parts[0].I == 64 and parts[0].I_pad == 128  # 96 -> 128: two slices of two scale blocks
    want = full(x, ids, wts)
    got = parts[0](x, ids, wts) + parts[1](x, ids, wts)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-4), (got - want).abs().max()


def test_long_prompts_with_sliding_window_kv_group(ckpt):
    """Prompts several windows long, prefilled in chunks: the sliding-window layers read their
    own KV group, whose blocks behind the window are returned while the request runs, and the
    greedy tokens still match HF."""
    from vllm_neuron_b200 import LLM, SamplingParams

    path, hf = ckpt
    prompts = workload(n=2, lo=300, hi=420, seed=3)
    want = _hf_greedy(hf, prompts, 8)
    llm = LLM(model=path, dtype="float32", max_model_len=512, max_num_seqs=4, max_num_batched_tokens=128,
              block_size=16, device="cpu", additional_config={"neuron_config": {"quantization": "bf16"}})
    try:
        kv = llm.engine.kv
        assert kv.swa_pool is not None and kv.window == 128
        seen = []
        orig = kv._trim_window

        def spy(req):
            orig(req)
            seen.append(req.swa_freed)

        kv._trim_window = spy
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    finally:
        llm.shutdown()
    assert max(seen) >= 10  # blocks behind the window were returned during prefill and decode
    assert [o.outputs[0].token_ids for o in outs] == want
