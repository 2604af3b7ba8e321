"""Qwen3-Next kernels on the GPU vs the fp32 PyTorch reference: causal conv with state,
chunked gated-DeltaNet prefill (varlen, carried-in state), recurrent decode, gating
kernels, bf16 grouped experts; and the whole hybrid model through the engine."""

import pytest
import torch

from tiny_configs import hf_torch_path

pytestmark = pytest.mark.gpu


def _meta(lens, init, device="cuda"):
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=device)
    B = len(lens)
    m = AttentionMetadata(int(qsl[-1]), B, max(lens) == 1, qsl, None, None, None, None, max(lens), max(lens))
    m.extras = {"state_slots": torch.arange(B, dtype=torch.int32, device=device).flip(0).contiguous(),
                "state_init": torch.tensor(init, dtype=torch.int32, device=device)}
    return m


@pytest.mark.parametrize("lens,init", [([1, 1, 1], [1, 0, 1]), ([5, 70, 130, 2], [0, 1, 1, 0])])
def test_causal_conv1d(lens, init):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.reference import deltanet as dn

    torch.manual_seed(0)
    C, K = 384, 4
    meta = _meta(lens, init)
    T = meta.num_tokens
    y = torch.randn(T, C + 64, device="cuda").bfloat16()
    x = y[:, :C]
    w = (0.5 * torch.randn(C, K, device="cuda")).bfloat16()
    st = torch.randn(len(lens), C, K - 1, device="cuda").bfloat16()
    st_ref = st.float().clone()
    got = ops.causal_conv1d(x, w, st, meta)
    want = dn.causal_conv1d(x.float(), w.float(), st_ref, meta.query_start_loc.cpu(),
                            meta.extras["state_slots"].cpu(), meta.extras["state_init"].cpu())
    torch.testing.assert_close(got.float(), want, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(st.float(), st_ref, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("lens,init", [([1, 1, 1, 1], [1, 1, 0, 1]), ([37, 64, 150, 1, 200], [0, 1, 1, 0, 1])])
def test_gated_delta_net(lens, init):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.reference import deltanet as dn

    torch.manual_seed(1)
    nk, nv, d = 2, 4, 128
    meta = _meta(lens, init)
    T, B = meta.num_tokens, len(lens)
    mixed = torch.randn(T, 2 * nk * d + nv * d, device="cuda").bfloat16()
    proj = torch.randn(T, nv * d + 2 * nv + 8, device="cuda").bfloat16()
    z, b, a = proj[:, :nv * d], proj[:, nv * d:nv * d + nv], proj[:, nv * d + nv:nv * d + 2 * nv]
    A_log = torch.log(torch.empty(nv, device="cuda").uniform_(1, 16))
    dt_bias = torch.randn(nv, device="cuda")
    norm_w = 1 + 0.1 * torch.randn(d, device="cuda")
    state = 0.1 * torch.randn(B, nv, d, d, device="cuda")
    st_ref = state.clone().cpu()
    got = ops.gated_delta_net(mixed, z, b, a, A_log, dt_bias, norm_w, 1e-6, state, meta, nk, nv, d, d)
    q = mixed[:, :nk * d].reshape(T, nk, d).float().cpu()
    k = mixed[:, nk * d:2 * nk * d].reshape(T, nk, d).float().cpu()
    v = mixed[:, 2 * nk * d:].reshape(T, nv, d).float().cpu()
    g, beta = dn.gate_and_beta(a.float().cpu(), b.float().cpu(), A_log.cpu(), dt_bias.cpu())
    o = dn.gated_delta_rule(q, k, v, g, beta, st_ref, meta.query_start_loc.cpu(), meta.extras["state_slots"].cpu(),
                            meta.extras["state_init"].cpu())
    want = dn.gated_rms_norm(o.bfloat16(), z.reshape(T, nv, d).cpu(), norm_w.cpu(), 1e-6).reshape(T, nv * d)
    gf, wf = got.float().cpu().reshape(T, nv, d), want.float().reshape(T, nv, d)
    rel = (gf - wf).norm(dim=-1) / wf.norm(dim=-1).clamp_min(1e-3)  # per (token, head)
    # rows whose pre-norm output nearly cancels (|o| << typical) are amplified by the RMSNorm;
    # there the bf16 tensor-core dot products differ from fp32 by design
    on = o.norm(dim=-1)
    typical = on > 0.25 * on.median()
    err = (gf - wf).abs()
    assert rel[typical].max() < 0.05 and err.mean() < 5e-3, (rel[typical].max(), err.mean())
    serr = (state.cpu() - st_ref).abs()
    assert serr.max() < 2e-2 * max(1.0, st_ref.abs().max().item()), serr.max()


def test_gates():
    from vllm_neuron_b200 import ops

    torch.manual_seed(2)
    x = torch.randn(7, 512, device="cuda").bfloat16()
    g = torch.randn(7, 1024, device="cuda").bfloat16()[:, 256:768]
    torch.testing.assert_close(ops.sigmoid_gate_mul(x, g).float(), x.float() * torch.sigmoid(g.float()),
                               atol=2e-2, rtol=2e-2)
    y = torch.randn(7, 512, device="cuda").bfloat16()
    sg = torch.randn(7, 1, device="cuda").bfloat16()
    torch.testing.assert_close(ops.gated_add(x, y, sg).float(), x.float() + torch.sigmoid(sg.float()) * y.float(),
                               atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("T,E,H,I,k,act", [(5, 8, 256, 128, 2, "silu"), (40, 64, 512, 192, 10, "silu"),
                                           (300, 16, 2880, 2880, 4, "swiglu_clamp")])
def test_moe_bf16(T, E, H, I, k, act):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops import reference as ref

    torch.manual_seed(3)
    x = torch.randn(T, H, device="cuda").bfloat16()
    w13 = (torch.randn(E, 2 * I, H, device="cuda") / H ** 0.5).bfloat16()
    w2 = (torch.randn(E, H, I, device="cuda") / I ** 0.5).bfloat16()
    logits = torch.randn(T, E, device="cuda")
    wts, ids = torch.topk(torch.softmax(logits, -1), k, -1)
    ids = ids.to(torch.int32)
    interleaved = act == "swiglu_clamp"
    limit = 7.0 if interleaved else None
    want = ref.moe_experts(x, ids, wts, w13.float(), None, w2.float(), None, 1.702, limit, interleaved, 0, act)
    t13, t2 = ops.prepare_moe_bf16(w13, w2, interleaved)
    got = ops.moe_dense(x, ids, wts, t13, None, t2, None, 0, 1.702, limit, interleaved, act, H, I)
    torch.testing.assert_close(got.float(), want.float(), atol=3e-2, rtol=3e-2)


def test_qwen3_next_engine_bf16():
    """Tiny Qwen3-Next (real head dims: attention 256, DeltaNet 128) in bf16 on the GPU:
    greedy tokens must be the HF fp32 argmax or within a small logit gap of it."""
    from transformers import Qwen3NextConfig, Qwen3NextForCausalLM

    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = Qwen3NextConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                          num_attention_heads=4, num_key_value_heads=2, head_dim=256, linear_conv_kernel_dim=4,
                          linear_key_head_dim=128, linear_value_head_dim=128, linear_num_key_heads=2,
                          linear_num_value_heads=4, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=128,
                          shared_expert_intermediate_size=128, max_position_embeddings=2048,
                          rope_parameters={"rope_type": "default", "rope_theta": 10000.0,
                                           "partial_rotary_factor": 0.25})
    cfg._attn_implementation = "eager"
    hf = Qwen3NextForCausalLM(cfg).eval().float()
    hf_torch_path(hf)
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n:
                p.copy_(0.1 * torch.randn_like(p) + (1.0 if n.endswith("linear_attn.norm.weight") else 0.0))
            elif n.endswith("A_log"):
                p.copy_(torch.log(torch.empty_like(p).uniform_(1, 16)))
    import tempfile

    d = cfg.to_dict()
    d["architectures"] = ["Qwen3NextForCausalLM"]
    path = tempfile.mkdtemp()
    save_state_dict({k: v.detach().clone().contiguous() for k, v in hf.state_dict().items()}, path, d)
    prompts = [list(range(3, 3 + n)) for n in (9, 100, 260)]
    llm = LLM(model=path, dtype="bfloat16", max_model_len=512, max_num_seqs=4, max_num_batched_tokens=192,
              block_size=32, device="cuda")
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    finally:
        llm.shutdown()
    with torch.no_grad():
        for p, o in zip(prompts, outs):
            toks = o.outputs[0].token_ids
            full = torch.tensor([p + toks])
            logits = hf(full).logits[0, len(p) - 1:-1]
            for i, t in enumerate(toks):
                gap = (logits[i].max() - logits[i, t]).item()
                assert gap < 0.1 * logits[i].std().item() + 0.05, (i, gap)


@pytest.mark.parametrize("T,E,H,I,k", [(7, 16, 512, 256, 4), (64, 64, 2048, 512, 10)])
def test_moe_mxfp8_experts(T, E, H, I, k):
    """fp8-checkpoint experts: MXFP8 weights (e4m3 + ue8m0 per 32) on the block-scaled tcgen05
    GEMM with plain SiLU gating, vs the fp32 reference over the same quantised weights."""
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops import reference as ref
    from vllm_neuron_b200.ops.mx_layout import atoms_to_scales, interleave_gate_up, untile_values

    torch.manual_seed(4)
    x = torch.randn(T, H, device="cuda").bfloat16()
    w13 = torch.randn(E, 2 * I, H, device="cuda") / H ** 0.5
    w2 = torch.randn(E, H, I, device="cuda") / I ** 0.5
    wts, ids = torch.topk(torch.softmax(torch.randn(T, E, device="cuda"), -1), k, -1)
    ids = ids.to(torch.int32)
    t13, s13, t2, s2 = ops.prepare_moe_mxfp8(w13, w2, interleaved=False)
    b13 = torch.zeros(E, 2 * I, device="cuda")
    b2 = torch.zeros(E, H, device="cuda")
    got = ops.moe_mxfp4(x, ids, wts, t13, s13, b13, t2, s2, b2, 0, 1.0, -1.0, H, I, fp4=False)
    w13q = ref.dequant_mxfp8(untile_values(t13, 2 * I, H, False).view(torch.float8_e4m3fn),
                             atoms_to_scales(s13, 2 * I, H))
    w2q = ref.dequant_mxfp8(untile_values(t2, H, I, False).view(torch.float8_e4m3fn), atoms_to_scales(s2, H, I))
    wref = interleave_gate_up(w13)
    assert (w13q - wref).norm() / wref.norm() < 0.04  # e4m3 with a power-of-two scale per 32
    want = ref.moe_experts(x, ids, wts, w13q, None, w2q, None, 1.0, None, True, 0, "silu")
    rel = (got.float() - want.float()).norm() / want.float().norm()
    assert rel < 0.08, rel  # activations are MXFP8-quantised inside the kernel (e4m3, 3 mantissa bits)
