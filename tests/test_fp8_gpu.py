"""FP8 (e4m3) linear layers on the GPU: the tcgen05 kind::f8f6f4 GEMM of ``csrc/gemm.cu`` and
the quantisation kernels of ``csrc/fp8.cu`` against fp32 PyTorch references of the same ops;
then a static-FP8 (ModelOpt-format) Llama checkpoint through the engine on the GPU, scored
against the CPU fp32 engine (same quantisation, emulated) with teacher forcing."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _ext():
    from vllm_neuron_b200 import ops

    ops._k()  # load the extension (registers torch.ops.b200.*)


def _q(x, s):
    return (x.float() / s).clamp(-448, 448).to(torch.float8_e4m3fn)


@pytest.mark.parametrize("T", [1, 16, 64, 200, 2048])
@pytest.mark.parametrize("N,K", [(640, 2880), (5120, 2880), (2880, 4096), (256, 512)])
@pytest.mark.parametrize("per_channel", [False, True])
def test_gemm_fp8_matches_reference(T, N, K, per_channel):
    from vllm_neuron_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(T + N + K)
    x = torch.randn(T, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.05
    sx = (x.abs().amax() / 448).reshape(1)
    sw = (w.abs().amax(dim=1) / 448) if per_channel else (w.abs().amax() / 448).reshape(1)
    xq = _q(x, sx).to(DEV)
    wq = (w / sw.reshape(-1, 1)).clamp(-448, 448).to(torch.float8_e4m3fn).to(DEV)
    bias = (torch.randn(N, generator=g) * 0.1).bfloat16().to(DEV)
    alpha = (sx * sw).float().reshape(-1).to(DEV)
    y = torch.empty(T, N, dtype=torch.bfloat16, device=DEV)
    ws, cnt = ops._gemm_workspace(torch.device(DEV))
    torch.ops.b200.gemm_fp8(y, xq, wq, bias, alpha, ws, cnt, 16, ops.device_status(torch.device(DEV)))
    torch.cuda.synchronize()
    want = (xq.float() @ wq.float().t()) * alpha.reshape(1, -1) + bias.float()
    err = (y.float() - want).abs()
    assert (err > 1e-2 + 1e-2 * want.abs()).sum().item() == 0, f"max err {err.max().item()}"
    assert ops.check_device_status(torch.device(DEV)) == 0


@pytest.mark.parametrize("static", [True, False])
def test_fp8_quant_matches_torch(static):
    g = torch.Generator(device="cpu").manual_seed(1)
    x = (torch.randn(37, 1024, generator=g) * 3).bfloat16().to(DEV)
    s = torch.tensor([0.02], device=DEV) if static else None
    ws_ = torch.tensor([0.5, 2.0, 0.25], device=DEV)
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=DEV)
    alpha = torch.empty(3, device=DEV)
    amax = None if static else torch.empty(1, dtype=torch.int32, device=DEV)
    torch.ops.b200.fp8_quant(q, x, s, amax, ws_, alpha)
    torch.cuda.synchronize()
    sv = s if static else (x.float().abs().amax() / 448).reshape(1)
    want = _q(x, sv)
    assert torch.equal(q.view(torch.uint8), want.view(torch.uint8))
    assert torch.allclose(alpha, sv * ws_, rtol=1e-6)


def test_rms_norm_fp8_matches_reference():
    from vllm_neuron_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(19, 2880, generator=g).bfloat16().to(DEV)
    r = torch.randn(19, 2880, generator=g).bfloat16().to(DEV)
    w = (1 + 0.1 * torch.randn(2880, generator=g)).to(DEV)
    s = torch.tensor([0.01], device=DEV)
    r_want = (x.float() + r.float()).bfloat16()
    y = (r_want.float() * torch.rsqrt(r_want.float().pow(2).mean(-1, keepdim=True) + 1e-5) * w).bfloat16()
    want = _q(y, s)
    q, r_out = ops.rms_norm_fp8(x, w, 1e-5, s, r)
    torch.cuda.synchronize()
    assert torch.equal(r_out, r_want)
    diff = (q.float() - want.float()).abs()
    # an element exactly between two e4m3 values may round either way after fp32 reordering
    assert (diff > 0.13 * want.float().abs() + 1e-3).sum().item() == 0


def test_fp8_llama_engine_on_gpu_matches_cpu(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.testing import greedy_logit_gaps
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024,
                      tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).eval()
    sd = {}
    for k, v in m.state_dict().items():
        if k.endswith("proj.weight"):
            s = v.abs().amax() / 448
            sd[k] = (v / s).clamp(-448, 448).to(torch.float8_e4m3fn)
            sd[k.replace("weight", "weight_scale")] = s.reshape(())
            sd[k.replace("weight", "input_scale")] = torch.tensor(0.03)
        else:
            sd[k] = v.detach().clone().contiguous()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    d["quantization_config"] = {"quant_method": "modelopt", "quant_algo": "FP8"}
    path = str(tmp_path / "llama_fp8")
    save_state_dict(sd, path, d)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(1, 2000, (n,), generator=g).tolist() for n in (7, 60, 200)]
    kw = dict(model=path, max_model_len=512, max_num_seqs=4, max_num_batched_tokens=512, block_size=32)
    gpu = LLM(dtype="bfloat16", device="cuda", **kw)
    try:
        outs = gpu.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=12, ignore_eos=True))
        gen = [list(o.outputs[0].token_ids) for o in outs]
    finally:
        gpu.shutdown()
    cpu = LLM(dtype="float32", device="cpu", **kw)
    try:
        res = greedy_logit_gaps(cpu.engine, prompts, gen)
    finally:
        cpu.shutdown()
    assert res.outliers() <= res.n_tokens // 24, f"FP8 GPU tokens far from the CPU argmax: {res}"
    assert res.exact_fraction >= 0.75, f"too few exact matches: {res}"
