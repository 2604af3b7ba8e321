"""MLA decode (absorbed multi-head latent attention) on the GPU: the tcgen05 kernel of
``csrc/mla_decode.cu`` against the fp32 PyTorch reference of the same op
(``ops.reference.attention.mla_decode``), over head counts that take each head-tile width
(16 / 32 / 64 and two 64-head groups), block sizes, ragged sequence lengths, split-KV and a
peaked score distribution that exercises the lazy rescaling of O.  Cache slots the sequences
do not use hold NaN, so a key past a sequence's end that leaked into the softmax or P.V would
show."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _ext():
    from vllm_neuron_b200 import ops

    ops._k()


def _case(B, Hq, bs, lens, q_scale, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    max_blocks = max(1, max(-(-n // bs) for n in lens))
    num_blocks = B * max_blocks + 3
    cache = torch.full((num_blocks, bs, 576), float("nan"), dtype=torch.bfloat16)
    perm = torch.randperm(num_blocks, generator=g)[: B * max_blocks].reshape(B, max_blocks).to(torch.int32)
    for b, n in enumerate(lens):
        for t in range(n):
            cache[perm[b, t // bs], t % bs] = (torch.randn(576, generator=g) * 0.5).bfloat16()
    q = (torch.randn(B, Hq, 576, generator=g) * q_scale).bfloat16()
    return (q.to(DEV), cache.to(DEV), perm.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV))


@pytest.mark.parametrize("B,Hq,bs,lens,splits,q_scale", [
    (3, 16, 64, [1, 129, 700], 1, 1.0),
    (4, 64, 32, [128, 256, 1000, 77], 1, 1.0),
    (4, 64, 32, [128, 256, 1000, 77], 3, 1.0),
    (2, 128, 16, [300, 2048], 4, 1.0),
    (2, 8, 128, [5, 513], 2, 1.0),
    (3, 32, 64, [640, 0, 33], 2, 1.0),
    (2, 16, 32, [1500, 900], 1, 6.0),
])
def test_mla_decode_matches_fp32_reference(B, Hq, bs, lens, splits, q_scale):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.reference.attention import mla_decode as ref_mla

    q, cache, bt, sl = _case(B, Hq, bs, lens, q_scale, seed=B * 131 + Hq + bs + splits)
    scale = 192 ** -0.5
    out = ops.mla_decode(q, cache, bt, sl, scale, num_splits=splits)
    torch.cuda.synchronize()
    assert ops.check_device_status(q.device) == 0
    want = ref_mla(q.cpu(), cache.cpu(), bt.cpu(), sl.cpu(), scale).float()
    got = out.float().cpu()
    assert torch.isfinite(got).all(), "non-finite output"
    err = (got - want).abs()
    tol = 2e-2 + 2e-2 * want.abs()
    assert (err > tol).sum().item() == 0, f"max err {err.max().item():.4g}"


def test_mla_decode_default_splits_and_repeat():
    """The wrapper's own split count, twice in a row (the kernel keeps no state between calls)."""
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.reference.attention import mla_decode as ref_mla

    q, cache, bt, sl = _case(8, 16, 64, [2048, 1, 100, 4000, 128, 129, 257, 1024], 1.0, seed=7)
    want = ref_mla(q.cpu(), cache.cpu(), bt.cpu(), sl.cpu(), 0.1).float()
    for _ in range(2):
        got = ops.mla_decode(q, cache, bt, sl, 0.1).float().cpu()
        assert ((got - want).abs() > 2e-2 + 2e-2 * want.abs()).sum().item() == 0
