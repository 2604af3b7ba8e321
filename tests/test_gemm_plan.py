"""The dense GEMM planner's decisions (host code of ``csrc/gemm.cu``, no GPU needed): token tile
widths that balance the last wave on 148 SMs, narrow tiles before a global-atomic K split, and
the cluster split for decode widths."""

import pytest
import torch


@pytest.fixture(scope="module")
def plan():
    from vllm_neuron_b200.ops import _ext

    if not _ext.load():
        pytest.skip("extension not built")
    return lambda T, N, K: list(torch.ops.b200.gemm_plan(T, N, K, 16, 148))


@pytest.mark.parametrize("T,N,K,nt", [
    (2048, 2880, 2048, 192),  # 256-token tiles: 184 tiles, the second wave a quarter full
    (2048, 5120, 2880, 192),
    (4096, 2880, 2880, 224),
    (1, 128, 64, 16),
])
def test_wide_tiles_balance_the_last_wave(plan, T, N, K, nt):
    width, tiles, splits, cluster, _ = plan(T, N, K)
    assert width == nt and splits == 1 and cluster == 0, (width, tiles, splits, cluster)


def test_narrower_tiles_before_an_atomic_k_split(plan):
    # 46 tiles of 256 tokens would split K three ways through global atomics; 92 tiles of 128 do not
    width, tiles, splits, cluster, _ = plan(512, 2880, 2048)
    assert (width, tiles, splits, cluster) == (128, 92, 1, 0)


def test_decode_width_splits_k_across_a_cluster(plan):
    width, tiles, splits, cluster, sps = plan(64, 2880, 4096)
    assert width == 64 and tiles == 23 and cluster == 1 and splits > 1
    assert splits * sps <= 64  # every K stage covered once: 4096 / 64 stages
