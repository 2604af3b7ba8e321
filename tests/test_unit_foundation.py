"""Unit tests of pure host-side logic: config schema, buckets, group rank math."""

import pytest

from vllm_neuron_b200.config import EngineConfig, NeuronConfig, OnDeviceSamplingConfig, VisionNeuronConfig
from vllm_neuron_b200.parallel import state as ps
from vllm_neuron_b200.utils import bucket_utils as bu


def test_neuron_config_keys_and_defaults():
    nc = NeuronConfig.from_dict({"ep_degree": 8, "on_device_sampling_config": {"max_top_k": 128, "all_greedy": "true"},
                                 "num_seqs_buckets": [1, 8, 64], "quantization": "mxfp4",
                                 "tensor_capture": {"modules": ["model.layers.0"]}})
    assert nc.ep_degree == 8 and nc.on_device_sampling_config.max_top_k == 128
    assert nc.on_device_sampling_config.all_greedy is True
    assert nc.tensor_capture.modules == ["model.layers.0"]
    assert NeuronConfig.from_dict({"on_device_sampling_config": None}).on_device_sampling_config is None
    assert isinstance(NeuronConfig().on_device_sampling_config, OnDeviceSamplingConfig)
    with pytest.raises(ValueError):
        NeuronConfig.from_dict({"ep_degree": 0})
    with pytest.raises(ValueError):
        NeuronConfig.from_dict({"not_a_key": 1})


def test_engine_config_validation():
    cfg = EngineConfig.create(tensor_parallel_size=8, additional_config={"neuron_config": {"ep_degree": 8}})
    assert cfg.world_size == 8
    with pytest.raises(ValueError):
        EngineConfig.create(tensor_parallel_size=6, additional_config={"neuron_config": {"ep_degree": 4}})
    with pytest.raises(ValueError):
        EngineConfig.create(block_size=24)
    with pytest.raises(TypeError):
        EngineConfig.create(bogus=1)
    with pytest.raises(ValueError):
        EngineConfig.create(async_scheduling=True, speculative_config={"num_speculative_tokens": 2})


def test_vision_tp_dp():
    assert VisionNeuronConfig(dp_size=2).resolve_tp_dp(8) == (4, 2)
    with pytest.raises(ValueError):
        VisionNeuronConfig(tp_size=3, dp_size=2).resolve_tp_dp(8)


def test_buckets():
    assert bu.get_default_num_batched_tokens_buckets(2048) == [128, 256, 512, 1024, 2048]
    assert bu.get_default_num_batched_tokens_buckets(3000) == [128, 256, 512, 1024, 2048, 3000]
    assert bu.get_default_num_seqs_buckets(8) == [1, 2, 4, 8]
    assert bu.get_default_num_seqs_buckets(6) == [1, 2, 4, 6]
    assert bu.get_bucket_for_count(5, [1, 2, 4, 8]) == 8
    with pytest.raises(ValueError):
        bu.get_bucket_for_count(9, [1, 2, 4, 8])
    assert bu.validate_buckets("x", [8, 1, 4], 16) == [1, 4, 8, 16]
    with pytest.raises(ValueError):
        bu.validate_buckets("x", [32], 16)
    seg = bu.resolve_segmented_prefill_config(4096, 8192)
    assert seg.enabled and seg.segment_size == 4096
    assert not bu.resolve_segmented_prefill_config(8192, 8192).enabled
    assert bu.next_power_of_2(5) == 8


def test_group_rank_math():
    rows, cols = ps.build_ep_group_ranks(8, 2)
    assert rows == [[0, 1, 2, 3], [4, 5, 6, 7]] and cols == [[0, 4], [1, 5], [2, 6], [3, 7]]
    a2a, gather = ps.build_sampling_dp_meshes(8, 2)
    assert a2a == [[0, 1], [2, 3], [4, 5], [6, 7]] and gather == [[0, 2, 4, 6], [1, 3, 5, 7]]
    assert ps.build_component_tp_group_ranks(64, 8, 4) == [list(range(32)), list(range(32, 64))]
    cols = ps.build_dp_column_group_ranks(32, 8, 4)
    assert cols[0] == [0, 8, 16, 24] and cols[7] == [7, 15, 23, 31]
    assert ps.build_inter_node_peer_group_ranks(16, 2)[3] == [3, 11]
    kv, heads = ps.build_dcp_group_ranks(8, 8, 2)
    assert kv == [[0, 1], [2, 3], [4, 5], [6, 7]] and heads == [[0, 2, 4, 6], [1, 3, 5, 7]]
    with pytest.raises(ValueError):
        ps.build_component_tp_group_ranks(16, 8, 4)


def test_kv_head_sharding():
    from vllm_neuron_b200.models.base import kv_head_sharding

    assert kv_head_sharding(8, 8, 3) == (3, 1)
    assert kv_head_sharding(8, 2, 1) == (4, 4)
    assert kv_head_sharding(2, 8, 5) == (1, 1)  # replicated: ranks 4..7 hold head 1


def test_single_rank_parallel_state():
    st = ps.initialize_parallel_state()
    assert st.tp.world_size == 1 and st.tp.all_reduce is not None
    ps.destroy_parallel_state()


def test_attention_backend_spec():
    from vllm_neuron_b200.ops.metadata import AttentionMetadata, B200AttentionBackend as B
    from vllm_neuron_b200.platform import B200Platform

    assert B.get_kv_cache_shape(10, 32, 8, 64) == (2, 10, 8, 32, 64)  # K/V x HND
    assert B.get_metadata_cls() is AttentionMetadata
    B.validate(32, 128)
    with pytest.raises(ValueError):
        B.validate(24, 64)
    with pytest.raises(ValueError):
        B.validate(32, 96)
    assert B200Platform.get_attn_backend_cls() == "vllm_neuron_b200.ops.metadata.B200AttentionBackend"


def test_component_dp_group_math():
    assert ps.build_component_dp_group_ranks(8, 2, 2) == [[0, 2], [1, 3], [4, 6], [5, 7]]
    assert ps.build_component_dp_group_ranks(4, 1, 4) == [[0, 1, 2, 3]]
