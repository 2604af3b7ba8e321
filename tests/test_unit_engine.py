"""Block manager (prefix caching), scheduler policy and request lifecycle."""

from vllm_neuron_b200.engine.block_manager import KVCacheManager
from vllm_neuron_b200.engine.request import Request, RequestStatus
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.engine.scheduler import Scheduler


def _req(i, n, max_tokens=4):
    return Request(f"r{i}", list(range(100 * i, 100 * i + n)), SamplingParams(temperature=0, max_tokens=max_tokens))


def test_block_allocation_and_free():
    kv = KVCacheManager(16, 4)
    r = _req(0, 10)
    assert kv.allocate_slots(r, 10)
    assert len(r.block_ids) == 3 and 0 not in r.block_ids
    free_before = kv.pool.num_free
    kv.free(r)
    assert kv.pool.num_free == free_before + 3


def test_prefix_cache_hit_and_eviction():
    kv = KVCacheManager(16, 4, enable_caching=True)
    a = Request("a", list(range(13)), SamplingParams())
    assert kv.allocate_slots(a, 13)
    a.num_computed_tokens = 13
    kv.cache_full_blocks(a)
    blocks_a = list(a.block_ids)
    kv.free(a)
    b = Request("b", list(range(12)) + [99, 98], SamplingParams())
    hit, n = kv.get_computed_blocks(b)
    assert n == 12 and hit == blocks_a[:3]
    b.num_computed_tokens = n
    assert kv.allocate_slots(b, 2, hit)
    assert b.block_ids[:3] == blocks_a[:3]
    # a prompt fully covered by cached blocks recomputes its last block
    c = Request("c", list(range(12)), SamplingParams())
    hit, n = kv.get_computed_blocks(c)
    assert n == 8


def test_scheduler_prefill_decode_separation_and_finish():
    kv = KVCacheManager(64, 4)
    s = Scheduler(kv, max_num_seqs=4, max_num_batched_tokens=16, max_model_len=64, max_num_prefills_per_step=1)
    r0, r1 = _req(0, 10, 2), _req(1, 20, 2)
    s.add_request(r0)
    s.add_request(r1)
    o = s.schedule()
    assert o.kind == "prefill" and [x.req_id for x in o.seqs] == ["r0"]
    s.update_from_output(o, {"r0": [7]})
    o = s.schedule()  # r1 prefill (segment 1 of 2): decode held back
    assert o.kind == "prefill" and o.seqs[0].req_id == "r1" and len(o.seqs[0].token_ids) == 16
    assert not o.seqs[0].sample
    s.update_from_output(o, {})
    o = s.schedule()
    assert o.kind == "prefill" and len(o.seqs[0].token_ids) == 4 and o.seqs[0].sample
    s.update_from_output(o, {"r1": [5]})
    o = s.schedule()
    assert o.kind == "decode" and {x.req_id for x in o.seqs} == {"r0", "r1"}
    done = s.update_from_output(o, {"r0": [8], "r1": [6]})
    assert {d.request_id for d in done} == {"r0", "r1"}
    assert all(d.status == RequestStatus.FINISHED_LENGTH for d in done)
    assert not s.has_unfinished()
    assert kv.pool.num_free == 63


def test_kv_admission_control():
    kv = KVCacheManager(9, 4)  # 8 usable blocks; max_model_len 16 -> 4 blocks each -> 2 concurrent
    s = Scheduler(kv, max_num_seqs=8, max_num_batched_tokens=64, max_model_len=16, max_num_prefills_per_step=4)
    for i in range(3):
        s.add_request(_req(i, 4, 8))
    o = s.schedule()
    assert len(o.seqs) == 2  # third request deferred by admission control


def test_stop_conditions():
    r = Request("x", [1, 2], SamplingParams(max_tokens=10, stop_token_ids=[42]), eos_token_id=7)
    r.output_token_ids = [3]
    assert not r.check_stop(100)
    r.output_token_ids.append(7)
    assert r.check_stop(100) and r.status == RequestStatus.FINISHED_STOPPED
    r2 = Request("y", [1], SamplingParams(max_tokens=10, ignore_eos=True), eos_token_id=7)
    r2.output_token_ids = [7]
    assert not r2.check_stop(100)
    r2.output_token_ids.append(42)
    assert not r2.check_stop(100)
