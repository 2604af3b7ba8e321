"""Host utilities: cgroup-aware memory, dtypes, vision block packing, golden cache, topology
parsing (CPU only)."""

import pytest
import torch


def test_cgroup_memory(tmp_path):
    from vllm_neuron_b200.utils.memory import get_available_memory_bytes

    cg = tmp_path / "cg"
    cg.mkdir()
    (cg / "memory.max").write_text(str(8 << 30))
    (cg / "memory.current").write_text(str(3 << 30))
    mi = tmp_path / "meminfo"
    mi.write_text("MemTotal: 100000000 kB\nMemAvailable: 50000000 kB\n")
    assert get_available_memory_bytes(str(cg), str(mi)) == 5 << 30
    (cg / "memory.max").write_text("max")
    assert get_available_memory_bytes(str(cg), str(mi)) == 50000000 * 1024


def test_dtypes():
    from vllm_neuron_b200.utils.dtype_utils import element_size, to_torch_dtype, ulp

    assert to_torch_dtype("bf16") is torch.bfloat16 and element_size("fp8") == 1
    assert ulp(1.0, torch.bfloat16) == 2 ** -7


def test_vision_packing():
    from vllm_neuron_b200.utils.vision_utils import pack_sequences

    lens = [900, 300, 700, 100, 2500, 64]
    blocks = pack_sequences(lens, 1024)
    assert sorted(i for b in blocks for i in b) == list(range(len(lens)))
    for b in blocks:
        assert len(b) == 1 or sum(lens[i] for i in b) <= 1024
    assert len(blocks) == 4


def test_golden_cache(tmp_path, monkeypatch):
    from vllm_neuron_b200.utils.golden_cache import get_or_compute, golden_key

    monkeypatch.setenv("VLLM_B200_GOLDEN_CACHE_DIR", str(tmp_path))
    calls = []
    k = golden_key(model="tiny", prompts=[[1, 2]])
    f = lambda: calls.append(1) or torch.arange(3)  # noqa: E731
    assert get_or_compute(k, f).tolist() == [0, 1, 2]
    assert get_or_compute(k, f).tolist() == [0, 1, 2] and len(calls) == 1


def test_topology_parse():
    from vllm_neuron_b200.utils.hardware_config import all_nvlink, parse_topology

    text = ("\tGPU0\tGPU1\tNIC0\tCPU Affinity\tNUMA Affinity\tGPU NUMA ID\n"
            "GPU0\t X \tNV18\tPIX\t0-55\t0\t\tN/A\n"
            "GPU1\tNV18\t X \tSYS\t56-111\t1\t\tN/A\n"
            "NIC0\tPIX\tSYS\t X \n")
    g = parse_topology(text)
    assert [x.index for x in g] == [0, 1] and g[0].peer_links == {1: "NV18"}
    assert g[0].nics == ["NIC0"] and g[1].nics == [] and g[0].numa_node == 0 and g[1].cpu_affinity == "56-111"
    assert all_nvlink(g)


def test_device_allocator_contiguous_and_reclaims(tmp_path):
    import json

    from vllm_neuron_b200.utils.device_allocator import DeviceAllocator

    state = str(tmp_path / "dev.json")
    with open(state, "w") as f:
        json.dump({"0": 2 ** 22 + 12345}, f)  # a dead owner: reclaimed
    a = DeviceAllocator(4, state)
    assert a.acquire(2) == [0, 1]
    b = DeviceAllocator(4, state)
    assert b.acquire(2) == [2, 3]
    with pytest.raises(TimeoutError):
        DeviceAllocator(4, state).acquire(1, timeout_s=0.2, poll_s=0.05)
    a.release()
    assert DeviceAllocator(4, state).acquire(2) == [0, 1]


def test_spec_decode_utils():
    import torch

    from vllm_neuron_b200.utils.spec_decode_utils import (compute_token_indices_to_sample, extract_next_token_ids,
                                                          replicate_per_seq_rows)

    last, cnt = extract_next_token_ids(torch.tensor([[10, 20, -1], [5, -1, -1], [7, 99999, 3]]), 32000)
    assert last.tolist() == [20, 5, 7] and cnt.tolist() == [2, 1, 1]
    last, cnt = extract_next_token_ids([[1, 2], [3]], 100)
    assert last.tolist() == [2, 3] and cnt.tolist() == [2, 1]
    idx = compute_token_indices_to_sample(torch.tensor([3, 7]), torch.tensor([3, 0]), torch.tensor([2, 1]))
    assert idx.tolist() == [1, 7]
    r = replicate_per_seq_rows(torch.tensor([[1.0, 2.0], [3.0, 4.0]]), 3)
    assert torch.equal(r, torch.tensor([[1.0, 2.0]] * 3 + [[3.0, 4.0]] * 3))


def test_kv_cache_dtype_names_and_fp8_bound():
    import torch

    from vllm_neuron_b200.utils.dtype_utils import FP8_CLAMP_MAX, kv_cache_dtype_str_to_dtype

    assert FP8_CLAMP_MAX == float(torch.finfo(torch.float8_e4m3fn).max)
    assert kv_cache_dtype_str_to_dtype("auto", torch.bfloat16) == torch.bfloat16
    assert kv_cache_dtype_str_to_dtype("fp8_e4m3", torch.bfloat16) == torch.float8_e4m3fn
    with pytest.raises(ValueError, match="unsupported kv_cache_dtype"):
        kv_cache_dtype_str_to_dtype("int4", torch.bfloat16)


def test_bind_to_gpu_numa_with_fake_sysfs(tmp_path):
    """NUMA pinning reads the GPU's PCI numa_node and the node's CPU list from sysfs (a fake
    tree here) and never widens the process's allowed CPUs."""
    import os

    from vllm_neuron_b200.utils.hardware_config import bind_to_gpu_numa, parse_cpulist, pci_numa_node

    assert parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    before = os.sched_getaffinity(0)
    bus = "0000:1b:00.0"
    (tmp_path / "bus/pci/devices" / bus).mkdir(parents=True)
    (tmp_path / "bus/pci/devices" / bus / "numa_node").write_text("1\n")
    (tmp_path / "devices/system/node/node1").mkdir(parents=True)
    allowed = sorted(before)
    (tmp_path / "devices/system/node/node1/cpulist").write_text(f"{allowed[0]},{max(allowed) + 1000}\n")
    assert pci_numa_node(bus, str(tmp_path)) == 1
    try:
        cpus = bind_to_gpu_numa(0, bus, str(tmp_path))
        assert cpus == {allowed[0]} and os.sched_getaffinity(0) == {allowed[0]}
    finally:
        for tid in os.listdir("/proc/self/task"):
            try:
                os.sched_setaffinity(int(tid), before)
            except OSError:
                pass
    (tmp_path / "bus/pci/devices" / bus / "numa_node").write_text("-1\n")
    assert bind_to_gpu_numa(0, bus, str(tmp_path)) is None and os.sched_getaffinity(0) == before


def test_device_offset_moves_every_rank(monkeypatch):
    """VLLM_B200_DEVICE_OFFSET shifts the GPU of every rank (rank r -> GPU offset + r)."""
    from vllm_neuron_b200.config import EngineConfig
    from vllm_neuron_b200.engine.worker import Worker

    cfg = EngineConfig.create(model=None, device="cpu")
    assert Worker(cfg, rank=1, world_size=4, local_rank=1).device_index == 1
    monkeypatch.setenv("VLLM_B200_DEVICE_OFFSET", "4")
    assert Worker(cfg, rank=1, world_size=4, local_rank=1).device_index == 5


def test_cross_node_loopback_master_addr_refused(monkeypatch):
    """Several nodes (LOCAL_WORLD_SIZE below the world size) with a loopback MASTER_ADDR are
    refused before any rendezvous; one node, or a routable address, passes."""
    from vllm_neuron_b200.parallel.state import validate_master_addr

    monkeypatch.setenv("LOCAL_WORLD_SIZE", "4")
    monkeypatch.setenv("MASTER_ADDR", "127.0.0.1")
    with pytest.raises(ValueError, match="loopback"):
        validate_master_addr(8)
    validate_master_addr(4)  # one node
    validate_master_addr(8, "file:///tmp/x")  # not an env:// rendezvous
    monkeypatch.setenv("MASTER_ADDR", "10.1.2.3")
    validate_master_addr(8)


def _quick(ready):
    ready.set()


def _ignores_sigterm(ready):
    import signal
    import time

    signal.signal(signal.SIGTERM, signal.SIG_IGN)
    ready.set()
    time.sleep(60)


def _sleeps(ready):
    import time

    ready.set()
    time.sleep(60)


def test_stop_workers_escalates_to_sigkill():
    """A worker that exits is joined; one that hangs gets SIGTERM; one that ignores SIGTERM is
    killed after the termination timeout."""
    import multiprocessing as mp
    import time

    from vllm_neuron_b200.engine.llm import stop_workers

    ctx = mp.get_context("spawn")
    events = [ctx.Event() for _ in range(3)]
    procs = [ctx.Process(target=f, args=(e,), daemon=True) for f, e in zip((_quick, _sleeps, _ignores_sigterm), events)]
    for p in procs:
        p.start()
    assert all(e.wait(60) for e in events)
    procs[0].join(30)
    t0 = time.monotonic()
    assert stop_workers(procs, grace_s=1.0, term_timeout_s=1.0) == ["exited", "terminated", "killed"]
    assert time.monotonic() - t0 < 15 and not any(p.is_alive() for p in procs)
