"""Host hardware description (``utils/hardware_config.py`` of the Trainium plugin, which maps
Trainium instances to EFA NICs and NUMA nodes).

On a GPU host the equivalent facts come from ``nvidia-smi topo -m`` (read-only): per GPU,
its CPU affinity, NUMA node and the NICs on its PCIe switch (``PIX`` / ``PXB``), which is
what a disaggregated-serving deployment pins its transfer threads and NICs by; plus the
GPU-to-GPU link type (``NV18`` = 18 NVLink 5 links through NVSwitch).  ``parse_topology``
works on the command's text, so it is testable without a GPU.
"""

from __future__ import annotations

import re
import subprocess
from dataclasses import dataclass, field


@dataclass
class GpuTopo:
    index: int
    cpu_affinity: str = ""
    numa_node: int | None = None
    nics: list = field(default_factory=list)  # NICs on the GPU's PCIe switch
    peer_links: dict = field(default_factory=dict)  # gpu index -> link type (e.g. "NV18")


def parse_topology(text: str) -> list[GpuTopo]:
    lines = [l.rstrip() for l in text.splitlines() if l.strip()]
    if not lines:
        return []
    cols = [c.strip() for c in lines[0].split("\t") if c.strip()]
    gpus: list[GpuTopo] = []
    for line in lines[1:]:
        parts = [p.strip() for p in line.split("\t")]
        name, vals = parts[0], parts[1:]
        m = re.fullmatch(r"GPU(\d+)", name)
        if not m:
            continue
        g = GpuTopo(int(m.group(1)))
        for c, v in zip(cols, vals):
            if re.fullmatch(r"GPU\d+", c) and c != name:
                g.peer_links[int(c[3:])] = v
            elif re.fullmatch(r"(NIC|mlx|eth|ib)\S*", c) and v in ("PIX", "PXB"):
                g.nics.append(c)
            elif c == "CPU Affinity":
                g.cpu_affinity = v
            elif c == "NUMA Affinity" and v.isdigit():
                g.numa_node = int(v)
        gpus.append(g)
    return gpus


def detect() -> list[GpuTopo]:
    try:
        out = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True, timeout=20).stdout
    except (OSError, subprocess.TimeoutExpired):
        return []
    return parse_topology(out)


def all_nvlink(gpus: list[GpuTopo]) -> bool:
    return bool(gpus) and all(v.startswith("NV") for g in gpus for v in g.peer_links.values())


# ---------------------------------------------------------------- CPU affinity per rank
# The reference pins each worker's threads to the NUMA node of its NIC
# (``vllm/worker/neuron_worker.py:261-344``).  Here the anchor is the rank's GPU: its PCI
# device's ``numa_node`` in sysfs, whose CPU list is intersected with the CPUs the process may
# already use (a container's cpuset), so pinning never widens what the process may run on.

def parse_cpulist(text: str) -> set[int]:
    """Linux CPU list syntax ("0-3,8,10-11") -> set of CPU ids."""
    out: set[int] = set()
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-", 1)
            out.update(range(int(lo), int(hi) + 1))
        else:
            out.add(int(part))
    return out


def gpu_pci_bus_id(device_index: int) -> str | None:
    """``dddd:bb:dd.f`` of a CUDA device, lower case (None without CUDA)."""
    try:
        import torch

        p = torch.cuda.get_device_properties(device_index)
        return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except Exception:  # noqa: BLE001
        return None


def pci_numa_node(pci_bus_id: str, sysfs: str = "/sys") -> int | None:
    try:
        with open(f"{sysfs}/bus/pci/devices/{pci_bus_id.lower()}/numa_node") as f:
            n = int(f.read().strip())
    except (OSError, ValueError):
        return None
    return n if n >= 0 else None


def numa_cpus(node: int, sysfs: str = "/sys") -> set[int]:
    try:
        with open(f"{sysfs}/devices/system/node/node{node}/cpulist") as f:
            return parse_cpulist(f.read())
    except OSError:
        return set()


def bind_to_gpu_numa(device_index: int, pci_bus_id: str | None = None, sysfs: str = "/sys") -> set[int] | None:
    """Pin every thread of this process to the CPUs of the GPU's NUMA node (within the current
    allowed set).  Returns the CPUs, or None when the node or an overlap is unknown (nothing
    changed)."""
    import os

    bus = pci_bus_id or gpu_pci_bus_id(device_index)
    node = pci_numa_node(bus, sysfs) if bus else None
    if node is None:
        return None
    cpus = numa_cpus(node, sysfs) & os.sched_getaffinity(0)
    if not cpus:
        return None
    try:
        tids = [int(t) for t in os.listdir("/proc/self/task")]
    except OSError:
        tids = [0]
    for tid in tids:
        try:
            os.sched_setaffinity(tid, cpus)
        except OSError:
            pass  # the thread exited meanwhile
    return cpus
