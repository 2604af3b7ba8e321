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
