"""Host and device memory queries (``utils/memory.py`` of the Trainium plugin): the host
figure honours a cgroup limit (containers), so weight staging never plans on memory the
container cannot use."""

from __future__ import annotations

import os


def _read_int(path: str) -> int | None:
    try:
        with open(path) as f:
            v = f.read().strip()
    except OSError:
        return None
    if v in ("max", ""):
        return None
    try:
        return int(v)
    except ValueError:
        return None


def cgroup_memory_limit(root: str = "/sys/fs/cgroup") -> int | None:
    """Memory limit of this process's cgroup in bytes (v2 ``memory.max`` or v1
    ``memory.limit_in_bytes``), None when unlimited."""
    lim = _read_int(os.path.join(root, "memory.max"))
    if lim is None:
        lim = _read_int(os.path.join(root, "memory", "memory.limit_in_bytes"))
    if lim is not None and lim >= 1 << 60:  # v1 "unlimited" sentinel
        return None
    return lim


def cgroup_memory_usage(root: str = "/sys/fs/cgroup") -> int | None:
    u = _read_int(os.path.join(root, "memory.current"))
    return u if u is not None else _read_int(os.path.join(root, "memory", "memory.usage_in_bytes"))


def meminfo_available(path: str = "/proc/meminfo") -> int:
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def get_available_memory_bytes(cgroup_root: str = "/sys/fs/cgroup", meminfo: str = "/proc/meminfo") -> int:
    avail = meminfo_available(meminfo)
    lim = cgroup_memory_limit(cgroup_root)
    if lim is not None:
        used = cgroup_memory_usage(cgroup_root) or 0
        avail = min(avail, max(0, lim - used)) if avail else max(0, lim - used)
    return avail


def device_memory(device=None) -> dict:
    import torch

    if not torch.cuda.is_available():
        return {"free": 0, "total": 0}
    free, total = torch.cuda.mem_get_info(device)
    return {"free": free, "total": total, "allocated": torch.cuda.memory_allocated(device),
            "reserved": torch.cuda.memory_reserved(device)}
