"""KV-cache connector for disaggregated inference (1 prefill engine, 1 decode engine).

Counterpart of the Trainium plugin's NIXL connector (``vllm/kv_connector/neuron_nixl_connector.py``)
for engines on one host.  Protocol (vLLM's ``kv_transfer_params``):

* the prefill engine (``kv_role`` producer) gets a request with
  ``{"do_remote_decode": True}``; when the request finishes (the proxy asks for one token)
  its prompt KV is exported before the blocks are freed, and the request output carries
  ``{"do_remote_prefill": True, "transfer_id", "num_tokens", "remote_tp_size", "remote_engine_id"}``;
* the decode engine (``kv_role`` consumer) gets the request with those params; at admission
  it allocates blocks for the whole prompt, loads the KV of positions ``[0, num_tokens - 1)``
  and computes only the last prompt token itself (that step samples the first output token).

Transport ``HostStagedConnector``: each producer rank writes its KV heads of the request (raw
cache dtype, so the transfer is byte-exact) to one file in a shared store directory
(``kv_connector_extra_config.store_path``, default a directory under /dev/shm), atomically
renamed into place; consumer ranks read the files of every producer rank and take the
global kv heads they own, so producer and consumer may use different TP degrees (the
reference's head-ratio mapping).  A consumer waits for the files at most ``timeout_s``
(``kv_connector_extra_config.timeout_s``, default 30 s); a missing or malformed transfer
raises :class:`KVTransferError`, and the engine aborts that request instead of blocking.  The
producer removes its exports after ``ttl_s`` (default 600 s).
"""

from __future__ import annotations

import os
import time

import torch

from ..logging_config import init_logger

logger = init_logger(__name__)


class KVTransferError(RuntimeError):
    pass


class HostStagedConnector:
    def __init__(self, kv_caches: list, kv_head_range: tuple[int, int], block_size: int, rank: int, tp_size: int,
                 engine_id: str, role: str, extra: dict | None = None):
        extra = extra or {}
        self.store = extra.get("store_path") or os.path.join("/dev/shm" if os.path.isdir("/dev/shm") else "/tmp",
                                                             "vllm_b200_kv")
        os.makedirs(self.store, exist_ok=True)
        self.timeout_s = float(extra.get("timeout_s", 30.0))
        self.ttl_s = float(extra.get("ttl_s", 600.0))  # exported transfers older than this are removed
        # decode -> prefill exports of multi-turn chats live shorter: the next turn either comes
        # soon or never, and every export holds host (/dev/shm) or pool memory meanwhile
        self.return_ttl_s = float(extra.get("return_ttl_s", 60.0))
        self.cleanup_on_shutdown = bool(extra.get("cleanup_on_shutdown", False))
        self.kv = kv_caches
        self.h0, self.nh = kv_head_range
        self.bs = block_size
        self.rank, self.tp = rank, tp_size
        self.engine_id = engine_id
        self.role = role
        self.extra = extra
        self.exported: list[tuple[str, float]] = []  # (transfer id, expiry time)
        self.stats = {"exported": 0, "loaded": 0, "failed": 0, "bytes": 0}

    @property
    def is_producer(self) -> bool:
        return self.role in ("kv_producer", "kv_both")

    @property
    def is_consumer(self) -> bool:
        return self.role in ("kv_consumer", "kv_both")

    def _path(self, transfer_id: str, rank: int) -> str:
        return os.path.join(self.store, f"{transfer_id}.rank{rank}.pt")

    def _layers(self):
        return [(i, kv) for i, kv in enumerate(self.kv) if kv is not None]

    # ----------------------------------------------------------------- producer
    def export(self, request_id: str, block_ids: list[int], num_tokens: int, ttl_s: float | None = None) -> dict:
        """Write this rank's KV of positions [0, num_tokens) and return the params the
        decode engine needs.  The export is removed after ``ttl_s`` (default: the
        connector's ``ttl_s``) unless read earlier."""
        tid = f"{self.engine_id}-{request_id}"
        self._gc()
        nb = -(-num_tokens // self.bs)
        idx = torch.tensor(block_ids[:nb], dtype=torch.long, device=self.kv[self._layers()[0][0]][0].device)
        layers = {}
        for i, (kc, vc) in self._layers():
            k = kc.index_select(0, idx).permute(0, 2, 1, 3).reshape(nb * self.bs, kc.shape[1], kc.shape[3])
            v = vc.index_select(0, idx).permute(0, 2, 1, 3).reshape(nb * self.bs, vc.shape[1], vc.shape[3])
            layers[i] = (k[:num_tokens].cpu().contiguous(), v[:num_tokens].cpu().contiguous())
            self.stats["bytes"] += layers[i][0].numel() * layers[i][0].element_size() * 2
        tmp = self._path(tid, self.rank) + f".tmp{os.getpid()}"
        torch.save({"num_tokens": num_tokens, "heads": (self.h0, self.nh), "layers": layers}, tmp)
        os.replace(tmp, self._path(tid, self.rank))
        self.exported.append((tid, time.monotonic() + (self.ttl_s if ttl_s is None else ttl_s)))
        self.stats["exported"] += 1
        return {"do_remote_prefill": True, "transfer_id": tid, "num_tokens": num_tokens,
                "remote_tp_size": self.tp, "remote_engine_id": self.engine_id}

    # ----------------------------------------------------------------- consumer
    def load(self, params: dict, block_ids: list[int], num_tokens: int) -> None:
        """Write the remote KV of positions [0, num_tokens) into this engine's blocks."""
        tid = params.get("transfer_id")
        ptp = int(params.get("remote_tp_size", 1))
        if not tid:
            raise KVTransferError("kv_transfer_params without transfer_id")
        deadline = time.monotonic() + self.timeout_s
        paths = [self._path(tid, r) for r in range(ptp)]
        while not all(os.path.exists(p) for p in paths):
            if time.monotonic() > deadline:
                self.stats["failed"] += 1
                raise KVTransferError(f"KV transfer {tid} not available after {self.timeout_s:.1f}s")
            time.sleep(0.002)
        parts = [torch.load(p, weights_only=False) for p in paths]
        if any(pt["num_tokens"] < num_tokens for pt in parts):
            raise KVTransferError(f"KV transfer {tid} holds fewer than {num_tokens} tokens")
        pos = torch.arange(num_tokens)
        blk = torch.tensor(block_ids, dtype=torch.long)[pos // self.bs]
        off = pos % self.bs
        for i, (kc, vc) in self._layers():
            ks, vs = [], []
            for h in range(self.h0, self.h0 + self.nh):  # global kv head -> the part that holds it
                src = next((pt for pt in parts if pt["heads"][0] <= h < pt["heads"][0] + pt["heads"][1]), None)
                if src is None or i not in src["layers"]:
                    raise KVTransferError(f"KV transfer {tid}: no data for layer {i} kv head {h}")
                j = h - src["heads"][0]
                ks.append(src["layers"][i][0][:num_tokens, j])
                vs.append(src["layers"][i][1][:num_tokens, j])
            k = torch.stack(ks, 1).to(kc.device, kc.dtype)
            v = torch.stack(vs, 1).to(vc.device, vc.dtype)
            kc[blk.to(kc.device), :, off.to(kc.device)] = k
            vc[blk.to(vc.device), :, off.to(vc.device)] = v
        self.stats["loaded"] += 1

    def _gc(self) -> None:
        now = time.monotonic()
        keep = []
        for tid, t in self.exported:
            if now > t:
                try:
                    os.remove(self._path(tid, self.rank))
                except OSError:
                    pass
            else:
                keep.append((tid, t))
        self.exported = keep

    def cleanup(self) -> None:
        """Engine shutdown: remove this rank's exports if configured (otherwise they stay
        for a decode engine that has not read them yet, until ``ttl_s`` on a later run)."""
        if not self.cleanup_on_shutdown:
            return
        for tid, _ in self.exported:
            try:
                os.remove(self._path(tid, self.rank))
            except OSError:
                pass
        self.exported = []


class B200IpcConnector(HostStagedConnector):
    """Device-to-device transport for engines on one host (``csrc/kv_transfer.cu``).

    Every producer rank owns a device pool (``pool_mb``, default 1024 MB) shared by CUDA IPC;
    its handle is published once in the store directory.  ``export`` gathers the request's KV
    of positions [0, num_tokens) from the paged cache into a free range of the pool (one
    kernel), waits for it, and writes a small metadata file (offset, tokens, heads, layers).
    ``load`` maps the producer ranks' pools (once per producer rank), copies the rows of the
    kv heads this rank owns straight into its blocks (one kernel, peer loads), waits for it and
    leaves an acknowledgement file; the producer reuses a pool range once it is acknowledged
    or older than ``ttl_s``.  When the pool has no free range, or either side runs on the CPU,
    the transfer falls back to the host-staged files of :class:`HostStagedConnector` (the
    params carry the transport)."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        from ..ops import _ext

        _ext.load()
        layers = self._layers()
        kc0 = self.kv[layers[0][0]][0]
        self.device = kc0.device
        self.row_bytes = kc0.shape[3] * kc0.element_size()
        self.kptr = torch.tensor([kc.data_ptr() for _, (kc, _) in layers], dtype=torch.int64, device=self.device)
        self.vptr = torch.tensor([vc.data_ptr() for _, (_, vc) in layers], dtype=torch.int64, device=self.device)
        self.layer_ids = [i for i, _ in layers]
        self.pool = None
        self.pool_bytes = int(float(self.extra.get("pool_mb", 1024)) * (1 << 20)) // 256 * 256
        self.ranges: list[tuple[str, int, int, float]] = []  # (transfer id, offset, size, expiry)
        self._peers: dict[tuple[str, int], int] = {}
        from ..ops import device_status

        self.status = device_status(self.device)
        if self.is_producer and self.pool_bytes > 0:
            ops = torch.ops.b200
            # comm_alloc(n) allocates a 64 KB header + 2 n bytes; the pool starts after the header
            self.pool = ops.comm_alloc(self.pool_bytes // 2 + 256)
            self.pool0 = self.pool + 64 * 1024
            h = ops.ipc_get_handle(self.pool).numpy().tobytes()
            tmp = self._pool_path(self.engine_id, self.rank) + f".tmp{os.getpid()}"
            with open(tmp, "wb") as f:
                f.write(h)
            os.replace(tmp, self._pool_path(self.engine_id, self.rank))

    def _pool_path(self, engine_id: str, rank: int) -> str:
        return os.path.join(self.store, f"{engine_id}.rank{rank}.pool")

    def _meta_path(self, tid: str, rank: int) -> str:
        return os.path.join(self.store, f"{tid}.rank{rank}.ipc")

    def _ack_path(self, tid: str, rank: int) -> str:
        return os.path.join(self.store, f"{tid}.rank{rank}.ack")

    # ----------------------------------------------------------------- producer
    def _reserve(self, need: int) -> int | None:
        """First-fit range of the pool after dropping acknowledged / expired ranges."""
        now = time.monotonic()
        keep = []
        for tid, off, size, t in self.ranges:
            if os.path.exists(self._ack_path(tid, self.rank)) or now > t:
                for p in (self._ack_path(tid, self.rank), self._meta_path(tid, self.rank)):
                    try:
                        os.remove(p)
                    except OSError:
                        pass
            else:
                keep.append((tid, off, size, t))
        self.ranges = sorted(keep, key=lambda r: r[1])
        cur = 0
        for _, off, size, _ in self.ranges:
            if off - cur >= need:
                return cur
            cur = off + size
        return cur if self.pool_bytes - cur >= need else None

    def export(self, request_id: str, block_ids: list[int], num_tokens: int, ttl_s: float | None = None) -> dict:
        need = (2 * len(self.layer_ids) * num_tokens * self.nh * self.row_bytes + 255) // 256 * 256
        off = self._reserve(need) if self.pool is not None else None
        if off is None:
            return {**super().export(request_id, block_ids, num_tokens, ttl_s), "transport": "host"}
        tid = f"{self.engine_id}-{request_id}"
        nb = -(-num_tokens // self.bs)
        blocks = torch.tensor(block_ids[:nb], dtype=torch.int32, device=self.device)
        torch.ops.b200.kv_export(self.pool0 + off, self.kptr, self.vptr, blocks, num_tokens, self.nh,
                                 self.row_bytes, self.bs)
        torch.cuda.current_stream(self.device).synchronize()  # the consumer reads from another process
        self.ranges.append((tid, off, need, time.monotonic() + (self.ttl_s if ttl_s is None else ttl_s)))
        meta = {"offset": off, "num_tokens": num_tokens, "heads": (self.h0, self.nh), "layers": self.layer_ids,
                "row_bytes": self.row_bytes}
        tmp = self._meta_path(tid, self.rank) + f".tmp{os.getpid()}"
        torch.save(meta, tmp)
        os.replace(tmp, self._meta_path(tid, self.rank))
        self.stats["exported"] += 1
        self.stats["bytes"] += need
        return {"do_remote_prefill": True, "transfer_id": tid, "num_tokens": num_tokens,
                "remote_tp_size": self.tp, "remote_engine_id": self.engine_id, "transport": "ipc"}

    # ----------------------------------------------------------------- consumer
    def _peer(self, engine_id: str, rank: int, deadline: float) -> int:
        key = (engine_id, rank)
        if key not in self._peers:
            path = self._pool_path(engine_id, rank)
            while not os.path.exists(path):
                if time.monotonic() > deadline:
                    raise KVTransferError(f"no KV pool published by {engine_id} rank {rank}")
                time.sleep(0.002)
            with open(path, "rb") as f:
                h = f.read()
            self._peers[key] = torch.ops.b200.ipc_open_handle(torch.frombuffer(bytearray(h), dtype=torch.uint8))
        return self._peers[key]

    def load(self, params: dict, block_ids: list[int], num_tokens: int) -> None:
        if params.get("transport") != "ipc" or self.device.type != "cuda":
            return super().load(params, block_ids, num_tokens)
        tid = params.get("transfer_id")
        ptp = int(params.get("remote_tp_size", 1))
        eng = params.get("remote_engine_id")
        if not tid or not eng:
            raise KVTransferError("kv_transfer_params without transfer_id / remote_engine_id")
        deadline = time.monotonic() + self.timeout_s
        paths = [self._meta_path(tid, r) for r in range(ptp)]
        while not all(os.path.exists(p) for p in paths):
            if time.monotonic() > deadline:
                self.stats["failed"] += 1
                raise KVTransferError(f"KV transfer {tid} not available after {self.timeout_s:.1f}s")
            time.sleep(0.002)
        metas = [torch.load(p, weights_only=False) for p in paths]
        for m in metas:
            if m["num_tokens"] < num_tokens or m["layers"] != self.layer_ids or m["row_bytes"] != self.row_bytes:
                raise KVTransferError(f"KV transfer {tid}: layout does not match this engine")
        need_heads = range(self.h0, self.h0 + self.nh)
        if not all(any(m["heads"][0] <= h < m["heads"][0] + m["heads"][1] for m in metas) for h in need_heads):
            raise KVTransferError(f"KV transfer {tid}: kv heads {self.h0}..{self.h0 + self.nh - 1} missing")
        bases = [self._peer(eng, r, deadline) + 64 * 1024 + m["offset"] for r, m in enumerate(metas)]
        if any(m["num_tokens"] != metas[0]["num_tokens"] for m in metas):
            raise KVTransferError(f"KV transfer {tid}: producer ranks disagree on the token count")
        nb = -(-num_tokens // self.bs)
        blocks = torch.tensor(block_ids[:nb], dtype=torch.int32, device=self.device)
        torch.ops.b200.kv_import(bases, [m["heads"][0] for m in metas], [m["heads"][1] for m in metas], self.kptr,
                                 self.vptr, blocks, num_tokens, metas[0]["num_tokens"], self.h0, self.nh,
                                 self.row_bytes, self.bs, self.status)
        torch.cuda.current_stream(self.device).synchronize()  # the producer may reuse the range after the ack
        for r in range(ptp):
            with open(self._ack_path(tid, r), "w"):
                pass
        self.stats["loaded"] += 1
        self.stats["bytes"] += sum(2 * len(self.layer_ids) * num_tokens * m["heads"][1] * self.row_bytes
                                   for m in metas)

    def cleanup(self) -> None:
        super().cleanup()
        ops = torch.ops.b200
        try:
            torch.cuda.synchronize(self.device)
            for p in self._peers.values():
                ops.ipc_close(p)
            self._peers = {}
            if self.pool is not None:
                ops.comm_free(self.pool)
                self.pool = None
        except Exception:  # noqa: BLE001
            pass


class DecodeBenchConnector:
    """Decode-only benchmarking (the reference's ``NeuronDecodeBenchConnector``,
    ``vllm/kv_connector/neuron_decode_bench_connector.py``): every request is admitted as if
    its prompt had been prefilled elsewhere, so the engine runs no prefill and the first step of
    a request is a one-token decode.  ``load`` writes normal noise (``fill_mean``, ``fill_std``;
    default 0, 1) into the request's cache blocks on the device so attention reads finite values;
    the decode cost does not depend on the values.  ``fill: false`` leaves the blocks as they
    are."""

    prefill_all = True
    is_producer = False
    is_consumer = True

    def __init__(self, kv_caches: list, block_size: int, extra: dict | None = None):
        extra = extra or {}
        self.kv = kv_caches
        self.bs = block_size
        self.fill = bool(extra.get("fill", True))
        self.mean = float(extra.get("fill_mean", 0.0))
        self.std = float(extra.get("fill_std", 1.0))
        self.stats = {"exported": 0, "loaded": 0, "failed": 0, "bytes": 0}

    def export(self, request_id: str, block_ids: list[int], num_tokens: int, ttl_s: float | None = None) -> dict:
        return {}

    def load(self, params: dict, block_ids: list[int], num_tokens: int) -> None:
        self.stats["loaded"] += 1
        if not self.fill or num_tokens <= 0:
            return
        nb = -(-num_tokens // self.bs)
        for kv in self.kv:
            if not isinstance(kv, tuple):
                continue
            for c in kv:
                idx = torch.tensor(block_ids[:nb], dtype=torch.long, device=c.device)
                noise = torch.randn((nb,) + tuple(c.shape[1:]), device=c.device) * self.std + self.mean
                c.index_copy_(0, idx, noise.to(c.dtype))

    def cleanup(self) -> None:
        return None


def make_connector(cfg, runner, rank: int, tp_size: int, kv_head_range: tuple[int, int]):
    kt = cfg.kv_transfer_config
    if kt is None:
        return None
    name = kt.kv_connector
    extra = dict(kt.kv_connector_extra_config or {})
    if name in ("DecodeBenchConnector", "NeuronDecodeBenchConnector"):
        return DecodeBenchConnector(runner.kv_caches, cfg.block_size, extra)
    if name not in ("B200IpcConnector", "HostStagedConnector", "NixlConnector", "NeuronNixlConnector"):
        raise ValueError(f"unsupported kv_connector {name!r}")
    engine_id = extra.get("engine_id") or f"eng{os.getpid()}"
    kv0 = next((kv for kv in runner.kv_caches if kv is not None), None)
    on_gpu = kv0 is not None and kv0[0].is_cuda
    # the NIXL names select the device transport: same-host engines, peer memory instead of
    # a network fabric
    cls = B200IpcConnector if (on_gpu and name != "HostStagedConnector") else HostStagedConnector
    return cls(runner.kv_caches, kv_head_range, cfg.block_size, rank, tp_size, engine_id, kt.kv_role, extra)
