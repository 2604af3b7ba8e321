"""Per-step execution: input preparation, model forward, sampling.

Counterpart of the Trainium plugin's ``NeuronModelRunner``
(``vllm_neuron/vllm/worker/neuron_model_runner.py:378``), designed for CUDA:
* inputs (token ids, positions, slot mapping, block tables, sequence lengths,
  sampling parameters) are assembled with numpy in pinned host buffers and copied
  to persistent device buffers with one async H2D copy each;
* decode steps replay a CUDA graph captured per ``num_seqs_buckets`` batch size
  (the counterpart of the reference's per-bucket NEFFs) covering model forward,
  LM head and sampling; the graph's only host traffic is the inputs and the
  sampled token ids;
* prefill steps (including segmented prefill and prefix-cache hits) run eagerly
  over the flat token batch; attention reads prior context from the paged cache;
* the KV cache is one (K, V) pair of ``[num_blocks, kv_heads, block_size, head_dim]``
  tensors per layer (HND, ``vllm/attention/attn.py:27-35``).
"""

from __future__ import annotations

import dataclasses
import hashlib
import math
import struct
import time
from dataclasses import dataclass

import numpy as np
import torch

from .. import envs
from ..config import EngineConfig
from ..logging_config import init_logger
from ..metrics import GRAPH_REPLAY_COUNT, NUM_SEQS_PADDING
from ..nn.sampler import Sampler
from ..ops.metadata import AttentionMetadata, B200AttentionBackend
from ..utils.bucket_utils import get_bucket_for_count, get_default_num_seqs_buckets, validate_buckets
from .scheduler import SchedulerOutput

logger = init_logger(__name__)


def request_uniform(seed: int, req_id: str, seq: int) -> float:
    """Deterministic U[0,1) per (seed, request, sample index), identical on every rank."""
    h = hashlib.blake2b(f"{seed}:{req_id}:{seq}".encode(), digest_size=8).digest()
    return (struct.unpack("<Q", h)[0] >> 11) * (1.0 / (1 << 53))


def decode_splits(batch: int, kv_heads: int, sms: int, cap: int = 32) -> int:
    """Largest power of two ``s`` with ``batch * kv_heads * s <= 4 * sms`` (at least 1)."""
    want = max(1, (4 * sms) // max(1, batch * kv_heads))
    return int(min(cap, 1 << (want.bit_length() - 1)))


@dataclass
class _GraphEntry:
    graph: torch.cuda.CUDAGraph
    batch: int


class _DoneEvent:
    def synchronize(self) -> None:
        return None


@dataclass
class AsyncStep:
    """A launched decode step whose sampled ids are still being copied to the host."""

    so: SchedulerOutput
    n_sel: int
    host: torch.Tensor
    event: object
    row_of: dict


class ModelRunner:
    def __init__(self, cfg: EngineConfig, model: torch.nn.Module, device: torch.device, tp_group,
                 vocab_size: int, cp_group=None, sampling_groups=None):
        self.cfg = cfg
        self.model = model
        self.device = device
        self.bs = cfg.block_size
        # decode context parallelism: a virtual block of bs * cp tokens is dealt to the cp
        # ranks bs tokens each (token t on rank (t // bs) % cp, at local index
        # (t // (bs * cp)) * bs + t % bs of the block)
        self.cp_group = cp_group if (cp_group is not None and cp_group.world_size > 1) else None
        self.cp = self.cp_group.world_size if self.cp_group is not None else 1
        self.cp_rank = self.cp_group.rank_in_group if self.cp_group is not None else 0
        self.vbs = self.bs * self.cp
        self.max_model_len = cfg.max_model_len
        self.max_blocks = math.ceil(cfg.max_model_len / self.vbs)
        nc = cfg.neuron_config
        buckets = nc.num_seqs_buckets or nc.decode_batch_buckets
        self.decode_buckets = (validate_buckets("num_seqs_buckets", buckets, cfg.max_num_seqs) if buckets
                               else get_default_num_seqs_buckets(cfg.max_num_seqs))
        ods = nc.on_device_sampling_config
        self.max_top_k = ods.max_top_k if ods is not None else 256
        self.all_greedy_cfg = bool(ods and ods.all_greedy)
        lm = model.lm_head
        self.tp_group = tp_group
        # lm_head DP: the head is sharded over a TP x DP supergroup and the rows to sample
        # are gathered over its DP ranks (``_sample_lm_dp``); the sampler reduces over the
        # supergroup
        self.lm_dp = getattr(lm, "dp_group", None)
        # attention DP: the model runs on the tokens of every replica of its supergroup
        # (gathered here), attention per replica inside the model
        self.adp = getattr(model, "attention_dp", None)
        self.sampler = Sampler(lm.group if self.lm_dp is not None else tp_group, lm.start, vocab_size,
                               self.max_top_k, sampling_groups)
        self.use_graphs = (device.type == "cuda" and not cfg.enforce_eager and not envs.VLLM_B200_DISABLE_CUDA_GRAPHS)
        self.kv_caches: list[tuple[torch.Tensor, torch.Tensor]] = []
        self.num_blocks = 0
        self.graphs: dict[tuple[int, bool], _GraphEntry] = {}
        self.graph_pool = None
        self.seed = cfg.seed
        T = max(cfg.max_num_batched_tokens, cfg.max_num_seqs * (1 + self._num_spec()))
        B = max(cfg.max_num_seqs, 1)
        self.max_tokens = T
        pin = device.type == "cuda"
        mk = lambda shape, dt: torch.zeros(shape, dtype=dt, pin_memory=pin)  # noqa: E731
        # pinned host staging buffers
        self.h_ids = mk(T, torch.int64)
        self.h_pos = mk(T, torch.int64)
        self.h_slot = mk(T, torch.int64)
        self.h_qsl = mk(B + 1, torch.int32)
        self.h_seqlen = mk(B, torch.int32)
        self.h_bt = mk((B, self.max_blocks), torch.int32)
        self.h_lidx = mk(B * (1 + self._num_spec()), torch.int64)
        self.h_temp = mk(B, torch.float32)
        self.h_topk = mk(B, torch.int32)
        self.h_topp = mk(B, torch.float32)
        self.h_unif = mk(B, torch.float32)
        self.h_out = mk(B * (1 + self._num_spec()), torch.int64)
        # persistent device buffers (graph inputs)
        d = device
        self.d_ids = torch.zeros(T, dtype=torch.int64, device=d)
        self.d_pos = torch.zeros(T, dtype=torch.int64, device=d)
        self.d_slot = torch.full((T,), -1, dtype=torch.int64, device=d)
        self.d_qsl = torch.zeros(B + 1, dtype=torch.int32, device=d)
        self.d_seqlen = torch.zeros(B, dtype=torch.int32, device=d)
        self.d_bt = torch.zeros(B, self.max_blocks, dtype=torch.int32, device=d)
        self.d_lidx = torch.zeros(B * (1 + self._num_spec()), dtype=torch.int64, device=d)
        self.d_temp = torch.zeros(B, dtype=torch.float32, device=d)
        self.d_topk = torch.zeros(B, dtype=torch.int32, device=d)
        self.d_topp = torch.ones(B, dtype=torch.float32, device=d)
        self.d_unif = torch.zeros(B, dtype=torch.float32, device=d)
        self.d_out = torch.zeros(B * (1 + self._num_spec()), dtype=torch.int64, device=d)
        # sliding-window KV group (set up by initialize_kv_cache when the windowed layers get
        # their own, smaller block pool): its block table and slot mapping
        self.swa_blocks = 0
        self.h_bt_swa = self.h_slot_swa = self.d_bt_swa = self.d_slot_swa = None
        # asynchronous decode: input rows taken from the previous step's sampled ids, and two
        # host buffers so one step's D2H never overwrites the ids being read for the last one
        self.h_src = mk(B, torch.int64)
        self.d_src = torch.zeros(B, dtype=torch.int64, device=d)
        self.h_out_async = [mk(B, torch.int64), mk(B, torch.int64)]
        self._parity = 0
        self._h2d_done = None
        # per verified position (speculative decoding with sampling)
        P = B * (1 + self._num_spec())
        self.h_pos_params = mk((6, P), torch.float32)  # temp, top_k, top_p, draft, u_accept, u_sample
        self.d_pos_params = torch.zeros(6, P, dtype=torch.float32, device=d)
        self.workspace: torch.Tensor | None = None
        self.encoder_cache = None
        if hasattr(model, "embed_multimodal"):
            from .encoder_cache import EncoderCache

            vc = model.vl_cfg.vision
            nd = len(vc.deepstack_visual_indexes)
            ecfg = cfg.vision_neuron_config
            nblk = ecfg.encoder_cache_num_blocks or min(64, max(4, cfg.max_num_seqs))
            blk_tok = ecfg.max_vision_seq_len or 4096
            self.encoder_cache = EncoderCache(nblk, blk_tok, model.cfg.hidden_size * (1 + nd), model.dtype, device)
        # recurrent-state slots (hybrid linear-attention models): one slot per running
        # request plus a scratch slot for decode padding rows
        self.state_caches: list | None = None
        self.slot_of: dict[str, int] = {}
        if hasattr(model, "get_state_spec"):
            S = cfg.max_num_seqs + 1
            self.state_caches = []
            for sp in model.get_state_spec():
                if sp is None:
                    self.state_caches.append(None)
                    continue
                (C, K1), (hv, dk, dv) = sp
                self.state_caches.append((torch.zeros(S, C, K1, dtype=model.dtype, device=device),
                                          torch.zeros(S, hv, dk, dv, dtype=torch.float32, device=device)))
            self.free_slots = list(range(S - 2, -1, -1))
            self.scratch_slot = S - 1
            self.h_sslot = mk(B, torch.int32)
            self.h_sinit = mk(B, torch.int32)
            self.d_sslot = torch.zeros(B, dtype=torch.int32, device=d)
            self.d_sinit = torch.zeros(B, dtype=torch.int32, device=d)
        self.h2d_bytes_last = 0
        self.debug_logits = None
        if nc.debug_logits_dir:
            if self.lm_dp is not None:
                raise NotImplementedError("debug_logits_dir with lm_head data parallelism")
            from .debug_logits import DebugLogitsWriter

            self.debug_logits = DebugLogitsWriter(nc.debug_logits_dir, self.sampler.group, vocab_size)
        self.d2h_bytes_last = 0
        self.step_count = 0
        # optional device timing of every step: a list that receives one (start, end) pair of
        # CUDA events per step, recorded around the step's GPU work (H2D staging, forward,
        # sampling, D2H enqueue); None = off.  Benchmarks sum the spans for the device time
        # of a serving window without the host gaps between steps.
        self.step_spans: list | None = None
        # accuracy tooling: tensor capture / replacement hooks (eager steps only)
        self.capture = self.replacer = None
        rank = tp_group.rank_in_group if hasattr(tp_group, "rank_in_group") else 0
        if nc.tensor_capture is not None and nc.tensor_capture.modules:
            from ..accuracy.tensor_capture import TensorCapture

            tc = nc.tensor_capture
            self.capture = TensorCapture(model, tc.modules, tc.capture_dir, rank, tc.capture_filter)
            self.use_graphs = False
        if nc.tensor_replacement is not None:
            from ..accuracy.tensor_replacement import TensorReplacer

            tensors, _ = nc.tensor_replacement.resolve()
            self.replacer = TensorReplacer(model, tensors)
            self.use_graphs = False

    def release_state(self, req_id: str) -> None:
        """Return a request's recurrent-state slot (request finished or preempted)."""
        s = self.slot_of.pop(req_id, None)
        if s is not None:
            self.free_slots.append(s)

    def _slot_for(self, req_id: str) -> int:
        s = self.slot_of.get(req_id)
        if s is None:
            if not self.free_slots:
                raise RuntimeError("no free recurrent-state slot (more running requests than max_num_seqs)")
            s = self.free_slots.pop()
            self.slot_of[req_id] = s
        return s

    def _num_spec(self) -> int:
        sc = self.cfg.speculative_config
        return sc.num_speculative_tokens if sc is not None else 0

    # ------------------------------------------------------------------ KV cache
    def initialize_kv_cache(self, num_blocks: int, swa_blocks: int = 0) -> None:
        """KV caches of every attention layer: ``num_blocks`` blocks, or ``swa_blocks`` for the
        sliding-window layers when they form their own KV group (``swa_blocks`` > 0)."""
        spec = self.model.get_kv_spec()
        self.kv_caches = []
        self.swa_blocks = swa_blocks
        if swa_blocks:
            T, B = self.max_tokens, max(self.cfg.max_num_seqs, 1)
            pin = self.device.type == "cuda"
            self.h_bt_swa = torch.zeros((B, self.max_blocks), dtype=torch.int32, pin_memory=pin)
            self.h_slot_swa = torch.zeros(T, dtype=torch.int64, pin_memory=pin)
            self.d_bt_swa = torch.zeros(B, self.max_blocks, dtype=torch.int32, device=self.device)
            self.d_slot_swa = torch.full((T,), -1, dtype=torch.int64, device=self.device)
        for l in spec.layers:
            if l.kind != "attention":
                self.kv_caches.append(self.state_caches[len(self.kv_caches)] if self.state_caches else None)
                continue
            nb = swa_blocks if (swa_blocks and l.sliding_window) else num_blocks
            shape = B200AttentionBackend.get_kv_cache_shape(nb, self.bs, l.num_kv_heads, l.head_dim)[1:]
            self.kv_caches.append((torch.zeros(shape, dtype=l.dtype, device=self.device),
                                   torch.zeros(shape, dtype=l.dtype, device=self.device)))
        self.num_blocks = num_blocks
        # split-KV decode scratch: [B, Hq_local, splits, d + 2] fp32 partials
        hq = max((getattr(layer, "self_attn", None).nq if hasattr(layer, "self_attn") else 0)
                 for layer in getattr(self.model, "layers", [])) if hasattr(self.model, "layers") else 0
        d = max((l.head_dim for l in spec.layers), default=64)
        if self.device.type == "cuda" and hq:
            # with DCP every rank attends the query heads of its whole DCP group
            self.workspace = torch.empty(self.cfg.max_num_seqs * max(hq, 1) * self.cp * self.max_splits(1) * (d + 2),
                                         dtype=torch.float32, device=self.device)
        self._hq = hq

    def max_splits(self, batch: int) -> int:
        return 32

    def num_splits_for(self, batch: int) -> int:
        """Split-KV factor: the largest power of two with batch x kv_heads x splits CTAs at
        most about four per SM (the decode kernel keeps 3-4 resident), so a single long
        sequence is spread over the whole GPU while a full batch runs in one wave.  A power
        of two divides the cache-block count of a typical context evenly; on B200 at
        64 sequences x 2048 keys it measured 8 (one kv head) and 1 (eight kv heads) as the
        fastest factors, where the rounded-up quotient picked 10 and 2."""
        if self.device.type != "cuda":
            return 1
        spec = self.model.get_kv_spec()
        hkv = max(1, max(l.num_kv_heads for l in spec.layers if l.kind == "attention"))
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return decode_splits(batch, hkv, sms, self.max_splits(batch))

    # ------------------------------------------------------------------ inputs
    def _fill_sampling(self, so: SchedulerOutput, B: int) -> bool:
        n = len(so.seqs)
        temp, topk, topp, unif = (self.h_temp.numpy(), self.h_topk.numpy(), self.h_topp.numpy(),
                                  self.h_unif.numpy())
        all_greedy = True
        for i, s in enumerate(so.seqs):
            sp = s.sampling_params
            if sp is None or self.all_greedy_cfg or sp.temperature <= 0:
                temp[i] = 0.0
                topk[i] = 0
                topp[i] = 1.0
                unif[i] = 0.0
                continue
            all_greedy = False
            temp[i] = sp.temperature
            topk[i] = sp.top_k if sp.top_k > 0 else 0
            topp[i] = sp.top_p
            unif[i] = request_uniform(self.seed if sp.seed is None else sp.seed, s.req_id, s.sample_seq)
        if B > n:
            temp[n:B] = 0
            topk[n:B] = 0
            topp[n:B] = 1
            unif[n:B] = 0
        return all_greedy

    def _fill_spec_sampling(self, so: SchedulerOutput, n_sel: int) -> None:
        """Per verified position: the request's sampling parameters, the draft token to
        verify (-1 at the bonus position) and two deterministic uniforms."""
        hp = self.h_pos_params.numpy()
        j = 0
        for i, s in enumerate(so.seqs):
            k = len(s.token_ids)
            drafts = list(s.spec_token_ids) + [-1]
            seed = self.seed if s.sampling_params is None or s.sampling_params.seed is None else \
                s.sampling_params.seed
            for p in range(k):
                hp[0, j] = self.h_temp[i]
                hp[1, j] = self.h_topk[i]
                hp[2, j] = self.h_topp[i]
                hp[3, j] = drafts[p] if p < len(drafts) else -1
                hp[4, j] = request_uniform(seed, f"{s.req_id}/accept{p}", s.sample_seq)
                hp[5, j] = request_uniform(seed, f"{s.req_id}/sample{p}", s.sample_seq)
                j += 1
        self.d_pos_params[:, :n_sel].copy_(self.h_pos_params[:, :n_sel], non_blocking=True)

    def _prepare(self, so: SchedulerOutput, pad_to: int | None,
                 pad_tokens: int | None = None) -> tuple[AttentionMetadata, int, int, bool]:
        if self._h2d_done is not None:  # an asynchronous step may still be reading the staging buffers
            self._h2d_done.synchronize()
            self._h2d_done = None
        seqs = so.seqs
        n = len(seqs)
        B = pad_to or n
        n_real_tok = sum(len(s.token_ids) for s in seqs)
        pad_seq = pad_tokens is not None and pad_tokens > n_real_tok
        if pad_seq:  # one padding sequence (no KV write, not sampled) brings T to pad_tokens
            B = n + 1
        ids = self.h_ids.numpy()
        pos = self.h_pos.numpy()
        slot = self.h_slot.numpy()
        qsl = self.h_qsl.numpy()
        sl = self.h_seqlen.numpy()
        bt = self.h_bt.numpy()
        lidx = self.h_lidx.numpy()
        swa = self.swa_blocks > 0
        if swa:
            bt_s, slot_s = self.h_bt_swa.numpy(), self.h_slot_swa.numpy()
        t = 0
        qsl[0] = 0
        max_q, max_s = 1, 1
        n_sel = 0
        mm_rows: list = []
        has_mrope = False
        bs, vbs, cp, cpr = self.bs, self.vbs, self.cp, self.cp_rank
        plain_decode = so.kind == "decode" and all(len(x.token_ids) == 1 for x in seqs)
        for i, s in enumerate(seqs):
            k = len(s.token_ids)
            req = s.request
            nb = len(s.block_ids)
            # block-table entries past a sequence's own blocks are never read (its length
            # bounds every kernel), so rows are not cleared
            bt[i, :nb] = s.block_ids
            sl[i] = s.seq_len
            sw_ids = s.swa_block_ids if s.swa_block_ids is not None else s.block_ids
            if swa:
                bt_s[i, :len(sw_ids)] = sw_ids
            if plain_decode:  # one token: scalar work only
                p0 = s.start_pos
                ids[t] = s.token_ids[0]
                delta = req.mrope_delta if req is not None else 0
                pos[t] = p0 + delta
                slot[t] = s.block_ids[p0 // vbs] * bs + p0 % bs if (p0 // bs) % cp == cpr else -1
                if swa:
                    slot_s[t] = sw_ids[p0 // bs] * bs + p0 % bs
                lidx[n_sel] = t
                n_sel += 1
                t += 1
                qsl[i + 1] = t
                max_s = max(max_s, s.seq_len)
                continue
            ids[t:t + k] = s.token_ids
            p = np.arange(s.start_pos, s.start_pos + k)
            delta = req.mrope_delta if req is not None else 0
            dec_seq = so.kind == "decode" or (so.kind == "mixed" and i < so.num_decode)
            pos[t:t + k] = p + delta if (delta and dec_seq) else p
            if req is not None and req.mrope_positions is not None and not dec_seq:
                has_mrope = True
            blocks = np.asarray(s.block_ids, dtype=np.int64)
            if swa:
                slot_s[t:t + k] = np.asarray(sw_ids, dtype=np.int64)[p // bs] * bs + p % bs
            if cp == 1:
                slot[t:t + k] = blocks[p // bs] * bs + p % bs
            else:  # only the owning DCP rank writes a token
                slot[t:t + k] = np.where((p // bs) % cp == cpr, blocks[p // vbs] * bs + p % bs, -1)
            if so.kind == "decode" and s.spec_token_ids:
                lidx[n_sel:n_sel + k] = np.arange(t, t + k)
                n_sel += k
            else:
                lidx[n_sel] = t + k - 1
                n_sel += 1
            t += k
            qsl[i + 1] = t
            max_q = max(max_q, k)
            max_s = max(max_s, s.seq_len)
        T = t
        if pad_seq:
            k = pad_tokens - T
            ids[T:T + k] = 0
            pos[T:T + k] = np.arange(k)
            slot[T:T + k] = -1
            sl[n] = k
            bt[n] = 0
            if swa:
                slot_s[T:T + k] = -1
                bt_s[n] = 0
            qsl[n + 1] = T + k
            max_q, max_s = max(max_q, k), max(max_s, k)
            T += k
        elif B > n:  # decode padding rows: no KV write, no keys
            ids[T:T + (B - n)] = 0
            pos[T:T + (B - n)] = 0
            slot[T:T + (B - n)] = -1
            sl[n:B] = 0
            bt[n:B] = 0
            if swa:
                slot_s[T:T + (B - n)] = -1
                bt_s[n:B] = 0
            for j in range(n, B):
                qsl[j + 1] = qsl[j] + 1
                lidx[n_sel] = T + (j - n)
                n_sel += 1
            T += B - n
        greedy = self._fill_sampling(so, B)
        spec = so.kind == "decode" and any(s.spec_token_ids for s in seqs)
        extras_so = self._grammar_mask(seqs, n_sel) if not spec else None
        if spec and not greedy:
            self._fill_spec_sampling(so, n_sel)
        extras = self._mm_extras(so) if (has_mrope and self.encoder_cache is not None) else {}
        if self.state_caches is not None:
            hs, hi = self.h_sslot.numpy(), self.h_sinit.numpy()
            for i, s in enumerate(seqs):
                real = s.request is not None
                hs[i] = self._slot_for(s.req_id) if real else self.scratch_slot
                hi[i] = 1 if (s.start_pos > 0 or not real) else 0
            hs[n:B] = self.scratch_slot
            hi[n:B] = 1
            self.d_sslot[:B].copy_(self.h_sslot[:B], non_blocking=True)
            self.d_sinit[:B].copy_(self.h_sinit[:B], non_blocking=True)
            extras["state_slots"] = self.d_sslot[:B]
            extras["state_init"] = self.d_sinit[:B]
        # H2D: one async copy per buffer from pinned memory
        nb_ = 0
        for h, dv, cnt in ((self.h_ids, self.d_ids, T), (self.h_pos, self.d_pos, T), (self.h_slot, self.d_slot, T),
                           (self.h_qsl, self.d_qsl, B + 1), (self.h_seqlen, self.d_seqlen, B),
                           (self.h_lidx, self.d_lidx, n_sel), (self.h_temp, self.d_temp, B),
                           (self.h_topk, self.d_topk, B), (self.h_topp, self.d_topp, B),
                           (self.h_unif, self.d_unif, B)):
            dv[:cnt].copy_(h[:cnt], non_blocking=True)
            nb_ += cnt * h.element_size()
        max_nb = max(1, max(math.ceil(s.seq_len / vbs) for s in seqs)) if seqs else 1
        if pad_seq:
            max_nb = max(max_nb, math.ceil(int(sl[n]) / vbs))
        self.d_bt[:B, :max_nb].copy_(self.h_bt[:B, :max_nb], non_blocking=True)
        nb_ += B * max_nb * 4
        if swa:
            self.d_bt_swa[:B, :max_nb].copy_(self.h_bt_swa[:B, :max_nb], non_blocking=True)
            self.d_slot_swa[:T].copy_(self.h_slot_swa[:T], non_blocking=True)
            nb_ += B * max_nb * 4 + T * 8
        self.h2d_bytes_last = nb_
        meta = AttentionMetadata(
            num_tokens=T, num_seqs=B, is_decode=(so.kind == "decode" and max_q == 1),
            query_start_loc=self.d_qsl[:B + 1], seq_lens=self.d_seqlen[:B], block_tables=self.d_bt[:B],
            slot_mapping=self.d_slot[:T], logits_indices=self.d_lidx[:n_sel], max_query_len=max_q,
            max_seq_len=max_s, workspace=self.workspace, num_splits=self.num_splits_for(B), extras=extras,
            cp_group=self.cp_group, block_tables_swa=self.d_bt_swa[:B] if swa else None,
            slot_mapping_swa=self.d_slot_swa[:T] if swa else None,
            num_decode_seqs=so.num_decode if so.kind == "mixed" else 0)
        if spec:
            extras["spec"] = True
        if extras_so is not None:
            extras["token_bitmask"] = extras_so
        if not spec:
            lp = [s.request.sampling_params.logprobs for s in seqs
                  if s.request is not None and s.request.sampling_params.logprobs is not None]
            if lp:
                extras["logprobs_k"] = max(lp)
        if self.debug_logits is not None:
            extras["debug_logits"] = True
        return meta, T, n_sel, greedy

    def _grammar_mask(self, seqs, n_sel: int) -> torch.Tensor | None:
        """Packed allowed-token bitmask [n_sel, words] of this step's sampled rows (one row per
        sequence, in order; rows of unconstrained sequences and padding allow everything), or
        None when no sequence carries a grammar.  A mask set by the caller in
        ``external_bitmask`` (an outer engine's grammar, already in this layout) is used once."""
        ext = self.__dict__.pop("external_bitmask", None)
        if ext is not None:
            return ext.to(self.device, non_blocking=True)
        if not any(s.request is not None and s.request.grammar is not None for s in seqs):
            return None
        from .structured_output import fill_bitmask

        matchers = [s.request.grammar if s.request is not None else None for s in seqs]
        matchers += [None] * (n_sel - len(matchers))
        return fill_bitmask(matchers[:n_sel], self.sampler.vocab_size).to(self.device)

    def _mm_extras(self, so: SchedulerOutput) -> dict:
        """Multimodal inputs of a prefill step: image rows from the encoder cache (encoding
        images on first use), their token indices, and [3, T] multimodal positions."""
        model = self.model
        H = model.cfg.hidden_size
        # every image this step needs that is not cached yet: one batched (block-packed,
        # vision-DP) encoder pass; every rank runs the same step, so the collectives match
        todo = []
        for s in so.seqs:
            req = s.request
            if req is None or req.mrope_positions is None:
                continue
            k = len(s.token_ids)
            for it_i, it in enumerate(req.mm_items or []):
                if max(s.start_pos, it["offset"]) < min(s.start_pos + k, it["offset"] + it["n"]) and \
                        not self.encoder_cache.has(req.request_id, it_i):
                    todo.append((req.request_id, it_i, it["pixels"]))
        if todo:
            with torch.inference_mode():
                if hasattr(model, "embed_images"):
                    fats = model.embed_images([px for _, _, px in todo])
                else:
                    fats = []
                    for _, _, px in todo:
                        mm = model.embed_multimodal(px)
                        fats.append(torch.cat([mm["embeds"]] + list(mm["deepstack"]), dim=-1))
            for (rid, it_i, _), fat in zip(todo, fats):
                self.encoder_cache.put(rid, it_i, fat)
        p3_parts, idx, rows = [], [], []
        t = 0
        for s in so.seqs:
            k = len(s.token_ids)
            req = s.request
            p = torch.arange(s.start_pos, s.start_pos + k)
            if req is not None and req.mrope_positions is not None:
                P = req.mrope_positions
                inside = p < P.shape[1]
                col = torch.where(inside[None], P[:, p.clamp(max=P.shape[1] - 1)], (p + req.mrope_delta)[None])
                p3_parts.append(col)
                for it_i, it in enumerate(req.mm_items or []):
                    lo = max(s.start_pos, it["offset"])
                    hi = min(s.start_pos + k, it["offset"] + it["n"])
                    if lo >= hi:
                        continue
                    r = torch.arange(lo - it["offset"], hi - it["offset"], device=self.device)
                    rows.append(self.encoder_cache.gather(req.request_id, it_i, r))
                    idx.append(torch.arange(t + lo - s.start_pos, t + hi - s.start_pos))
            else:
                p3_parts.append(p[None].expand(3, k))
            t += k
        ex = {"mrope_positions": torch.cat(p3_parts, dim=1).to(self.device)}
        if rows:
            fat = torch.cat(rows)
            nd = (fat.shape[1] // H) - 1
            ex["mm_embeds"] = fat[:, :H]
            ex["deepstack"] = [fat[:, (j + 1) * H:(j + 2) * H] for j in range(nd)]
            ex["mm_index"] = torch.cat(idx).to(self.device)
        return ex

    # ------------------------------------------------------------------ forward
    def _sp_ok(self, meta: AttentionMetadata, T: int) -> bool:
        g = self.tp_group
        return (not meta.is_decode and g.world_size > 1 and self.adp is None and T > g.world_size and T % g.world_size == 0
                and envs.VLLM_B200_SEQUENCE_PARALLEL and not getattr(self.model, "aux_hidden_layers", ())
                and "mm_index" not in meta.extras)

    def _forward_sample(self, meta: AttentionMetadata, T: int, n_sel: int, greedy: bool) -> torch.Tensor:
        g = self.tp_group
        g.sp_active = self._sp_ok(meta, T)
        try:
            if self.adp is not None:
                h = self._forward_attention_dp(meta, T)
            else:
                h = self.model(self.d_ids[:T], self.d_pos[:T], meta, self.kv_caches)
        finally:
            g.sp_active = False
        if self.lm_dp is not None:
            return self._sample_lm_dp(h, meta, T, n_sel)
        if n_sel == 0:  # data-parallel padding step: nothing to sample
            return self.d_out[:0]
        hs = h if (meta.is_decode and n_sel == T) else h.index_select(0, meta.logits_indices)
        logits = self.model.compute_logits(hs)
        raw = logits
        if "token_bitmask" in meta.extras:  # structured outputs: this shard's disallowed ids -> -inf
            from .structured_output import mask_logits

            logits = mask_logits(logits, meta.extras["token_bitmask"], self.sampler.vocab_start)
        if not meta.extras.get("spec", False):  # one sampled token per row
            B = n_sel
            tok = self.sampler(logits, self.d_temp[:B], self.d_topk[:B], self.d_topp[:B], self.d_unif[:B], greedy)
        elif greedy:  # speculative verification, greedy: accept until the first mismatch
            tok = self.sampler.greedy(logits)
        else:  # speculative verification with sampling: rejection sampling per position
            from ..spec_decode.rejection_sampler import rejection_sample

            pp = self.d_pos_params[:, :n_sel]
            cv, ci = self.sampler.candidates(logits)
            tok, _ = rejection_sample(cv, ci, pp[3].long(), pp[0], pp[1].int(), pp[2], pp[4], pp[5], self.max_top_k)
        self.d_out[:n_sel].copy_(tok)
        self._last_logits = logits
        if "debug_logits" in meta.extras:
            self._last_raw = raw
        if "logprobs_k" in meta.extras:
            self._last_lp = self._logprobs(raw, tok, int(meta.extras["logprobs_k"]))
        return self.d_out[:n_sel]

    def _logprobs(self, logits: torch.Tensor, tok: torch.Tensor, k: int):
        """Log-probabilities of the raw model logits (before temperature, top-k/p and grammar
        masks, as vLLM reports them) over the vocabulary shards of the sampler group: the
        sampled token's and the top ``k`` (ids, values).  Returns host lists per row."""
        g = self.sampler.group
        lf = self.sampler._mask_padding(logits.float())
        lse = torch.logsumexp(lf, -1)
        start = self.sampler.vocab_start
        V = lf.shape[1]
        inside = (tok >= start) & (tok < start + V)
        t_logit = torch.where(inside, lf.gather(1, (tok - start).clamp(0, V - 1).long()[:, None]).squeeze(1),
                              torch.full_like(lse, float("-inf")))
        kk = min(k, V) if k > 0 else 0
        vals, ids = (torch.topk(lf, kk, -1) if kk else (lf[:, :0], lf[:, :0].long()))
        ids = ids + start
        if g.world_size > 1:
            lse = torch.logsumexp(g.all_gather(lse.unsqueeze(0), dim=0), 0)
            t_logit = g.all_gather(t_logit.unsqueeze(0), dim=0).amax(0)
            if kk:
                av = g.all_gather(vals.unsqueeze(0), dim=0).permute(1, 0, 2).reshape(lf.shape[0], -1)
                ai = g.all_gather(ids.unsqueeze(0), dim=0).permute(1, 0, 2).reshape(lf.shape[0], -1)
                vals, pos = torch.topk(av, min(k, av.shape[1]), -1)
                ids = ai.gather(1, pos)
        return ((t_logit - lse).tolist(), (vals - lse[:, None]).tolist(), ids.tolist())

    def _forward_attention_dp(self, meta: AttentionMetadata, T: int) -> torch.Tensor:
        """Attention DP: gather the token ids and positions of the a replicas (every replica
        brings T rows in lockstep), give the model a slot mapping that writes only this
        replica's rows, and keep this replica's rows of the output."""
        adp = self.adp
        a, j = adp.world_size, adp.rank_in_group
        ids = adp.all_gather(self.d_ids[:T], dim=0)
        pos = adp.all_gather(self.d_pos[:T], dim=0)
        slots = torch.full((a * T,), -1, dtype=meta.slot_mapping.dtype, device=meta.slot_mapping.device)
        slots[j * T:(j + 1) * T] = meta.slot_mapping[:T]
        h = self.model(ids, pos, dataclasses.replace(meta, slot_mapping=slots), self.kv_caches)
        return h[j * T:(j + 1) * T]

    def _sample_lm_dp(self, h: torch.Tensor, meta: AttentionMetadata, T: int, n_sel: int) -> torch.Tensor:
        """lm_head DP (``model_mxfp4.py:1928-2001``): every DP replica of the supergroup pads
        its rows to R (the decode batch, equal across replicas in lockstep; max_num_seqs for
        prefill), the rows and their sampling parameters are gathered, the supergroup computes
        the vocab-sharded logits and samples all of them (rows with temperature <= 0 greedily),
        and each replica keeps its own tokens.  Runs on padding-only steps too, since the
        collectives must match."""
        dpg = self.lm_dp
        R = n_sel if meta.is_decode else self.cfg.max_num_seqs
        hs = h if (meta.is_decode and n_sel == T) else h.index_select(0, meta.logits_indices)
        if hs.shape[0] < R:
            hs = torch.cat([hs, hs.new_zeros(R - hs.shape[0], hs.shape[1])])
        logits = self.model.compute_logits(dpg.all_gather(hs, dim=0))
        if "token_bitmask" in meta.extras:
            raise NotImplementedError("structured outputs with lm_head / attention data parallelism")
        prm = [dpg.all_gather(t[:R], dim=0) for t in (self.d_temp, self.d_topk, self.d_topp, self.d_unif)]
        tok = self.sampler(logits, *prm, False)
        j = dpg.rank_in_group
        self.d_out[:n_sel].copy_(tok[j * R:j * R + n_sel])
        return self.d_out[:n_sel]

    @torch.inference_mode()
    def execute(self, so: SchedulerOutput, dp_pad: tuple | None = None) -> dict[str, list[int]]:
        """Run one step.  ``dp_pad = (kind, max_tokens, max_seqs)`` (data parallelism): pad the
        step to the largest replica's size so the MoE collectives match; an idle ``so``
        then runs a batch of padding only."""
        pad_tokens = None
        if dp_pad is not None:
            kind, t_max, b_max = dp_pad
            if so.kind == "idle":
                so = SchedulerOutput(kind, [])
            if kind == "prefill":
                pad_tokens = max(1, t_max)
        elif so.kind == "idle" or not so.seqs:
            return {}
        self.step_count += 1
        span0 = self._span_start()
        n = len(so.seqs)
        pad_to = None
        is_plain_decode = so.kind == "decode" and all(len(s.token_ids) == 1 for s in so.seqs)
        if is_plain_decode:
            want = max(n, dp_pad[2]) if dp_pad is not None else n
            pad_to = get_bucket_for_count(want, self.decode_buckets) if self.use_graphs else want
            NUM_SEQS_PADDING.labels(model_name=self.cfg.served_model_name or "model").observe(pad_to - n)
        meta, T, n_sel, greedy = self._prepare(so, pad_to, pad_tokens)
        if (is_plain_decode and self.use_graphs and "token_bitmask" not in meta.extras
                and "logprobs_k" not in meta.extras and "debug_logits" not in meta.extras):
            key = (pad_to, greedy)
            entry = self.graphs.get(key)
            if entry is None:
                if self.state_caches is not None:
                    # capture warm-up runs must not advance live recurrent states
                    self.d_sslot[:pad_to].fill_(self.scratch_slot)
                entry = self._capture(pad_to, greedy, meta, T, n_sel)
                if self.state_caches is not None:
                    self.d_sslot[:pad_to].copy_(self.h_sslot[:pad_to], non_blocking=True)
            entry.graph.replay()
            GRAPH_REPLAY_COUNT.labels(model_name=self.cfg.served_model_name or "model",
                                      bucket_name=f"decode_b{pad_to}").inc()
            out_d = self.d_out[:n_sel]
        else:
            out_d = self._forward_sample(meta, T, n_sel, greedy)
        if self.capture is not None:
            self.capture.flush({"kind": so.kind, "req_ids": [s.req_id for s in so.seqs],
                                "start_pos": [s.start_pos for s in so.seqs],
                                "num_tokens": [len(s.token_ids) for s in so.seqs]})
        if self.replacer is not None:
            self.replacer.next_step()
        # D2H of the sampled ids (the step's only device->host traffic)
        self.h_out[:n_sel].copy_(out_d, non_blocking=out_d.is_cuda)
        self._span_end(span0)
        if out_d.is_cuda:
            torch.cuda.current_stream().synchronize()
        self.d2h_bytes_last = n_sel * 8
        toks = self.h_out[:n_sel].tolist()
        raw = self.__dict__.pop("_last_raw", None)
        if raw is not None:
            self.debug_logits.write(so, raw, toks)
        res: dict[str, list[int]] = {}
        if so.kind == "decode" and any(s.spec_token_ids for s in so.seqs):
            off = 0
            for s in so.seqs:
                k = len(s.token_ids)
                res[s.req_id] = toks[off:off + k]
                off += k
            return res
        lp = self.__dict__.pop("_last_lp", None)
        self.last_logprobs = {}
        for i, s in enumerate(so.seqs):
            if s.sample:
                res[s.req_id] = [toks[i]]
                if lp is not None and s.request is not None and s.request.sampling_params.logprobs is not None:
                    n = s.request.sampling_params.logprobs
                    entry = {int(t): float(v) for t, v in zip(lp[2][i][:n], lp[1][i][:n])}
                    entry[int(toks[i])] = float(lp[0][i])
                    self.last_logprobs[s.req_id] = entry
        return res

    @torch.inference_mode()
    def score(self, so: SchedulerOutput, vocab_size: int) -> torch.Tensor:
        """Logits [T, vocab] of every token of a one-sequence prefill step (all TP vocab
        shards gathered); used by the accuracy tools."""
        meta, T, _, _ = self._prepare(so, None)
        h = self.model(self.d_ids[:T], self.d_pos[:T], meta, self.kv_caches)
        if self.lm_dp is not None:
            raise NotImplementedError("score() with lm_head data parallelism")
        logits = self.model.compute_logits(h).float()
        g = self.sampler.group
        if g.world_size > 1:
            logits = g.all_gather(logits, dim=-1)
        return logits[:, :vocab_size]

    # ---------------------------------------------------------- async decode steps
    def can_launch_async(self, so: SchedulerOutput) -> bool:
        """Plain decode steps and mixed steps (decodes + prompt chunks) without per-token host
        work (logprobs, grammars, debug dumps, tensor capture / replacement)."""
        if so.kind not in ("decode", "mixed") or not so.seqs:
            return False
        if self.capture is not None or self.replacer is not None or self.debug_logits is not None:
            return False
        if so.kind == "mixed" and self.state_caches is not None:
            return False  # recurrent-state models keep their mixed steps synchronous
        dec = so.seqs[:so.num_decode] if so.kind == "mixed" else so.seqs
        if not all(len(s.token_ids) == 1 and not s.spec_token_ids for s in dec):
            return False
        return not any(s.request is not None and (s.request.sampling_params.logprobs is not None
                                                  or s.request.grammar is not None) for s in so.seqs)

    def _span_start(self):
        if self.step_spans is None or self.device.type != "cuda":
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def _span_end(self, start) -> None:
        if start is not None and self.step_spans is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.step_spans.append((start, ev))

    def _event(self):
        if self.device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record()
            return ev
        return _DoneEvent()

    @torch.inference_mode()
    def launch(self, so: SchedulerOutput, prev: "AsyncStep | None" = None) -> "AsyncStep":
        """Start a plain decode step without waiting for it: stage the inputs, take the input
        token of every sequence that was in ``prev`` from ``prev``'s sampled ids in device
        memory, replay the decode graph and queue the D2H copy of the sampled ids.
        ``commit`` waits for it."""
        self.step_count += 1
        span0 = self._span_start()
        n = len(so.seqs)
        graphed = self.use_graphs and so.kind == "decode"
        pad_to = get_bucket_for_count(n, self.decode_buckets) if graphed else n
        NUM_SEQS_PADDING.labels(model_name=self.cfg.served_model_name or "model").observe(pad_to - n)
        meta, T, n_sel, greedy = self._prepare(so, pad_to if so.kind == "decode" else None)
        if prev is not None:
            src = self.h_src.numpy()
            src[:pad_to] = -1
            # decode sequences come first, one token row each; prompt chunks keep their host tokens
            for i, s in enumerate(so.seqs[:so.num_decode] if so.kind == "mixed" else so.seqs):
                src[i] = prev.row_of.get(s.req_id, -1)
            self.d_src[:pad_to].copy_(self.h_src[:pad_to], non_blocking=True)
            idx = self.d_src[:pad_to]
            prev_ids = self.d_out[:pad_to].index_select(0, idx.clamp(min=0))
            self.d_ids[:pad_to] = torch.where(idx >= 0, prev_ids, self.d_ids[:pad_to])
        self._h2d_done = self._event()  # the staging buffers are free again after this point
        if graphed:
            key = (pad_to, greedy)
            entry = self.graphs.get(key)
            if entry is None:
                if self.state_caches is not None:
                    self.d_sslot[:pad_to].fill_(self.scratch_slot)
                entry = self._capture(pad_to, greedy, meta, T, n_sel)
                if self.state_caches is not None:
                    self.d_sslot[:pad_to].copy_(self.h_sslot[:pad_to], non_blocking=True)
            entry.graph.replay()
            GRAPH_REPLAY_COUNT.labels(model_name=self.cfg.served_model_name or "model",
                                      bucket_name=f"decode_b{pad_to}").inc()
        else:
            self._forward_sample(meta, T, n_sel, greedy)
        self._parity ^= 1
        host = self.h_out_async[self._parity]
        host[:n_sel].copy_(self.d_out[:n_sel], non_blocking=self.device.type == "cuda")
        self._span_end(span0)
        ev = self._event()
        self.d2h_bytes_last = n_sel * 8
        return AsyncStep(so, n_sel, host, ev, {s.req_id: i for i, s in enumerate(so.seqs)})

    def commit(self, step: "AsyncStep") -> dict[str, list[int]]:
        step.event.synchronize()
        toks = step.host[:step.n_sel].tolist()
        return {s.req_id: [toks[i]] for i, s in enumerate(step.so.seqs) if s.sample}

    def _capture(self, B: int, greedy: bool, meta: AttentionMetadata, T: int, n_sel: int) -> _GraphEntry:
        t0 = time.time()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside the graph (cuBLAS/NCCL init)
                self._forward_sample(meta, T, n_sel, greedy)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.graph_pool):
            self._forward_sample(meta, T, n_sel, greedy)
        torch.cuda.synchronize()
        e = _GraphEntry(g, B)
        self.graphs[(B, greedy)] = e
        logger.info("captured decode graph batch=%d greedy=%s in %.2fs", B, greedy, time.time() - t0)
        return e

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.graph_pool = None
