"""EAGLE-3 proposer (``vllm/spec_decode/eagle.py:31`` of the Trainium plugin).

Per engine step:
1. target verification: every running request feeds ``[last, d1..dk]``; for greedy
   requests the target returns its argmax at each of the k+1 positions and the longest
   matching prefix of drafts is accepted plus one bonus token (``nn/rejection_sampler.py:12``
   semantics: accept until the first mismatch), so the output equals non-speculative greedy
   decoding exactly; requests that sample are verified by rejection sampling
   (``spec_decode/rejection_sampler.py``), which keeps their output distribution.
2. draft catch-up: the draft layer runs over the positions verified in this step, with
   input token = the token at position p+1 and hidden = fc(target aux hidden at p),
   writing its own KV cache (same block tables as the target);
3. the first draft comes from the hidden at the last accepted position, then k-1
   recurrent single-token draft steps (input: previous draft token, previous draft
   hidden) produce the rest (the reference unrolls this loop in one graph,
   ``eagle3_model.py:811-851``).
"""

from __future__ import annotations

import torch

from ..config import EngineConfig, load_hf_config
from ..logging_config import init_logger
from ..models.base import random_init_, random_init_device_
from ..models.eagle3 import Eagle3Config, Eagle3LlamaForCausalLM
from ..ops.metadata import AttentionMetadata

logger = init_logger(__name__)


class EagleProposer:
    def __init__(self, cfg: EngineConfig, worker):
        sc = cfg.speculative_config
        self.k = sc.num_speculative_tokens
        self.worker = worker
        self.runner = worker.runner
        self.device = worker.device
        hf = sc.draft_hf_config if sc.draft_hf_config is not None else load_hf_config(sc.model)
        dcfg = Eagle3Config.from_hf(hf)
        dtype = worker.model.dtype
        self.draft = Eagle3LlamaForCausalLM(dcfg, None, dtype=dtype, device=self.device).eval()
        if sc.model is None or cfg.load_format == "dummy":
            (random_init_device_ if self.device.type == "cuda" else random_init_)(self.draft, cfg.seed + 17)
            self.draft.d2t.zero_()
        else:
            from ..utils.checkpoints import SafetensorsCheckpoint

            self.draft.load_weights(SafetensorsCheckpoint(sc.model))
        if not self.draft.has_embed and hasattr(worker.model, "embed_tokens"):
            emb = worker.model.embed_tokens.weight  # share the target's embedding (TP=1 layout)
            if emb.shape == self.draft.embed_tokens.shape:
                self.draft.embed_tokens.data.copy_(emb)
        target = worker.model
        layers = target.get_eagle3_aux_hidden_state_layers() if hasattr(target, "get_eagle3_aux_hidden_state_layers") \
            else (2, len(target.layers) // 2, len(target.layers) - 3)
        target.aux_hidden_layers = tuple(layers)
        nb = self.runner.num_blocks
        shape = (nb, dcfg.num_key_value_heads, cfg.block_size, dcfg.head_dim)
        self.kv = (torch.zeros(shape, dtype=dtype, device=self.device),
                   torch.zeros(shape, dtype=dtype, device=self.device))
        self.bs = cfg.block_size
        self.max_blocks = self.runner.max_blocks
        self._aux = None
        self.stats = {"proposed": 0, "accepted": 0, "steps": 0}
        logger.info("EAGLE-3 proposer: %d speculative tokens, aux layers %s", self.k, layers)

    # --------------------------------------------------------------- verification
    def execute_with_speculation(self, so) -> dict[str, list[int]]:
        out = self.runner.execute(so)
        self._aux = getattr(self.worker.model, "_aux", None)
        res = {}
        for s in so.seqs:
            toks = out.get(s.req_id, [])
            drafts = s.spec_token_ids
            n_acc = 0
            while n_acc < len(drafts) and n_acc < len(toks) and drafts[n_acc] == toks[n_acc]:
                n_acc += 1
            res[s.req_id] = toks[:n_acc + 1]
            self.stats["proposed"] += len(drafts)
            self.stats["accepted"] += n_acc
        self.stats["steps"] += 1
        return res

    # -------------------------------------------------------------------- helpers
    def _meta(self, q_lens: list[int], seq_lens: list[int], block_rows: list[list[int]], positions: list[int],
              is_decode: bool) -> AttentionMetadata:
        dev = self.device
        B = len(q_lens)
        qsl = torch.zeros(B + 1, dtype=torch.int32)
        qsl[1:] = torch.tensor(q_lens).cumsum(0)
        bt = torch.zeros(B, self.max_blocks, dtype=torch.int32)
        for i, row in enumerate(block_rows):
            bt[i, :len(row)] = torch.tensor(row, dtype=torch.int32)
        slots = []
        for i, row in enumerate(block_rows):
            start = seq_lens[i] - q_lens[i]
            for p in range(start, seq_lens[i]):
                slots.append(row[p // self.bs] * self.bs + p % self.bs)
        return AttentionMetadata(
            num_tokens=sum(q_lens), num_seqs=B, is_decode=is_decode, query_start_loc=qsl.to(dev),
            seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=dev), block_tables=bt.to(dev),
            slot_mapping=torch.tensor(slots, dtype=torch.int64, device=dev), logits_indices=None,
            max_query_len=max(q_lens), max_seq_len=max(seq_lens), workspace=None, num_splits=1)

    # -------------------------------------------------------------------- propose
    @torch.inference_mode()
    def propose(self, so, sampled: dict[str, list[int]], scheduler) -> None:
        if so.kind not in ("prefill", "decode"):
            return
        if so.kind == "prefill":
            self._aux = getattr(self.worker.model, "_aux", None)
        aux = self._aux
        if aux is None:
            return
        tok_in, pos_in, rows_in, q_lens, seq_lens, blocks, last_idx, reqs = [], [], [], [], [], [], [], []
        off = 0
        for s in so.seqs:
            n = len(s.token_ids)
            req = scheduler.requests.get(s.req_id)
            if so.kind == "decode":
                m = len(sampled.get(s.req_id, []))  # accepted drafts + bonus
            else:
                m = n
            if req is None or m == 0:
                off += n
                continue
            all_ids = req.all_token_ids
            if s.start_pos + m >= len(all_ids) + 1:
                m = len(all_ids) - s.start_pos - 1
            if m <= 0:
                off += n
                continue
            tok_in += all_ids[s.start_pos + 1:s.start_pos + 1 + m]
            pos_in += list(range(s.start_pos, s.start_pos + m))
            rows_in += list(range(off, off + m))
            q_lens.append(m)
            seq_lens.append(s.start_pos + m)
            blocks.append(list(req.block_ids))
            last_idx.append(sum(q_lens) - 1)
            reqs.append((req, s.sample))
            off += n
        if not q_lens:
            return
        dev = self.device
        hid = self.draft.combine_hidden_states(aux[torch.tensor(rows_in, device=dev)])
        meta = self._meta(q_lens, seq_lens, blocks, pos_in, False)
        h = self.draft.step(torch.tensor(tok_in, device=dev), torch.tensor(pos_in, device=dev), hid, meta, self.kv)
        sel = [i for i, (_, smp) in enumerate(reqs) if smp]
        if not sel:
            return
        live = []
        for i in sel:
            req = reqs[i][0]
            if req.status.finished or not scheduler.kv.allocate_slots(req, self.k + 1):
                req.spec_token_ids = []
                continue
            live.append(i)
        if not live:
            return
        hcur = h[torch.tensor([last_idx[i] for i in live], device=dev)]
        d = self.draft.logits_to_target_ids(hcur)
        drafts = [d]
        pos = torch.tensor([seq_lens[i] - 1 for i in live], device=dev)
        for _ in range(self.k - 1):
            pos = pos + 1
            plist = pos.tolist()
            meta = self._meta([1] * len(live), [p + 1 for p in plist], [list(reqs[i][0].block_ids) for i in live],
                              plist, True)
            hcur = self.draft.step(d, pos, hcur, meta, self.kv)
            d = self.draft.logits_to_target_ids(hcur)
            drafts.append(d)
        allk = torch.stack(drafts, dim=1).tolist()
        for j, i in enumerate(live):
            reqs[i][0].spec_token_ids = [int(x) for x in allk[j]]

    def acceptance_rate(self) -> float:
        return self.stats["accepted"] / max(1, self.stats["proposed"])
