"""Raw-logit dumps for accuracy tests (``neuron_config.debug_logits_dir``; the reference's
``NeuronModelRunner._debug_write_logits``, ``vllm/worker/neuron_model_runner.py:6847``).

With ``debug_logits_dir`` set, every engine step that samples writes the full-vocabulary fp32
logits of its sampled rows to ``{dir}/step_{N}_dp{replica}.bin`` (written to a ``.tmp`` name
and renamed, so a reader never sees a partial file).  This is cheaper than the logprobs path
for golden comparisons: no top-k, no host formatting, one file per step.

File format (little-endian, the same layout the reference's readers parse):

* header: ``num_items`` (int64), ``vocab_size`` (int64)
* per item: ``batch_idx`` (int64), ``position_id`` (int64), ``logits`` (float32[vocab_size])

``position_id`` is the sequence position whose logits these are (the first sampled row of a
request sits at ``prompt_len - 1`` and predicts output token 0); it comes from a per-request
counter of emitted rows, so partial prefill chunks (which sample nothing) and speculative
rows after the first rejected draft are never written.  Rows past ``max_tokens`` are dropped.
``batch_idx`` is the trailing integer of the request id (``LLM.generate`` names requests
``req-<n>``), or the row index when the id has none.

The vocabulary shards of a tensor-parallel sampler group are gathered before writing (a
collective every rank of the group takes); rank 0 of the group writes.
"""

from __future__ import annotations

import glob
import os
import re

import numpy as np
import torch

_ID_TAIL = re.compile(r"(\d+)(?:#\d+)?$")
_FILE = re.compile(r"step_(\d+)_dp(\d+)\.bin$")


def batch_index(req_id: str, row: int) -> int:
    m = _ID_TAIL.search(req_id)
    return int(m.group(1)) if m else row


class DebugLogitsWriter:
    def __init__(self, path: str, group, vocab_size: int, replica: int = 0):
        self.path = path
        self.group = group
        self.vocab_size = vocab_size
        self.replica = replica
        self.step = 0
        self.emitted: dict[str, int] = {}
        if self._writes():
            os.makedirs(path, exist_ok=True)

    def _writes(self) -> bool:
        return self.group is None or self.group.world_size == 1 or self.group.rank_in_group == 0

    def release(self, req_id: str) -> None:
        self.emitted.pop(req_id, None)

    @staticmethod
    def rows(so, toks: list[int]) -> list[tuple[int, object]]:
        """(logit row, scheduled sequence) pairs whose logits are real model outputs."""
        out = []
        spec = so.kind == "decode" and any(s.spec_token_ids for s in so.seqs)
        off = 0
        for i, s in enumerate(so.seqs):
            if s.request is None:
                off += len(s.token_ids) if spec else 1
                continue
            if not spec:
                if s.sample:
                    out.append((i, s))
                continue
            k = len(s.token_ids)
            drafts = list(s.spec_token_ids or [])
            for j in range(k):
                # row j counts when every draft before it was accepted
                if j > 0 and (j - 1 >= len(drafts) or toks[off + j - 1] != drafts[j - 1]):
                    break
                out.append((off + j, s))
            off += k
        return out

    def write(self, so, logits: torch.Tensor, toks: list[int]) -> None:
        g = self.group
        if g is not None and g.world_size > 1:
            logits = g.all_gather(logits.contiguous(), dim=-1)
        sel = self.rows(so, toks)
        items = []
        for row, s in sel:
            req = s.request
            n = self.emitted.get(s.req_id, 0)
            pos = req.num_prompt_tokens - 1 + n
            mt = req.sampling_params.max_tokens
            if mt is not None and pos > req.num_prompt_tokens + mt - 2:
                continue
            self.emitted[s.req_id] = n + 1
            items.append((batch_index(s.req_id, row), pos, row))
        if not items or not self._writes():
            return
        rows = torch.tensor([r for _, _, r in items], device=logits.device)
        data = logits.index_select(0, rows)[:, :self.vocab_size].float().cpu().numpy()
        base = os.path.join(self.path, f"step_{self.step}_dp{self.replica}")
        with open(base + ".tmp", "wb") as f:
            np.array([len(items), data.shape[1]], dtype="<i8").tofile(f)
            for (b, pos, _), row in zip(items, data):
                np.array([b, pos], dtype="<i8").tofile(f)
                row.astype("<f4").tofile(f)
        os.replace(base + ".tmp", base + ".bin")
        self.step += 1


def read_step_file(path: str) -> list[tuple[int, int, torch.Tensor]]:
    """Items (batch_idx, position_id, logits [vocab] float32) of one step file."""
    raw = np.fromfile(path, dtype=np.uint8)
    n, vocab = np.frombuffer(raw[:16].tobytes(), dtype="<i8")
    item = 16 + 4 * int(vocab)
    out = []
    for i in range(int(n)):
        o = 16 + i * item
        b, pos = np.frombuffer(raw[o:o + 16].tobytes(), dtype="<i8")
        row = np.frombuffer(raw[o + 16:o + item].tobytes(), dtype="<f4")
        out.append((int(b), int(pos), torch.from_numpy(row.copy())))
    return out


def read_debug_logits(path: str, replica: int | None = None) -> dict[int, dict[int, torch.Tensor]]:
    """All complete step files of a directory (one replica, or every replica) as
    ``{batch_idx: {position_id: logits}}``; a later step overwrites an earlier one."""
    files = []
    for f in glob.glob(os.path.join(path, "step_*_dp*.bin")):
        m = _FILE.search(f)
        if m and (replica is None or int(m.group(2)) == replica):
            files.append((int(m.group(2)), int(m.group(1)), f))
    out: dict[int, dict[int, torch.Tensor]] = {}
    for _, _, f in sorted(files):
        for b, pos, row in read_step_file(f):
            out.setdefault(b, {})[pos] = row
    return out


def stack_debug_logits(path: str, num_tokens: int | None = None, replica: int | None = None
                       ) -> torch.Tensor:
    """Logits [S, B, V] in the layout golden comparisons use: batch entries in increasing
    ``batch_idx`` order, positions from each entry's first written position on.  ``S`` is
    ``num_tokens`` or the shortest entry's length."""
    d = read_debug_logits(path, replica)
    if not d:
        raise FileNotFoundError(f"no debug logits under {path}")
    seqs = []
    for b in sorted(d):
        ps = sorted(d[b])
        seqs.append([d[b][p] for p in ps])
    S = num_tokens if num_tokens is not None else min(len(s) for s in seqs)
    if any(len(s) < S for s in seqs):
        raise ValueError(f"fewer than {S} logit rows for some batch entries")
    return torch.stack([torch.stack(s[:S]) for s in seqs], dim=1)


def clear_debug_logits(path: str) -> None:
    for f in glob.glob(os.path.join(path, "step_*_dp*.bin")) + glob.glob(os.path.join(path, "step_*_dp*.tmp")):
        os.remove(f)
