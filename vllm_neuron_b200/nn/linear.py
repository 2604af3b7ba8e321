"""Tensor-parallel layers.

Behaviour of the Trainium plugin's ``ColumnParallelLinear`` (``nn/cpl.py:27,135``),
``RowParallelLinear`` (``nn/rpl.py:23,136``) and ``VocabDimShardedEmbedding``
(``nn/embedding.py:23,174,236-249``):
* column-parallel: the output features are sharded; optional all-gather of the output;
* row-parallel: input features sharded; partial products summed with an all-reduce
  (decode) or reduce-scatter (sequence-parallel prefill); the bias is added once,
  after the reduction;
* vocab-parallel embedding: each rank holds a contiguous vocab slice, looks up the
  ids it owns, zero elsewhere, then all-reduce (or reduce-scatter under SP).

Every parameter carries ``weight_loader(param, full_tensor)`` which slices the
checkpoint tensor for this rank (``utils/weight_loader.py:139``).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ..parallel.state import GroupCoordinator


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"dimension {n} not divisible by {world}")
    per = n // world
    return rank * per, (rank + 1) * per


def _narrow_loader(dim: int, group: GroupCoordinator):
    def load(param: torch.Tensor, full: torch.Tensor) -> None:
        s, e = shard_range(full.shape[dim], group.rank_in_group, group.world_size)
        param.data.copy_(full.narrow(dim, s, e - s).to(param.dtype))

    return load


def _replicated_loader(param: torch.Tensor, full: torch.Tensor) -> None:
    param.data.copy_(full.to(param.dtype))


class ColumnParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, group: GroupCoordinator, bias: bool = True,
                 gather_output: bool = False, dtype: torch.dtype = torch.bfloat16, device=None):
        super().__init__()
        self.group = group
        self.in_features, self.out_features = in_features, out_features
        self.out_local = out_features // group.world_size
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(self.out_local, in_features, dtype=dtype, device=device),
                                   requires_grad=False)
        self.weight.weight_loader = _narrow_loader(0, group)
        if bias:
            self.bias = nn.Parameter(torch.zeros(self.out_local, dtype=dtype, device=device), requires_grad=False)
            self.bias.weight_loader = _narrow_loader(0, group)
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = ops.linear(x, self.weight, self.bias)
        if self.gather_output:
            y = self.group.all_gather(y, dim=-1)
        return y


class RowParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, group: GroupCoordinator, bias: bool = True,
                 reduce_results: bool = True, dtype: torch.dtype = torch.bfloat16, device=None):
        super().__init__()
        self.group = group
        self.in_local = in_features // group.world_size
        self.reduce_results = reduce_results
        self.weight = nn.Parameter(torch.empty(out_features, self.in_local, dtype=dtype, device=device),
                                   requires_grad=False)
        self.weight.weight_loader = _narrow_loader(1, group)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=dtype, device=device), requires_grad=False)
            self.bias.weight_loader = _replicated_loader
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor, sequence_parallel: bool = False) -> torch.Tensor:
        if self.group.world_size == 1 or not self.reduce_results:
            return ops.linear(x, self.weight, self.bias)
        y = ops.linear(x, self.weight, None)
        if sequence_parallel:
            y = self.group.reduce_scatter(y, dim=0)
        else:
            y = self.group.all_reduce(y)
        if self.bias is not None:
            y = y + self.bias
        return y


class VocabParallelEmbedding(nn.Module):
    """Vocab-sharded embedding.  With embedding DP (``dp_group``) the table is sharded over a
    TP x DP supergroup (``group``): the token ids of the supergroup's DP replicas are gathered,
    looked up, reduced over the supergroup, and each replica keeps its own rows
    (``model_mxfp4.py:1718-1733``).  Every replica must bring the same token count."""

    def __init__(self, vocab: int, hidden: int, group: GroupCoordinator, dtype=torch.bfloat16, device=None,
                 dp_group: GroupCoordinator | None = None):
        super().__init__()
        self.group = group
        self.dp_group = dp_group
        self.vocab = vocab
        self.vocab_padded = ((vocab + group.world_size - 1) // group.world_size) * group.world_size
        self.per = self.vocab_padded // group.world_size
        self.start = group.rank_in_group * self.per
        self.weight = nn.Parameter(torch.zeros(self.per, hidden, dtype=dtype, device=device), requires_grad=False)
        self.weight.weight_loader = self._load

    def _load(self, param: torch.Tensor, full: torch.Tensor) -> None:
        s = self.start
        e = min(s + self.per, full.shape[0])
        param.data.zero_()
        if e > s:
            param.data[: e - s].copy_(full[s:e].to(param.dtype))

    def forward(self, ids: torch.Tensor, sequence_parallel: bool = False) -> torch.Tensor:
        if self.dp_group is not None:
            T = ids.shape[0]
            y = self.group.all_reduce(ops.embedding(self.dp_group.all_gather(ids, dim=0), self.weight, self.start))
            return y[self.dp_group.rank_in_group * T:(self.dp_group.rank_in_group + 1) * T]
        if self.group.world_size == 1:
            return ops.embedding(ids, self.weight, 0)
        y = ops.embedding(ids, self.weight, self.start)
        if sequence_parallel:
            return self.group.reduce_scatter(y, dim=0)
        return self.group.all_reduce(y)


class ParallelLMHead(nn.Module):
    """Vocab-sharded LM head: each rank produces logits for its vocab slice; the
    sampler works on the shards (distributed top-k / argmax) so the full logits
    are only gathered when requested (``nn/cpl.py:141``)."""

    def __init__(self, vocab: int, hidden: int, group: GroupCoordinator, dtype=torch.bfloat16, device=None,
                 dp_group: GroupCoordinator | None = None):
        super().__init__()
        self.group = group
        # lm_head DP: ``group`` is a TP x DP supergroup; the runner gathers the rows to sample
        # over ``dp_group`` and keeps its own tokens (``model_mxfp4.py:1928-2001``)
        self.dp_group = dp_group
        self.vocab = vocab
        self.vocab_padded = ((vocab + group.world_size - 1) // group.world_size) * group.world_size
        self.per = self.vocab_padded // group.world_size
        self.start = group.rank_in_group * self.per
        self.weight = nn.Parameter(torch.zeros(self.per, hidden, dtype=dtype, device=device), requires_grad=False)
        self.weight.weight_loader = VocabParallelEmbedding._load.__get__(self)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        return ops.linear(h, self.weight, None)


class RMSNorm(nn.Module):
    def __init__(self, hidden: int, eps: float = 1e-5, dtype=torch.float32, device=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden, dtype=dtype, device=device), requires_grad=False)
        self.weight.weight_loader = _replicated_loader

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return ops.rms_norm(x, self.weight, self.eps)
        return ops.fused_add_rms_norm(x, residual, self.weight, self.eps)
