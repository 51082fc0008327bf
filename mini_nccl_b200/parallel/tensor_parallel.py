"""Tensor parallelism: Megatron column/row layers and head-split attention.

Same layers and autograd placement as the reference
(mini_nccl/tensor_parallel.py:53-304):

* ``f`` (:class:`_CopyToGroup`): identity forward, all-reduce of ``dL/dx``
  backward -- at a column-parallel layer's input;
* ``g`` (:class:`_ReduceFromGroup`): all-reduce of the partial sums forward,
  identity backward -- at a row-parallel layer's output;
* ``ColumnParallelLinear`` (output features split; ``shard_rows`` for the fused
  QKV head mapping; optional ``gather_output``), ``RowParallelLinear`` (input
  features split, unsharded bias added after the reduction,
  ``input_is_sharded=False`` slices locally), ``ParallelMLP`` and
  ``ParallelSelfAttention`` (each rank owns whole heads).

B200 addition, ``sequence_parallel=True``: activations *between* the
tensor-parallel layers are split along the token dimension, so ``f`` becomes
an all-gather of the token shards before the column GEMM and ``g`` becomes a
reduce-scatter after the row GEMM (Megatron-SP).  Same FLOPs, half the
activation traffic of the all-reduce pair, and LayerNorm/residual work is done
once per token instead of once per rank.  On CUDA these boundaries run as
the fused peer-memory kernels in :mod:`mini_nccl_b200.ops.fused_tp`.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .. import collectives
from ..communicator import Communicator
from ..ops import functional as OF


class _CopyToGroup(torch.autograd.Function):
    """Megatron ``f``: identity forward, all-reduce backward."""

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        ctx.pg = pg
        return x

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        pg = ctx.pg
        if pg.world_size > 1:
            grad = grad.contiguous()
            collectives.all_reduce(pg, grad)
        return None, grad


class _ReduceFromGroup(torch.autograd.Function):
    """Megatron ``g``: all-reduce forward, identity backward."""

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        if pg.world_size > 1:
            x = x.contiguous()
            collectives.all_reduce(pg, x)
        return x

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        return None, grad


class _GatherLastDim(torch.autograd.Function):
    """Concatenate feature shards forward; keep this rank's slice backward."""

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        ctx.pg = pg
        ctx.width = x.shape[-1]
        if pg.world_size == 1:
            return x
        return torch.cat(collectives.all_gather(pg, x.contiguous()), dim=-1)

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        pg = ctx.pg
        if pg.world_size == 1:
            return None, grad
        lo = pg.rank * ctx.width
        return None, grad[..., lo : lo + ctx.width].contiguous()


class _GatherTokens(torch.autograd.Function):
    """Sequence-parallel ``f``: all-gather token shards forward, reduce-scatter backward."""

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        ctx.pg = pg
        if pg.world_size == 1:
            return x
        x = x.contiguous()
        out = torch.empty((pg.world_size * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
        collectives.all_gather_into(pg, out.view(-1), x)
        return out

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        pg = ctx.pg
        if pg.world_size == 1:
            return None, grad
        g = grad.contiguous()
        part = collectives.reduce_scatter(pg, g.view(-1))
        return None, part.view(g.shape[0] // pg.world_size, *g.shape[1:])


class _ScatterTokens(torch.autograd.Function):
    """Sequence-parallel ``g``: reduce-scatter over tokens forward, all-gather backward."""

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        ctx.pg = pg
        if pg.world_size == 1:
            return x
        x = x.contiguous()
        if x.shape[0] % pg.world_size:
            raise ValueError("sequence parallelism needs tokens divisible by the group size")
        part = collectives.reduce_scatter(pg, x.view(-1))
        return part.view(x.shape[0] // pg.world_size, *x.shape[1:])

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        pg = ctx.pg
        if pg.world_size == 1:
            return None, grad
        g = grad.contiguous()
        out = torch.empty((pg.world_size * g.shape[0], *g.shape[1:]), dtype=g.dtype, device=g.device)
        collectives.all_gather_into(pg, out.view(-1), g)
        return None, out


def _shard_size(total: int, world_size: int, rank: int) -> tuple[int, int]:
    """(start, size) of an even split with the remainder on the leading ranks."""
    q, extra = divmod(total, world_size)
    return rank * q + min(rank, extra), q + (1 if rank < extra else 0)


class ColumnParallelLinear(nn.Module):
    """``y = x A^T + b`` with ``A``'s output features split across ranks."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        pg: Communicator,
        bias: bool = True,
        gather_output: bool = False,
        shard_rows: torch.Tensor | None = None,
        sequence_parallel: bool = False,
        device=None,
        dtype=None,
    ) -> None:
        super().__init__()
        self.pg = pg
        self.in_features = in_features
        self.out_features = out_features
        self.gather_output = gather_output
        self.sequence_parallel = sequence_parallel
        if shard_rows is None:
            self.shard_start, self.shard_size = _shard_size(out_features, pg.world_size, pg.rank)
            self.shard_rows = None
        else:
            self.register_buffer("shard_rows", shard_rows, persistent=False)
            self.shard_start, self.shard_size = -1, int(shard_rows.numel())
        kw = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(torch.empty(self.shard_size, in_features, **kw))
        self.bias = nn.Parameter(torch.zeros(self.shard_size, **kw)) if bias else None
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sequence_parallel:
            x = _GatherTokens.apply(self.pg, x)
        else:
            x = _CopyToGroup.apply(self.pg, x)
        y = OF.linear(x, self.weight, self.bias)
        if self.gather_output:
            if self.shard_rows is not None:
                raise RuntimeError("gather_output assumes a contiguous output shard")
            y = _GatherLastDim.apply(self.pg, y)
        return y

    @torch.no_grad()
    def load_full_weight(self, weight: torch.Tensor, bias: torch.Tensor | None = None) -> None:
        """Copy this rank's rows out of an unsharded weight (tests, loading)."""
        if self.shard_rows is not None:
            rows = self.shard_rows.to(weight.device)
            self.weight.copy_(weight.index_select(0, rows))
            if self.bias is not None and bias is not None:
                self.bias.copy_(bias.index_select(0, rows))
            return
        stop = self.shard_start + self.shard_size
        self.weight.copy_(weight[self.shard_start : stop])
        if self.bias is not None and bias is not None:
            self.bias.copy_(bias[self.shard_start : stop])


class RowParallelLinear(nn.Module):
    """``y = x A^T + b`` with ``A``'s input features split; bias added once, after."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        pg: Communicator,
        bias: bool = True,
        input_is_sharded: bool = True,
        sequence_parallel: bool = False,
        device=None,
        dtype=None,
    ) -> None:
        super().__init__()
        self.pg = pg
        self.in_features = in_features
        self.out_features = out_features
        self.input_is_sharded = input_is_sharded
        self.sequence_parallel = sequence_parallel
        self.shard_start, self.shard_size = _shard_size(in_features, pg.world_size, pg.rank)
        kw = {"device": device, "dtype": dtype}
        self.weight = nn.Parameter(torch.empty(out_features, self.shard_size, **kw))
        self.bias = nn.Parameter(torch.zeros(out_features, **kw)) if bias else None
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.input_is_sharded:
            x = x[..., self.shard_start : self.shard_start + self.shard_size]
        partial = OF.linear(x, self.weight, None)
        if self.sequence_parallel:
            y = _ScatterTokens.apply(self.pg, partial)
        else:
            y = _ReduceFromGroup.apply(self.pg, partial)
        if self.bias is not None:
            y = y + self.bias
        return y

    @torch.no_grad()
    def load_full_weight(self, weight: torch.Tensor, bias: torch.Tensor | None = None) -> None:
        self.weight.copy_(weight[:, self.shard_start : self.shard_start + self.shard_size])
        if self.bias is not None and bias is not None:
            self.bias.copy_(bias)


class ParallelMLP(nn.Module):
    """Column-parallel up projection, GELU, row-parallel down projection."""

    def __init__(
        self, width: int, pg: Communicator, expansion: int = 4, sequence_parallel: bool = False,
        device=None, dtype=None,
    ) -> None:
        super().__init__()
        kw = {"device": device, "dtype": dtype}
        self.up = ColumnParallelLinear(width, expansion * width, pg, sequence_parallel=sequence_parallel, **kw)
        self.down = RowParallelLinear(expansion * width, width, pg, sequence_parallel=sequence_parallel, **kw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down(OF.gelu(self.up(x)))


def _qkv_shard_rows(width: int, n_head: int, head_dim: int, pg: Communicator) -> torch.Tensor:
    """Rows of a fused ``[q | k | v]`` weight holding this rank's heads in each third."""
    per = n_head // pg.world_size
    heads = torch.arange(pg.rank * per, (pg.rank + 1) * per)
    within = torch.arange(head_dim)
    rows = [third * width + (heads[:, None] * head_dim + within[None, :]).reshape(-1) for third in range(3)]
    return torch.cat(rows).to(torch.long)


class ParallelSelfAttention(nn.Module):
    """Causal self-attention with whole heads per rank."""

    def __init__(
        self, width: int, n_head: int, pg: Communicator, sequence_parallel: bool = False,
        device=None, dtype=None,
    ) -> None:
        super().__init__()
        if n_head % pg.world_size:
            raise ValueError(f"n_head={n_head} must be divisible by world_size={pg.world_size}")
        if width % n_head:
            raise ValueError(f"width={width} must be divisible by n_head={n_head}")
        kw = {"device": device, "dtype": dtype}
        self.pg = pg
        self.n_head = n_head
        self.local_heads = n_head // pg.world_size
        self.head_dim = width // n_head
        self.sequence_parallel = sequence_parallel
        self.qkv = ColumnParallelLinear(
            width, 3 * width, pg, shard_rows=_qkv_shard_rows(width, n_head, self.head_dim, pg),
            sequence_parallel=sequence_parallel, **kw,
        )
        self.proj = RowParallelLinear(width, width, pg, sequence_parallel=sequence_parallel, **kw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        qkv = self.qkv(x)
        if self.sequence_parallel:
            # Sequence-parallel activations are sequence-major, [T, B, C]: the
            # token gather concatenates along T, attention wants [B, T, C].
            y = self._attend(qkv.transpose(0, 1)).transpose(0, 1).contiguous()
        else:
            y = self._attend(qkv)
        return self.proj(y)

    def _attend(self, qkv: torch.Tensor) -> torch.Tensor:
        B, T, _ = qkv.shape
        w = self.local_heads * self.head_dim
        return OF.causal_attention(qkv, self.local_heads).reshape(B, T, w)


__all__ = [
    "ColumnParallelLinear",
    "ParallelMLP",
    "ParallelSelfAttention",
    "RowParallelLinear",
    "_qkv_shard_rows",
    "_shard_size",
]
