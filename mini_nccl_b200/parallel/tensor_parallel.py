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
the fused peer-memory kernels in :mod:`mini_nccl_b200.ops.fused_tp` (one
kernel per GEMM + collective pair).  Parameters that see only this rank's
tokens under sequence parallelism (the row-parallel bias, LayerNorms inside
the region) get partial gradients: :func:`allreduce_sequence_parallel_grads`
sums them over the group after backward.  :func:`scatter_to_sequence_parallel`
and :func:`gather_from_sequence_parallel` enter and leave the region from
replicated compute (embeddings, the head).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .. import collectives
from ..communicator import Communicator
from ..ops import functional as OF
from ..ops import fused_tp as FT


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


class _SplitTokens(torch.autograd.Function):
    """Enter the sequence-parallel region from replicated compute.

    Forward keeps this rank's run of tokens (dim 0); backward all-gathers the
    gradient, so replicated producers (embeddings) see every token's gradient.
    """

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        ctx.pg = pg
        W, r = pg.world_size, pg.rank
        if W == 1:
            return x
        if x.shape[0] % W:
            raise ValueError("sequence parallelism needs tokens divisible by the group size")
        per = x.shape[0] // W
        return x[r * per : (r + 1) * per].contiguous()

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        pg = ctx.pg
        if pg.world_size == 1:
            return None, grad
        g = grad.contiguous()
        out = torch.empty((pg.world_size * g.shape[0], *g.shape[1:]), dtype=g.dtype, device=g.device)
        collectives.all_gather_into(pg, out.view(-1), g)
        return None, out


class _JoinTokens(torch.autograd.Function):
    """Leave the sequence-parallel region into replicated compute.

    Forward all-gathers the token shards; the consumer runs identically on
    every rank, so backward just keeps this rank's slice of the gradient.
    """

    @staticmethod
    def forward(ctx, pg: Communicator, x: torch.Tensor):
        ctx.pg = pg
        if pg.world_size == 1:
            return x
        x = x.contiguous()
        out = torch.empty((pg.world_size * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
        collectives.all_gather_into(pg, out.view(-1), x)
        ctx.per = x.shape[0]
        return out

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        pg = ctx.pg
        if pg.world_size == 1:
            return None, grad
        r, per = pg.rank, ctx.per
        return None, grad[r * per : (r + 1) * per].contiguous()


def scatter_to_sequence_parallel(pg: Communicator, x: torch.Tensor) -> torch.Tensor:
    """This rank's tokens (dim 0, sequence-major) of a replicated activation."""
    return _SplitTokens.apply(pg, x)


def gather_from_sequence_parallel(pg: Communicator, x: torch.Tensor) -> torch.Tensor:
    """Every rank's tokens (dim 0) for replicated compute after the region."""
    return _JoinTokens.apply(pg, x)


def mark_sequence_parallel(*modules: nn.Module) -> None:
    """Tag the parameters of replicated modules that run inside the region."""
    for m in modules:
        for p in m.parameters():
            p.sequence_parallel = True


def allreduce_sequence_parallel_grads(module: nn.Module, pg: Communicator) -> int:
    """Sum, over the group, the gradients of parameters tagged ``sequence_parallel``.

    Under sequence parallelism each rank's gradient of a replicated parameter
    inside the region covers only its own tokens; the full gradient is the
    sum.  One all-reduce over the concatenated gradients; returns its bytes.
    """
    grads = [p.grad for p in module.parameters() if getattr(p, "sequence_parallel", False) and p.grad is not None]
    if pg.world_size == 1 or not grads:
        return 0
    by_dtype: dict[torch.dtype, list[torch.Tensor]] = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    total = 0
    for group in by_dtype.values():
        flat = torch.cat([g.reshape(-1) for g in group])
        collectives.all_reduce(pg, flat)
        at = 0
        for g in group:
            g.copy_(flat[at : at + g.numel()].view_as(g))
            at += g.numel()
        total += flat.numel() * flat.element_size()
    return total


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
        if self.sequence_parallel and not self.gather_output:
            dc = FT.usable(self.pg, x, self.weight)
            if dc is not None:  # one kernel: gather the token shards inside the GEMM
                y2 = FT.AllGatherLinear.apply(dc, x.reshape(-1, x.shape[-1]), self.weight, self.bias)
                return y2.view(self.pg.world_size * x.shape[0], *x.shape[1:-1], self.shard_size)
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
        if self.bias is not None and sequence_parallel:
            self.bias.sequence_parallel = True  # added to this rank's tokens only
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``x W^T + b`` reduced over the group (+ ``residual``, same shape as the output)."""
        if not self.input_is_sharded:
            x = x[..., self.shard_start : self.shard_start + self.shard_size]
        if self.sequence_parallel:
            dc = FT.usable(self.pg, x, self.weight)
            if dc is not None and (residual is None or residual.dtype == torch.bfloat16):
                # one kernel: tiles go to the ranks owning their tokens, bias and residual added once
                lead = x.shape[:-1]
                r2 = residual.reshape(-1, self.out_features) if residual is not None else None
                y2 = FT.LinearReduceScatter.apply(dc, x.reshape(-1, x.shape[-1]), self.weight, self.bias, r2)
                return y2.view(lead[0] // self.pg.world_size, *lead[1:], self.out_features)
        partial = OF.linear(x, self.weight, None)
        if self.sequence_parallel:
            y = _ScatterTokens.apply(self.pg, partial)
        else:
            y = _ReduceFromGroup.apply(self.pg, partial)
        if self.bias is not None:
            y = y + self.bias
        return y if residual is None else residual + y

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

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        if self.up.sequence_parallel and self.down.sequence_parallel:
            dc = FT.usable(self.up.pg, x, self.up.weight, self.down.weight)
            if dc is not None and (residual is None or residual.dtype == torch.bfloat16):
                # AG->GEMM+GELU and GEMM->RS(+bias+residual): two kernels forward, two backward
                r2 = residual.reshape(-1, x.shape[-1]) if residual is not None else None
                y2 = FT.ParallelMLPFused.apply(dc, x.reshape(-1, x.shape[-1]), self.up.weight, self.up.bias,
                                               self.down.weight, self.down.bias, r2)
                return y2.view(x.shape)
        return self.down(OF.gelu(self.up(x)), residual=residual)


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

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        qkv = self.qkv(x)
        if self.sequence_parallel:
            # Sequence-parallel activations are sequence-major, [T, B, C]: the
            # token gather concatenates along T, attention wants [B, T, C].
            y = self._attend(qkv.transpose(0, 1).contiguous()).transpose(0, 1).contiguous()
        else:
            y = self._attend(qkv)
        return self.proj(y, residual=residual)

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
    "allreduce_sequence_parallel_grads",
    "gather_from_sequence_parallel",
    "mark_sequence_parallel",
    "scatter_to_sequence_parallel",
]
