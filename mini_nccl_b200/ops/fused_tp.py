"""Tensor-parallel layers on fused GEMM + collective kernels (sequence parallel).

With a sequence-parallel layout the activations between tensor-parallel
layers hold only this rank's tokens, so the column-parallel layer starts with
an all-gather of the token shards and the row-parallel layer ends with a
reduce-scatter of the partial sums (the reference does the non-sequence-
parallel form with an all-reduce, mini_nccl/tensor_parallel.py:53-91).  On
CUDA each of those pairs is ONE kernel of the device communicator:

* :meth:`DeviceComm.all_gather_gemm` -- gather warps inside the tcgen05 GEMM
  copy the peers' token shards into local memory while the tiles of the local
  shard compute;
* :meth:`DeviceComm.gemm_reduce_scatter` -- the GEMM epilogue stores each
  finished tile into the memory of the rank that owns those tokens, then the
  owners sum the slots (bias and residual added once).

Backward passes use the same two kernels with the roles swapped: the
data-gradient of an all-gather -> GEMM is a GEMM -> reduce-scatter and vice
versa; the weight gradients reuse the gathered operand the fused kernel left
in local memory.

Activations are 2-D ``[tokens, features]`` here (rows = tokens in
sequence-major order, this rank's rows contiguous).
"""

from __future__ import annotations

import torch

from . import kernels as K


class AllGatherLinear(torch.autograd.Function):
    """Column-parallel ``y = all_gather(x_shard) @ W^T + b``."""

    @staticmethod
    def forward(ctx, dc, x, weight, bias):
        y, gathered = dc.all_gather_gemm(x, weight, bias=bias)
        ctx.dc = dc
        ctx.has_bias = bias is not None
        ctx.save_for_backward(gathered, weight)
        return y

    @staticmethod
    def backward(ctx, gy):
        gathered, weight = ctx.saved_tensors
        gy = gy.contiguous()
        dx = ctx.dc.gemm_reduce_scatter(gy, weight, w_mn=True)
        dw = K.gemm(gy, gathered, a_mn=True, b_mn=True)
        db = K.bias_grad(gy, weight.dtype) if ctx.has_bias else None
        return None, dx, dw, db


class LinearReduceScatter(torch.autograd.Function):
    """Row-parallel ``y_shard = reduce_scatter(x @ W^T) + b + resid_shard``.

    The bias is replicated; its gradient here covers this rank's tokens only
    (sum it over the group, see ``allreduce_sequence_parallel_grads``).
    """

    @staticmethod
    def forward(ctx, dc, x, weight, bias, resid):
        y = dc.gemm_reduce_scatter(x, weight, bias=bias, resid=resid)
        ctx.dc = dc
        ctx.has_bias = bias is not None
        ctx.has_resid = resid is not None
        ctx.save_for_backward(x, weight)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, weight = ctx.saved_tensors
        gy = gy.contiguous()
        dx, gy_full = ctx.dc.all_gather_gemm(gy, weight, w_mn=True)
        dw = K.gemm(gy_full, x, a_mn=True, b_mn=True)
        db = K.bias_grad(gy, weight.dtype) if ctx.has_bias else None
        return None, dx, dw, db, (gy if ctx.has_resid else None)


class ParallelMLPFused(torch.autograd.Function):
    """``resid + b2 + reduce_scatter(gelu(all_gather(x) @ W1^T + b1) @ W2^T)``.

    Four fused kernels per step: AG->GEMM(+bias+GELU) and GEMM->RS forward;
    AG->GEMM(*GELU') and GEMM->RS backward (plus two local weight-gradient
    GEMMs).  The GELU pre-activation is kept for the backward.
    """

    @staticmethod
    def forward(ctx, dc, x, w1, b1, w2, b2, resid):
        rows = x.shape[0] * dc.world_size
        pre = torch.empty(rows, w1.shape[0], dtype=torch.bfloat16, device=x.device)
        h, gathered = dc.all_gather_gemm(x, w1, bias=b1, gelu_out_aux=pre)
        y = dc.gemm_reduce_scatter(h, w2, bias=b2, resid=resid)
        ctx.dc = dc
        ctx.flags = (b1 is not None, b2 is not None, resid is not None)
        ctx.save_for_backward(gathered, pre, h, w1, w2)
        return y

    @staticmethod
    def backward(ctx, gy):
        gathered, pre, h, w1, w2 = ctx.saved_tensors
        has_b1, has_b2, has_resid = ctx.flags
        dc = ctx.dc
        gy = gy.contiguous()
        dpre, gy_full = dc.all_gather_gemm(gy, w2, w_mn=True, gelu_grad_aux=pre)
        dw2 = K.gemm(gy_full, h, a_mn=True, b_mn=True)
        db2 = K.bias_grad(gy, w2.dtype) if has_b2 else None
        dx = dc.gemm_reduce_scatter(dpre, w1, w_mn=True)
        dw1 = K.gemm(dpre, gathered, a_mn=True, b_mn=True)
        db1 = K.bias_grad(dpre, w1.dtype) if has_b1 else None
        return None, dx, dw1, db1, dw2, db2, (gy if has_resid else None)


def usable(pg, x: torch.Tensor, *weights: torch.Tensor) -> object | None:
    """The device communicator when the fused path applies to these tensors, else None."""
    if not x.is_cuda or x.dtype != torch.bfloat16 or pg.world_size == 1:
        return None
    if any(w.dtype != torch.bfloat16 or w.shape[0] % 8 or w.shape[1] % 8 for w in weights):
        return None
    getter = getattr(pg, "device_comm", None)
    return getter() if callable(getter) else None
