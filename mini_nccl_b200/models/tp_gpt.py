"""GPT split three ways: tensor parallel blocks, pipeline stages, data parallel replicas.

The building blocks of the reference's 3D example (examples/three_dimensional_gpt.py:
56-251) as a reusable model: :class:`ParallelBlock` is the pre-LN GPT block
with head-split attention and a column/row MLP over a tensor-parallel group;
:class:`GPTStage` is one pipeline stage of a GPT (the first stage owns the
embeddings, the last the final LayerNorm and the LM head).

With ``sequence_parallel=True`` (the default on GPUs) the activations between
blocks hold only this rank's tokens, sequence-major ``[T / tp, B, C]``; every
column-parallel GEMM then starts with an all-gather and every row-parallel
GEMM ends with a reduce-scatter, each run as ONE fused kernel on CUDA
(:mod:`mini_nccl_b200.ops.fused_tp`).  LayerNorm parameters and row biases
inside the region get partial gradients; :func:`sync_tensor_parallel_grads`
sums them over the tensor-parallel group after the pipeline has drained.

Deliberate difference from the single-GPU GPT: the LM head of the last stage
is its own parameter (not tied to the first stage's embedding, which lives on
another pipeline rank).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import functional as OF
from ..parallel.tensor_parallel import (
    ParallelMLP,
    ParallelSelfAttention,
    allreduce_sequence_parallel_grads,
    gather_from_sequence_parallel,
    mark_sequence_parallel,
    scatter_to_sequence_parallel,
)


def _kernels():
    from ..ops import kernels

    return kernels


class ParallelBlock(nn.Module):
    """Pre-LN GPT block whose attention heads and MLP columns are split over ``tp``."""

    def __init__(self, n_embd: int, n_head: int, tp, sequence_parallel: bool = True) -> None:
        super().__init__()
        self.ln1 = nn.LayerNorm(n_embd)
        self.attn = ParallelSelfAttention(n_embd, n_head, tp, sequence_parallel=sequence_parallel)
        self.ln2 = nn.LayerNorm(n_embd)
        self.mlp = ParallelMLP(n_embd, tp, sequence_parallel=sequence_parallel)
        if sequence_parallel:
            mark_sequence_parallel(self.ln1, self.ln2)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.attn(OF.layer_norm(x, self.ln1.weight, self.ln1.bias, self.ln1.eps), residual=x)
        return self.mlp(OF.layer_norm(x, self.ln2.weight, self.ln2.bias, self.ln2.eps), residual=x)


class GPTStage(nn.Module):
    """Layers ``[stage * L / n_stages, (stage + 1) * L / n_stages)`` of a GPT.

    Input of the first stage: token ids ``[B, T]``; of the others: the
    previous stage's activation.  Output of every stage but the last: the
    activation, sequence-major ``[T / tp, B, C]`` under sequence parallelism
    (``[B, T, C]`` otherwise); the last stage returns its final hidden states
    and :meth:`loss` turns them into the mean cross-entropy.
    """

    def __init__(self, vocab_size: int, block_size: int, n_layer: int, n_head: int, n_embd: int, tp,
                 stage: int = 0, n_stages: int = 1, sequence_parallel: bool = True) -> None:
        super().__init__()
        if n_layer % n_stages:
            raise ValueError(f"{n_layer} layers do not split evenly over {n_stages} stages")
        self.tp = tp
        self.sp = sequence_parallel and tp.world_size > 1
        self.first, self.last = stage == 0, stage == n_stages - 1
        per = n_layer // n_stages
        if self.first:
            self.tok_emb = nn.Embedding(vocab_size, n_embd)
            self.pos_emb = nn.Parameter(torch.zeros(1, block_size, n_embd))
            nn.init.normal_(self.tok_emb.weight, std=0.02)
        self.blocks = nn.ModuleList(ParallelBlock(n_embd, n_head, tp, self.sp) for _ in range(per))
        if self.last:
            self.ln_f = nn.LayerNorm(n_embd)
            self.head = nn.Linear(n_embd, vocab_size, bias=False)
            nn.init.normal_(self.head.weight, std=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.first:
            T = x.shape[1]
            if x.is_cuda:
                x = _kernels().Embedding.apply(x, self.tok_emb.weight, self.pos_emb[0, :T])
            else:
                x = self.tok_emb(x) + self.pos_emb[:, :T]
            if self.sp:
                x = scatter_to_sequence_parallel(self.tp, x.transpose(0, 1).contiguous())
        for blk in self.blocks:
            x = blk(x)
        return x

    def loss(self, h: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Mean next-token cross-entropy of the last stage's hidden states."""
        if self.sp:
            h = gather_from_sequence_parallel(self.tp, h).transpose(0, 1).contiguous()
        h = OF.layer_norm(h, self.ln_f.weight, self.ln_f.bias, self.ln_f.eps)
        if h.is_cuda and torch.is_grad_enabled():
            return _kernels().HeadCrossEntropy.apply(h, self.head.weight, targets)
        logits = self.head(h)
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))


def sync_tensor_parallel_grads(stage: nn.Module, tp) -> int:
    """Sum the sequence-parallel partial gradients over the tensor-parallel group."""
    return allreduce_sequence_parallel_grads(stage, tp)
