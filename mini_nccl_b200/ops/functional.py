"""Functional ops used by the models and parallel layers.

Each op has exactly two implementations, chosen by where the tensor lives:

* a CUDA tensor runs the hand-written sm_100a kernel from
  :mod:`mini_nccl_b200.ops.kernels` (tcgen05 GEMM, flash attention,
  LayerNorm, GELU, cross-entropy).  If the extension cannot be loaded on a GPU
  machine this raises; there is no silent eager fallback;
* a CPU tensor runs the plain PyTorch expression of the same math, which is
  also what the GPU tests compare the kernels against.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _kernels():
    from . import kernels

    return kernels


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T + bias`` (tcgen05 GEMM with a bias epilogue on CUDA)."""
    if x.is_cuda and _kernels().supports_gemm(x, weight):
        return _kernels().Linear.apply(x, weight, bias)
    return F.linear(x, weight, bias)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Exact (erf) GELU, as ``nn.GELU()``."""
    if x.is_cuda:
        return _kernels().Gelu.apply(x)
    return F.gelu(x)


def linear_gelu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """``gelu(x @ weight.T + bias)``; one GEMM with a fused GELU epilogue on CUDA."""
    if x.is_cuda and _kernels().supports_gemm(x, weight):
        return _kernels().LinearGelu.apply(x, weight, bias)
    return F.gelu(F.linear(x, weight, bias))


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    if x.is_cuda:
        return _kernels().LayerNorm.apply(x, weight, bias, eps)
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def causal_attention(qkv: torch.Tensor, n_head: int) -> torch.Tensor:
    """Causal softmax attention on a fused ``[B, T, 3*H*D]`` tensor laid out
    ``[q | k | v]``; returns ``[B, T, H, D]``."""
    B, T, C3 = qkv.shape
    C = C3 // 3
    D = C // n_head
    if qkv.is_cuda:
        return _kernels().FlashAttention.apply(qkv, n_head)
    q, k, v = qkv.split(C, dim=-1)
    qh, kh, vh = (t.reshape(B, T, n_head, D).transpose(1, 2) for t in (q, k, v))
    y = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True)
    return y.transpose(1, 2)


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    if logits.is_cuda:
        return _kernels().CrossEntropy.apply(logits, targets)
    return F.cross_entropy(logits.float(), targets)
