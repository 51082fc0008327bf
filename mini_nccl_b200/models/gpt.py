"""Decoder-only GPT (pre-LayerNorm, learned positions, tied head).

Same architecture, parameter names and initialisation as the reference's
example model (examples/model.py:10-87): token embedding plus a learned
``pos_emb`` of shape ``[1, block_size, n_embd]``; each block is LayerNorm ->
fused QKV ``Linear(C, 3C)`` -> causal attention -> ``proj`` -> residual, then
LayerNorm -> ``mlp = Sequential(Linear(C, 4C), GELU, Linear(4C, C))`` ->
residual; final LayerNorm and a head tied to the token embedding; weights
N(0, 0.02), biases zero.  A state dict of either model loads into the other.

On CUDA every op runs a kernel from :mod:`mini_nccl_b200.ops.kernels`:

* LayerNorm (warp-per-row, fp32 statistics);
* the QKV / projection / MLP GEMMs on tcgen05 with bias, GELU, GELU' and the
  residual add fused into their epilogues (the MLP is one autograd node);
* flash attention reading q, k, v straight out of the fused QKV output;
* the LM head fused with cross-entropy: logits are produced, turned into
  ``dlogits`` in place and consumed by the two gradient GEMMs inside the
  forward, so training never materialises fp32 logits (``forward`` then
  returns ``logits=None``);
* the embedding gather with the position add, and its scatter-add backward.

On CPU the same module runs plain PyTorch, which is what the numerics tests
compare the kernels against.
"""

from __future__ import annotations

from dataclasses import dataclass

import os

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class GPTConfig:
    vocab_size: int = 50304
    block_size: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768

    @property
    def n_params(self) -> int:
        C, L, V, T = self.n_embd, self.n_layer, self.vocab_size, self.block_size
        per_block = 12 * C * C + 13 * C
        return V * C + T * C + L * per_block + 2 * C


def _kernels():
    from ..ops import kernels

    return kernels


#: The LayerNorm backward also adds the residual branch's gradient (one kernel
#: instead of LayerNorm backward + an autograd accumulation add).
_FUSED_RESIDUAL_GRAD = os.environ.get("MNB_FUSED_RESIDUAL_GRAD", "1") != "0"


class Block(nn.Module):
    def __init__(self, n_embd: int, n_head: int) -> None:
        super().__init__()
        self.n_head = n_head
        self.ln1 = nn.LayerNorm(n_embd)
        self.qkv = nn.Linear(n_embd, 3 * n_embd)
        self.proj = nn.Linear(n_embd, n_embd)
        self.ln2 = nn.LayerNorm(n_embd)
        self.mlp = nn.Sequential(nn.Linear(n_embd, 4 * n_embd), nn.GELU(), nn.Linear(4 * n_embd, n_embd))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda:
            return self._forward_cuda(x)
        B, T, C = x.shape
        q, k, v = self.qkv(self.ln1(x)).split(C, dim=-1)
        q, k, v = (t.view(B, T, self.n_head, C // self.n_head).transpose(1, 2) for t in (q, k, v))
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.proj(y.transpose(1, 2).reshape(B, T, C))
        return x + self.mlp(self.ln2(x))

    def _forward_cuda(self, x: torch.Tensor) -> torch.Tensor:
        K = _kernels()
        B, T, C = x.shape
        # x feeds both the norm and the residual add: LayerNormResidual hands the
        # residual branch its own alias so the two gradients meet in one kernel
        if not _FUSED_RESIDUAL_GRAD:
            return self._forward_cuda_unfused(x)
        h, x = K.LayerNormResidual.apply(x, self.ln1.weight, self.ln1.bias, self.ln1.eps)
        qkv = K.Linear.apply(h, self.qkv.weight, self.qkv.bias)
        y = K.FlashAttention.apply(qkv, self.n_head)
        x = K.Linear.apply(y.view(B, T, C), self.proj.weight, self.proj.bias, x)
        h, x = K.LayerNormResidual.apply(x, self.ln2.weight, self.ln2.bias, self.ln2.eps)
        fc, out = self.mlp[0], self.mlp[2]
        return K.MLP.apply(h, fc.weight, fc.bias, out.weight, out.bias, x)


    # ---- FSDP: the QKV projection is the block's first GEMM over its parameters --------

    def fsdp_forward_with_gathered_gemm(self, x: torch.Tensor, gather_gemm) -> torch.Tensor:
        """The CUDA forward, with the QKV GEMM computed by ``gather_gemm``.

        FullyShardedDataParallel(fuse_gather_gemm=True) passes a callable that
        runs the QKV projection as one kernel with the all-gather of this
        block's sharded parameters (its 1-D parameters -- LayerNorm scales and
        biases, linear biases -- stay whole on every rank, so LayerNorm runs
        before anything is gathered).  Every later GEMM reads the gathered
        weights.
        """
        K = _kernels()
        B, T, C = x.shape
        h, x = K.LayerNormResidual.apply(x, self.ln1.weight, self.ln1.bias, self.ln1.eps)
        qkv = K.GatheredLinear.apply(h, self.qkv.weight, self.qkv.bias, gather_gemm)
        y = K.FlashAttention.apply(qkv, self.n_head)
        x = K.Linear.apply(y.view(B, T, C), self.proj.weight, self.proj.bias, x)
        h, x = K.LayerNormResidual.apply(x, self.ln2.weight, self.ln2.bias, self.ln2.eps)
        fc, out = self.mlp[0], self.mlp[2]
        return K.MLP.apply(h, fc.weight, fc.bias, out.weight, out.bias, x)

    def fsdp_first_gemm(self) -> tuple[nn.Parameter, nn.Parameter]:
        """(weight, bias) of the first GEMM ``fsdp_forward_with_gathered_gemm`` runs."""
        return self.qkv.weight, self.qkv.bias

    def _forward_cuda_unfused(self, x: torch.Tensor) -> torch.Tensor:
        """Same block; autograd sums the residual and LayerNorm input gradients."""
        K = _kernels()
        B, T, C = x.shape
        h = K.LayerNorm.apply(x, self.ln1.weight, self.ln1.bias, self.ln1.eps)
        qkv = K.Linear.apply(h, self.qkv.weight, self.qkv.bias)
        y = K.FlashAttention.apply(qkv, self.n_head)
        x = K.Linear.apply(y.view(B, T, C), self.proj.weight, self.proj.bias, x)
        h = K.LayerNorm.apply(x, self.ln2.weight, self.ln2.bias, self.ln2.eps)
        fc, out = self.mlp[0], self.mlp[2]
        return K.MLP.apply(h, fc.weight, fc.bias, out.weight, out.bias, x)


class GPT(nn.Module):
    def __init__(self, vocab_size: int, block_size: int = 128, n_layer: int = 4, n_head: int = 4,
                 n_embd: int = 128) -> None:
        super().__init__()
        self.config = GPTConfig(vocab_size, block_size, n_layer, n_head, n_embd)
        self.block_size = block_size
        self.tok_emb = nn.Embedding(vocab_size, n_embd)
        self.pos_emb = nn.Parameter(torch.zeros(1, block_size, n_embd))
        self.blocks = nn.ModuleList(Block(n_embd, n_head) for _ in range(n_layer))
        self.ln_f = nn.LayerNorm(n_embd)
        self.head = nn.Linear(n_embd, vocab_size, bias=False)
        self.head.weight = self.tok_emb.weight
        self.apply(self._init)

    @classmethod
    def from_config(cls, cfg: GPTConfig) -> GPT:
        return cls(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)

    @staticmethod
    def _init(m: nn.Module) -> None:
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, std=0.02)
            if isinstance(m, nn.Linear) and m.bias is not None:
                nn.init.zeros_(m.bias)

    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None):
        T = idx.shape[1]
        if idx.is_cuda:
            K = _kernels()
            x = K.Embedding.apply(idx, self.tok_emb.weight, self.pos_emb[0, :T])
            for blk in self.blocks:
                x = blk(x)
            h = K.LayerNorm.apply(x, self.ln_f.weight, self.ln_f.bias, self.ln_f.eps)
            if targets is not None and torch.is_grad_enabled():
                return None, K.HeadCrossEntropy.apply(h, self.tok_emb.weight, targets)
            logits = K.Linear.apply(h, self.tok_emb.weight, None)
            loss = None
            if targets is not None:
                loss = K.CrossEntropy.apply(logits, targets)
            return logits, loss
        x = self.tok_emb(idx) + self.pos_emb[:, :T]
        for blk in self.blocks:
            x = blk(x)
        logits = self.head(self.ln_f(x))
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))
        return logits, loss

    @torch.no_grad()
    def generate(self, idx: torch.Tensor, max_new_tokens: int, temperature: float = 0.8) -> torch.Tensor:
        self.eval()
        for _ in range(max_new_tokens):
            logits, _ = self(idx[:, -self.block_size :])
            probs = F.softmax(logits[:, -1].float() / temperature, dim=-1)
            idx = torch.cat([idx, torch.multinomial(probs, 1)], dim=1)
        return idx
