"""A GPT whose attention and MLP weights are split across ranks (Megatron TP).

    python examples/tensor_parallel_gpt.py --world-size 4 --steps 100
    python examples/tensor_parallel_gpt.py --world-size 2 --device cuda --sequence-parallel

Every rank sees the same batch and holds a different slice of every block:
attention splits by head, the MLP by hidden unit, two all-reduces per block
(reference: examples/tensor_parallel_gpt.py:44-188).  Embeddings, norms and
the tied head stay replicated and stay *bitwise* identical because every rank
receives the identical activation gradient.  ``--sequence-parallel`` keeps
the activations between TP layers split along the sequence (all-gather before
each column GEMM, reduce-scatter after each row GEMM; on GPUs each pair is one
fused kernel); LayerNorm and row-bias gradients, which then cover only local
tokens, are summed over the group after backward.
"""

from __future__ import annotations

import argparse
import time

import torch
import torch.nn.functional as F
from torch import nn

from _common import batch, encode, load_corpus, to_device

import mini_nccl_b200 as mn
from mini_nccl_b200 import collectives
from mini_nccl_b200.tensor_parallel import (
    ParallelMLP,
    ParallelSelfAttention,
    allreduce_sequence_parallel_grads,
    gather_from_sequence_parallel,
    mark_sequence_parallel,
    scatter_to_sequence_parallel,
)


class ParallelBlock(nn.Module):
    def __init__(self, width: int, n_head: int, pg, sp: bool) -> None:
        super().__init__()
        self.ln1 = nn.LayerNorm(width)
        self.attn = ParallelSelfAttention(width, n_head, pg, sequence_parallel=sp)
        self.ln2 = nn.LayerNorm(width)
        self.mlp = ParallelMLP(width, pg, sequence_parallel=sp)
        if sp:
            mark_sequence_parallel(self.ln1, self.ln2)

    def forward(self, x):
        x = self.attn(self.ln1(x), residual=x)
        return self.mlp(self.ln2(x), residual=x)


class TPGPT(nn.Module):
    def __init__(self, vocab: int, cfg: dict, pg) -> None:
        super().__init__()
        C = cfg["n_embd"]
        self.sp = cfg["sequence_parallel"]
        self.pg = pg
        self.tok_emb = nn.Embedding(vocab, C)
        self.pos_emb = nn.Parameter(torch.zeros(1, cfg["block_size"], C))
        self.blocks = nn.ModuleList(ParallelBlock(C, cfg["n_head"], pg, self.sp) for _ in range(cfg["n_layer"]))
        self.ln_f = nn.LayerNorm(C)
        nn.init.normal_(self.tok_emb.weight, std=0.02)

    def forward(self, idx, targets):
        T = idx.shape[1]
        x = self.tok_emb(idx) + self.pos_emb[:, :T]
        if self.sp:  # sequence-major, this rank's run of positions
            x = scatter_to_sequence_parallel(self.pg, x.transpose(0, 1))
        for blk in self.blocks:
            x = blk(x)
        if self.sp:  # every rank runs the replicated head on all tokens
            x = gather_from_sequence_parallel(self.pg, x).transpose(0, 1)
        logits = F.linear(self.ln_f(x), self.tok_emb.weight)
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))


def worker(pg, data, vocab_size: int, cfg: dict) -> float:
    torch.manual_seed(7)  # identical replicated weights everywhere
    model, dev = to_device(TPGPT(vocab_size, cfg, pg), cfg["device"])
    opt = torch.optim.AdamW(model.parameters(), lr=cfg["lr"], betas=(0.9, 0.95))
    local = sum(p.numel() for p in model.parameters())
    if pg.rank == 0:
        print(f"tensor parallel over {pg.world_size} ranks: {local / 1e6:.2f}M params on rank 0", flush=True)
    B, T = cfg["batch_size"], cfg["block_size"]
    t0, final = time.perf_counter(), 0.0
    for step in range(cfg["steps"]):
        x, y = batch(data, T, B, seed=step)  # same batch on every rank
        loss = model(x.to(dev), y.to(dev))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        if cfg["sequence_parallel"]:
            allreduce_sequence_parallel_grads(model, pg)
        opt.step()
        final = float(loss.detach())
        if pg.rank == 0 and (step % 20 == 0 or step == cfg["steps"] - 1):
            dt = time.perf_counter() - t0
            print(f"step {step:4d} | loss {final:.4f} | {B * T * (step + 1) / dt:,.0f} tok/s", flush=True)
    losses = collectives.all_gather(pg, torch.tensor([final]))
    spread = max(t.item() for t in losses) - min(t.item() for t in losses)
    if pg.rank == 0:
        print(f"\nloss on each rank: {[round(t.item(), 5) for t in losses]}\nmax disagreement: {spread:.2e}")
    return final


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=2)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--block-size", type=int, default=64)
    ap.add_argument("--n-layer", type=int, default=2)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=128)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--sequence-parallel", action="store_true")
    ap.add_argument("--data")
    args = ap.parse_args()
    if args.n_head % args.world_size:
        raise SystemExit("n_head must divide by world_size")
    data, vocab = encode(load_corpus(args.data))
    print(f"corpus: {len(data):,} chars, vocab {len(vocab)}", flush=True)
    cfg = vars(args).copy()
    world = cfg.pop("world_size")
    losses = mn.run(worker, world, data, len(vocab), cfg, timeout=3600.0,
                    devices="cuda" if args.device == "cuda" else None)
    print(f"final loss: {max(losses):.4f}")


if __name__ == "__main__":
    main()
