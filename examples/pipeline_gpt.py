"""A GPT split by depth across ranks, trained with GPipe or 1F1B.

    python examples/pipeline_gpt.py --world-size 4 --microbatches 8
    python examples/pipeline_gpt.py --world-size 4 --schedule gpipe

Stage 0 owns the embeddings and the first blocks, the last stage the final
blocks, LayerNorm and head (reference: examples/pipeline_gpt.py:48-206).
Prints each stage's measured in-flight depth against the 1F1B bound ``W - s``
and the bubble fraction ``(W-1)/(M+W-1)``.
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
from mini_nccl_b200.models.gpt import Block


class FirstStage(nn.Module):
    def __init__(self, vocab, cfg, depth):
        super().__init__()
        C = cfg["n_embd"]
        self.tok_emb = nn.Embedding(vocab, C)
        self.pos_emb = nn.Parameter(torch.zeros(1, cfg["block_size"], C))
        self.blocks = nn.Sequential(*[Block(C, cfg["n_head"]) for _ in range(depth)])
        nn.init.normal_(self.tok_emb.weight, std=0.02)

    def forward(self, idx):
        return self.blocks(self.tok_emb(idx) + self.pos_emb[:, : idx.shape[1]])


class MiddleStage(nn.Module):
    def __init__(self, cfg, depth):
        super().__init__()
        self.blocks = nn.Sequential(*[Block(cfg["n_embd"], cfg["n_head"]) for _ in range(depth)])

    def forward(self, x):
        return self.blocks(x)


class LastStage(nn.Module):
    def __init__(self, vocab, cfg, depth):
        super().__init__()
        C = cfg["n_embd"]
        self.blocks = nn.Sequential(*[Block(C, cfg["n_head"]) for _ in range(depth)])
        self.ln_f = nn.LayerNorm(C)
        self.head = nn.Linear(C, vocab, bias=False)
        nn.init.normal_(self.head.weight, std=0.02)

    def forward(self, x):
        return self.head(self.ln_f(self.blocks(x)))


def build_stage(rank, world, vocab, cfg):
    depth = cfg["n_layer"] // world
    if rank == 0:
        return FirstStage(vocab, cfg, depth)
    if rank == world - 1:
        return LastStage(vocab, cfg, depth)
    return MiddleStage(cfg, depth)


def xent(logits, targets):
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))


def worker(pg, data, vocab_size, cfg):
    torch.manual_seed(11 + pg.rank)
    stage, dev = to_device(build_stage(pg.rank, pg.world_size, vocab_size, cfg), cfg["device"])
    micro = cfg["batch_size"] // cfg["microbatches"]
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    pp = mn.PipelineParallel(stage, pg, (micro, cfg["block_size"], cfg["n_embd"]),
                             loss_fn=xent if pg.rank == pg.world_size - 1 else None,
                             schedule=cfg["schedule"], dtype=dtype, device=dev)
    opt = torch.optim.AdamW(stage.parameters(), lr=cfg["lr"], betas=(0.9, 0.95))
    B, T = cfg["batch_size"], cfg["block_size"]
    t0, loss = time.perf_counter(), 0.0
    for step in range(cfg["steps"]):
        x, y = batch(data, T, B, seed=step)
        opt.zero_grad(set_to_none=True)
        loss = pp.step(x.to(dev) if pg.rank == 0 else None,
                       y.to(dev) if pg.rank == pg.world_size - 1 else None, cfg["microbatches"])
        opt.step()
        if pg.rank == pg.world_size - 1 and (step % 20 == 0 or step == cfg["steps"] - 1):
            print(f"step {step:4d} | loss {loss:.4f} | {B * T * (step + 1) / (time.perf_counter() - t0):,.0f} tok/s",
                  flush=True)
    peaks = collectives.all_gather(pg, torch.tensor([float(pp.in_flight_peak)]))
    if pg.rank == 0:
        W, M = pg.world_size, cfg["microbatches"]
        print(f"\nmicrobatches in flight per stage ({cfg['schedule']}): {[int(p.item()) for p in peaks]}"
              f"  (1F1B bound W-s: {[W - s for s in range(W)]})")
        print(f"bubble fraction (W-1)/(M+W-1) = {(W - 1) / (M + W - 1):.1%}")
    return loss


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=2)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--schedule", choices=["1f1b", "gpipe"], default="1f1b")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--batch-size", type=int, default=16)
    ap.add_argument("--microbatches", type=int, default=4)
    ap.add_argument("--block-size", type=int, default=64)
    ap.add_argument("--n-layer", type=int, default=4)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=128)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--data")
    args = ap.parse_args()
    if args.n_layer % args.world_size or args.batch_size % args.microbatches:
        raise SystemExit("n_layer must divide by world_size and batch_size by microbatches")
    data, vocab = encode(load_corpus(args.data))
    print(f"corpus: {len(data):,} chars, vocab {len(vocab)}", flush=True)
    cfg = vars(args).copy()
    world = cfg.pop("world_size")
    mn.run(worker, world, data, len(vocab), cfg, timeout=3600.0, devices="cuda" if args.device == "cuda" else None)
    print("done")


if __name__ == "__main__":
    main()
