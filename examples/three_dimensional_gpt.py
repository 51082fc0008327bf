"""3D parallelism: data x pipeline x tensor on one mesh.

    python examples/three_dimensional_gpt.py --world-size 8 --pp 2 --tp 2

Each rank holds one pipeline stage, one tensor shard of that stage's blocks
and belongs to one replica (reference: examples/three_dimensional_gpt.py:
56-251).  Gradients are averaged along dp only, once, after the 1F1B
schedule drains (``average_gradients``), never in a per-microbatch hook.
"""

from __future__ import annotations

import argparse
import time

import torch
import torch.nn.functional as F
from torch import nn

from _common import batch, encode, load_corpus, to_device
from tensor_parallel_gpt import ParallelBlock

import mini_nccl_b200 as mn
from mini_nccl_b200 import collectives
from mini_nccl_b200.ddp import average_gradients
from mini_nccl_b200.mesh import ParallelMesh


class Stage(nn.Module):
    def __init__(self, vocab, cfg, tp, first, last, depth):
        super().__init__()
        C = cfg["n_embd"]
        self.first, self.last = first, last
        if first:
            self.tok_emb = nn.Embedding(vocab, C)
            self.pos_emb = nn.Parameter(torch.zeros(1, cfg["block_size"], C))
            nn.init.normal_(self.tok_emb.weight, std=0.02)
        self.blocks = nn.Sequential(*[ParallelBlock(C, cfg["n_head"], tp, False) for _ in range(depth)])
        if last:
            self.ln_f = nn.LayerNorm(C)
            self.head = nn.Linear(C, vocab, bias=False)
            nn.init.normal_(self.head.weight, std=0.02)

    def forward(self, x):
        if self.first:
            x = self.tok_emb(x) + self.pos_emb[:, : x.shape[1]]
        x = self.blocks(x)
        return self.head(self.ln_f(x)) if self.last else x


def xent(logits, targets):
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))


def worker(pg, data, vocab_size, cfg):
    mesh = ParallelMesh(pg, dp=cfg["dp"], pp=cfg["pp"], tp=cfg["tp"])
    tp, pp, dp = mesh.group("tp"), mesh.group("pp"), mesh.group("dp")
    s, P = mesh.coordinate("pp"), mesh.size("pp")
    torch.manual_seed(7 + s)  # same stage weights on every replica and tp peer
    stage, dev = to_device(Stage(vocab_size, cfg, tp, s == 0, s == P - 1, cfg["n_layer"] // P), cfg["device"])
    micro = cfg["batch_size"] // cfg["microbatches"]
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    pipe = mn.PipelineParallel(stage, pp, (micro, cfg["block_size"], cfg["n_embd"]),
                               loss_fn=xent if s == P - 1 else None, dtype=dtype, device=dev)
    opt = torch.optim.AdamW(stage.parameters(), lr=cfg["lr"], betas=(0.9, 0.95))
    local = sum(p.numel() for p in stage.parameters())
    totals = collectives.all_gather(pg, torch.tensor([float(local)]))
    if pg.rank == 0:
        whole = sum(t.item() for t in totals) / mesh.size("dp")
        print(f"mesh dp={mesh.size('dp')} x pp={P} x tp={mesh.size('tp')} ({pg.world_size} ranks)\n"
              f"  {mesh.describe()}\n"
              f"  tensor group {mesh.ranks_along('tp')} | pipeline group {mesh.ranks_along('pp')} | "
              f"data group {mesh.ranks_along('dp')}\n"
              f"  per-rank params {local / 1e6:.2f}M of {whole / 1e6:.2f}M total ({whole / local:.1f}x smaller)",
              flush=True)
    B, T = cfg["batch_size"], cfg["block_size"]
    t0, loss = time.perf_counter(), 0.0
    for step in range(cfg["steps"]):
        x, y = batch(data, T, B, seed=step * mesh.size("dp") + mesh.coordinate("dp"))
        opt.zero_grad(set_to_none=True)
        loss = pipe.step(x.to(dev) if s == 0 else None, y.to(dev) if s == P - 1 else None, cfg["microbatches"])
        average_gradients(dp, list(stage.parameters()))
        opt.step()
        if s == P - 1 and mesh.coordinate("dp") == 0 and mesh.coordinate("tp") == 0 and (
                step % 20 == 0 or step == cfg["steps"] - 1):
            print(f"step {step:4d} | loss {loss:.4f} | "
                  f"{B * T * mesh.size('dp') * (step + 1) / (time.perf_counter() - t0):,.0f} tok/s", flush=True)
    if s == P - 1:
        same = collectives.all_gather(tp, torch.tensor([loss]))
        if mesh.coordinate("dp") == 0 and mesh.coordinate("tp") == 0:
            spread = max(t.item() for t in same) - min(t.item() for t in same)
            print(f"\nloss spread across the tensor group: {spread:.2e}\n"
                  f"in-flight microbatches on the last stage: {pipe.in_flight_peak}", flush=True)
    return loss


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=8)
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--batch-size", type=int, default=8, help="per replica")
    ap.add_argument("--microbatches", type=int, default=4)
    ap.add_argument("--block-size", type=int, default=64)
    ap.add_argument("--n-layer", type=int, default=4)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=128)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--data")
    args = ap.parse_args()
    if args.world_size % (args.pp * args.tp) or args.n_layer % args.pp or args.n_head % args.tp \
            or args.batch_size % args.microbatches:
        raise SystemExit("world_size % (pp*tp), n_layer % pp, n_head % tp, batch % microbatches must be 0")
    data, vocab = encode(load_corpus(args.data))
    print(f"corpus: {len(data):,} chars, vocab {len(vocab)}", flush=True)
    cfg = vars(args).copy()
    world = cfg.pop("world_size")
    cfg["dp"] = world // (args.pp * args.tp)
    cfg["sequence_parallel"] = False
    losses = mn.run(worker, world, data, len(vocab), cfg, timeout=3600.0,
                    devices="cuda" if args.device == "cuda" else None)
    print(f"final loss: {max(losses):.4f}")


if __name__ == "__main__":
    main()
