"""2D parallelism: tensor parallel inside groups, data parallel across them.

    python examples/two_dimensional_gpt.py --world-size 4 --tp 2

``ParallelMesh(pg, dp=W/tp, tp=tp)``: TP blocks run on this rank's tp
sub-group, DDP averages gradients over its dp sub-group (reference:
examples/two_dimensional_gpt.py:50-199).  Replicas (dp coordinates) sample
different data; ranks inside a tp group share a batch and must report the
same loss.
"""

from __future__ import annotations

import argparse
import time

import torch

from _common import batch, encode, load_corpus, to_device
from tensor_parallel_gpt import TPGPT

import mini_nccl_b200 as mn
from mini_nccl_b200 import collectives
from mini_nccl_b200.mesh import ParallelMesh


def worker(pg, data, vocab_size, cfg):
    mesh = ParallelMesh(pg, dp=pg.world_size // cfg["tp"], tp=cfg["tp"])
    tp, dp = mesh.group("tp"), mesh.group("dp")
    torch.manual_seed(7)
    model, dev = to_device(TPGPT(vocab_size, cfg, tp), cfg["device"])
    ddp = mn.DistributedDataParallel(model, dp, bucket_cap_mb=1.0)
    opt = torch.optim.AdamW(model.parameters(), lr=cfg["lr"], betas=(0.9, 0.95))
    if pg.rank == 0:
        print(f"mesh dp={mesh.size('dp')} x tp={mesh.size('tp')} | {mesh.describe()} | "
              f"tensor group {mesh.ranks_along('tp')} | data group {mesh.ranks_along('dp')}", flush=True)
    B, T = cfg["batch_size"], cfg["block_size"]
    t0, loss = time.perf_counter(), None
    for step in range(cfg["steps"]):
        x, y = batch(data, T, B, seed=step * mesh.size("dp") + mesh.coordinate("dp"))
        ddp.zero_grad()
        loss = ddp(x.to(dev), y.to(dev))
        loss.backward()
        ddp.sync()
        opt.step()
        if pg.rank == 0 and (step % 20 == 0 or step == cfg["steps"] - 1):
            print(f"step {step:4d} | loss {float(loss):.4f} | "
                  f"{B * T * mesh.size('dp') * (step + 1) / (time.perf_counter() - t0):,.0f} tok/s", flush=True)
    same = collectives.all_gather(tp, torch.tensor([float(loss)]))
    spread = max(t.item() for t in same) - min(t.item() for t in same)
    if pg.rank == 0:
        print(f"\nloss across the tensor group: {[round(t.item(), 5) for t in same]} (spread {spread:.2e})")
    return float(loss)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=4)
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--block-size", type=int, default=64)
    ap.add_argument("--n-layer", type=int, default=2)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=128)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--data")
    args = ap.parse_args()
    if args.world_size % args.tp or args.n_head % args.tp:
        raise SystemExit("world_size and n_head must divide by tp")
    data, vocab = encode(load_corpus(args.data))
    print(f"corpus: {len(data):,} chars, vocab {len(vocab)}", flush=True)
    cfg = vars(args).copy()
    cfg["sequence_parallel"] = False
    world = cfg.pop("world_size")
    losses = mn.run(worker, world, data, len(vocab), cfg, timeout=3600.0,
                    devices="cuda" if args.device == "cuda" else None)
    print(f"final loss: {max(losses):.4f}")


if __name__ == "__main__":
    main()
