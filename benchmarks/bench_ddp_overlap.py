#!/usr/bin/env python
"""DDP step time with the gradient reduction overlapped with backward vs not.

    python benchmarks/bench_ddp_overlap.py --world-size 2                 # CPU ranks, TCP
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29800 benchmarks/bench_ddp_overlap.py --device cuda  # GPUs, peer memory

Same model and data both ways; the only difference is ``overlap=``
(reference: benchmarks/bench_ddp_overlap.py:26-90).  On GPUs the overlapped
reducer launches each bucket's all-reduce on a side stream as soon as the
bucket's gradients exist, so the interesting number is how much of the
communication disappears under backward.
"""

from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import nn

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import mini_nccl_b200 as mn  # noqa: E402


def build(width: int, depth: int, dev, dtype) -> nn.Module:
    torch.manual_seed(0)
    layers = []
    for _ in range(depth):
        layers += [nn.Linear(width, width), nn.Tanh()]
    return nn.Sequential(*layers, nn.Linear(width, 1)).to(dev, dtype)


def measure(pg, overlap: bool, args, dev, dtype) -> float:
    model = build(args.width, args.depth, dev, dtype)
    ddp = mn.DistributedDataParallel(model, pg, bucket_cap_mb=args.bucket_mb, overlap=overlap, algorithm="auto")
    x = torch.randn(args.batch, args.width, device=dev, dtype=dtype)
    y = torch.randn(args.batch, 1, device=dev, dtype=dtype)

    def step():
        ddp.zero_grad()
        F.mse_loss(ddp(x), y).backward()
        ddp.sync()

    for _ in range(3):
        step()
    if dev.type == "cuda":
        torch.cuda.synchronize()
    mn.collectives.barrier(pg)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    if dev.type == "cuda":
        torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / args.steps
    worst = torch.tensor([dt], dtype=torch.float64)
    mn.collectives.all_reduce(pg, worst, op="max")
    return worst.item()


def _worker(pg, args):
    dev = torch.device("cuda", torch.cuda.current_device()) if args.device == "cuda" else torch.device("cpu")
    dtype = torch.bfloat16 if args.device == "cuda" else torch.float32
    on, off = measure(pg, True, args, dev, dtype), measure(pg, False, args, dev, dtype)
    if pg.rank == 0:
        print(f"world={pg.world_size} device={dev} step: overlap {on * 1e3:.2f} ms | no overlap {off * 1e3:.2f} ms | "
              f"gain {off / on:.3f}x", flush=True)
    return on, off


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=2)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--width", type=int, default=1024)
    ap.add_argument("--depth", type=int, default=16)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--bucket-mb", type=float, default=4.0)
    ap.add_argument("--steps", type=int, default=20)
    args = ap.parse_args()
    if "RANK" in os.environ:  # torchrun
        pg = mn.init_process_group()
        _worker(pg, args)
        mn.destroy_process_group()
    else:
        mn.run(_worker, args.world_size, args, timeout=3600.0, devices="cuda" if args.device == "cuda" else None)


if __name__ == "__main__":
    main()
