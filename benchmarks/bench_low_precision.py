#!/usr/bin/env python
"""Narrow-wire all-reduce: speed and error of a bf16 wire with fp32 accumulation.

    python benchmarks/bench_low_precision.py --world-size 4 --max-mib 64

For ring and tree on the host path: time of a fp32 all-reduce with and
without ``wire_dtype=torch.bfloat16``, and the maximum error against the
exact float64 sum (reference: benchmarks/bench_low_precision.py:31-101).
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import collectives as C  # noqa: E402


def _worker(pg, sizes):
    rows = []
    W = pg.world_size
    for nbytes in sizes:
        n = nbytes // 4
        base = [torch.randn(n, generator=torch.Generator().manual_seed(r)) for r in range(W)]
        exact = sum(b.double() for b in base)
        for algo in ("ring", "tree"):
            for wire in (None, torch.bfloat16):
                t = base[pg.rank].clone()
                C.barrier(pg)
                t0 = time.perf_counter()
                C.all_reduce(pg, t, algorithm=algo, wire_dtype=wire)
                dt = time.perf_counter() - t0
                worst = torch.tensor([dt], dtype=torch.float64)
                C.all_reduce(pg, worst, op="max")
                err = float((t.double() - exact).abs().max())
                rows.append({"bytes": nbytes, "algorithm": algo, "wire": str(wire or "fp32"),
                             "ms": round(worst.item() * 1e3, 3), "max_err": err})
    return rows


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=4)
    ap.add_argument("--max-mib", type=int, default=16)
    args = ap.parse_args()
    sizes, s = [], 1 << 20
    while s <= args.max_mib << 20:
        sizes.append(s)
        s *= 4
    for row in mn.run(_worker, args.world_size, sizes, timeout=3600.0)[0]:
        print(row)


if __name__ == "__main__":
    main()
