#!/usr/bin/env python
"""Host-path all-reduce sweep (CPU tensors over the native TCP mesh).

    python benchmarks/bench_allreduce.py --world-sizes 2 4 --max-mib 64 --out results/allreduce.csv

nccl-tests style: each rank times ``--iters`` calls after a warm-up, the
reported time is the max over ranks, ``busbw = algbw * 2(W-1)/W``
(reference: benchmarks/bench_allreduce.py:10-144).  ``--gloo`` adds
torch.distributed's gloo all-reduce on the same tensors for comparison.
GPU tensors are covered by benchmarks/bench_collectives.py.
"""

from __future__ import annotations

import argparse
import csv
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import collectives as C  # noqa: E402


def _worker(pg, sizes, iters, gloo_port):
    rows = []
    gloo = None
    if gloo_port:
        import torch.distributed as dist

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{gloo_port}", rank=pg.rank,
                                world_size=pg.world_size)
        gloo = dist
    W = pg.world_size
    for nbytes in sizes:
        t = torch.ones(max(1, nbytes // 4))
        impls = [(a, lambda a=a: C.all_reduce(pg, t, algorithm=a)) for a in mn.ALGORITHMS]
        if gloo is not None:
            impls.append(("gloo", lambda: gloo.all_reduce(t)))
        for name, fn in impls:
            fn()
            C.barrier(pg)
            t0 = time.perf_counter()
            for _ in range(iters):
                fn()
            dt = (time.perf_counter() - t0) / iters
            worst = torch.tensor([dt], dtype=torch.float64)
            C.all_reduce(pg, worst, op="max")
            s = worst.item()
            rows.append({"world": W, "bytes": nbytes, "algorithm": name, "ms": round(s * 1e3, 4),
                         "busbw_GBs": round(nbytes / s * 2 * (W - 1) / W / 1e9, 4)})
    if gloo is not None:
        gloo.destroy_process_group()
    return rows if pg.rank == 0 else []


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-sizes", type=int, nargs="+", default=[2, 4])
    ap.add_argument("--min-kib", type=int, default=4)
    ap.add_argument("--max-mib", type=int, default=64)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--channels", type=int, default=2)
    ap.add_argument("--gloo", action="store_true")
    ap.add_argument("--out")
    args = ap.parse_args()
    sizes, s = [], args.min_kib * 1024
    while s <= args.max_mib << 20:
        sizes.append(s)
        s *= 4
    rows = []
    for W in args.world_sizes:
        port = mn.launcher._free_ports(1)[0] if args.gloo else 0
        rows += mn.run(_worker, W, sizes, args.iters, port, n_channels=args.channels, timeout=3600.0)[0]
    for r in rows:
        print(r)
    if args.out:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        with open(args.out, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(rows[0]))
            w.writeheader()
            w.writerows(rows)


if __name__ == "__main__":
    main()
