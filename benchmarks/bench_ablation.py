#!/usr/bin/env python
"""Channel and slice ablation of the host ring all-reduce.

    python benchmarks/bench_ablation.py --world-size 4 --out results/ablation.csv

``MINI_NCCL_CHANNEL_MIN_BYTES`` and ``MINI_NCCL_MAX_SLICES`` are read when
``mini_nccl_b200.collectives`` is imported, so every (channels, slices)
setting runs in a fresh interpreter (reference: benchmarks/bench_ablation.py:
33-54).  The device path's counterpart of "channels" is the CTA count, swept
by ``MINI_NCCL_DEVICE_BLOCKS`` with benchmarks/bench_collectives.py.
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent



def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=4)
    ap.add_argument("--channels", type=int, nargs="+", default=[1, 2, 4, 8])
    ap.add_argument("--slices", type=int, nargs="+", default=[1, 16])
    ap.add_argument("--sizes-mib", type=int, nargs="+", default=[1, 4, 16, 64])
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--out")
    args = ap.parse_args()
    rows = []
    for ch in args.channels:
        for sl in args.slices:
            env = dict(os.environ, MINI_NCCL_CHANNEL_MIN_BYTES=str(1 << 20), MINI_NCCL_MAX_SLICES=str(sl))
            cfg = {"world": args.world_size, "channels": ch, "iters": args.iters,
                   "sizes": [m << 20 for m in args.sizes_mib]}
            proc = subprocess.run([sys.executable, str(ROOT / "benchmarks" / "_ablation_worker.py"), json.dumps(cfg)],
                                  env=env, capture_output=True, text=True, check=True)
            for nbytes, sec in json.loads(proc.stdout.strip().splitlines()[-1]):
                W = args.world_size
                row = {"world": W, "channels": ch, "slices": sl, "bytes": nbytes, "ms": round(sec * 1e3, 3),
                       "busbw_GBs": round(nbytes / sec * 2 * (W - 1) / W / 1e9, 4)}
                rows.append(row)
                print(row, flush=True)
    if args.out:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        with open(args.out, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(rows[0]))
            w.writeheader()
            w.writerows(rows)


if __name__ == "__main__":
    main()
