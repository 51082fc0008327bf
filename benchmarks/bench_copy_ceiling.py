#!/usr/bin/env python
"""What the host-staged device path can reach at best: D2H / H2D copy bandwidth.

    python benchmarks/bench_copy_ceiling.py --max-mib 256

Pinned vs pageable host memory, both directions, CUDA events, best of
``--iters`` (reference: benchmarks/bench_copy_ceiling.py:27-96).  On one
NVSwitch box the library never stages through the host; this bounds the
cross-host path (``device.all_reduce_staged`` / ``all_reduce_pipelined``).
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--max-mib", type=int, default=256)
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    size = 1 << 20
    while size <= args.max_mib << 20:
        d = torch.empty(size, dtype=torch.uint8, device=dev)
        for pinned in (True, False):
            h = torch.empty(size, dtype=torch.uint8, pin_memory=pinned)
            for direction in ("d2h", "h2d"):
                best = float("inf")
                for _ in range(args.iters):
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    (h.copy_(d, non_blocking=pinned) if direction == "d2h" else d.copy_(h, non_blocking=pinned))
                    e.record()
                    torch.cuda.synchronize()
                    best = min(best, s.elapsed_time(e))
                print(json.dumps({"bytes": size, "pinned": pinned, "direction": direction, "ms": round(best, 4),
                                  "GBs": round(size / best / 1e6, 2)}), flush=True)
        size *= 4


if __name__ == "__main__":
    main()
