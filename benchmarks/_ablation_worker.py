"""One (channels, slices) setting of bench_ablation.py, in a fresh interpreter.

The environment knobs are read when the collectives module is imported, so
each setting needs its own process; spawned ranks re-import this file.
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import collectives as C  # noqa: E402


def body(pg, sizes, iters):
    out = []
    for nbytes in sizes:
        t = torch.ones(nbytes // 4)
        C.all_reduce(pg, t, algorithm="ring")
        C.barrier(pg)
        t0 = time.perf_counter()
        for _ in range(iters):
            C.all_reduce(pg, t, algorithm="ring")
        dt = torch.tensor([(time.perf_counter() - t0) / iters], dtype=torch.float64)
        C.all_reduce(pg, dt, op="max")
        out.append((nbytes, dt.item()))
    return out


if __name__ == "__main__":
    cfg = json.loads(sys.argv[1])
    res = mn.run(body, cfg["world"], cfg["sizes"], cfg["iters"], n_channels=cfg["channels"], timeout=3600.0)[0]
    print(json.dumps(res))
