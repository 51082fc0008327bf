#!/usr/bin/env python
"""All-reduce of CUDA tensors three ways: the reference's host-staged schemes vs peer memory.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29720 benchmarks/bench_device.py --max-mib 64

* ``staged``    -- whole tensor to pinned host memory, host ring, back
                   (``device.all_reduce_staged``, the reference's baseline);
* ``pipelined`` -- host ring with chunked copies overlapped with the wire and
                   the reduction on the device (``device.all_reduce_pipelined``);
* ``peer``      -- one kernel over NVLink peer memory (``all_reduce`` on a CUDA
                   tensor).
CUDA events around each call, max over ranks (reference: benchmarks/
bench_device.py:40-78).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import device as D  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--max-mib", type=int, default=64)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    pg = mn.init_process_group(rank, world, device=dev, op_timeout=300.0)
    impls = {
        "staged": lambda t: D.all_reduce_staged(pg, t),
        "pipelined": lambda t: D.all_reduce_pipelined(pg, t),
        "peer": lambda t: mn.collectives.all_reduce(pg, t),
    }
    size = 1 << 20
    while size <= args.max_mib << 20:
        t = torch.randn(size // 4, device=dev)
        for name, fn in impls.items():
            fn(t)
            torch.cuda.synchronize()
            mn.collectives.barrier(pg)
            t0 = time.perf_counter()
            for _ in range(args.iters):
                fn(t)
            torch.cuda.synchronize()
            dt = torch.tensor([(time.perf_counter() - t0) / args.iters], dtype=torch.float64)
            mn.collectives.all_reduce(pg, dt, op="max")
            if rank == 0:
                print(json.dumps({"bytes": size, "impl": name, "world": world, "ms": round(dt.item() * 1e3, 3),
                                  "busbw_GBs": round(size / dt.item() * 2 * (world - 1) / world / 1e9, 3)}),
                      flush=True)
        size *= 4
    pg.device_comm().synchronize()
    mn.destroy_process_group()


if __name__ == "__main__":
    main()
