"""All-reduce sweep bootstrapped purely from the environment (multi-node contract).

Each rank is started independently (ssh, Slurm, a container per rank) with
``RANK``, ``WORLD_SIZE`` and ``MINI_NCCL_HOSTS=host:port,...`` (or under
torchrun), and ``init_process_group()`` takes no arguments
(reference: examples/multinode_allreduce.py:29-77).  CPU tensors by default;
``--device cuda`` sweeps the peer-memory kernels instead.

    MINI_NCCL_HOSTS=a:29500,b:29500 WORLD_SIZE=2 RANK=0 python examples/multinode_allreduce.py
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import mini_nccl_b200 as mn  # noqa: E402


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--max-mib", type=int, default=64)
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args()
    pg = mn.init_process_group()
    W = pg.world_size
    algos = mn.ALGORITHMS if args.device == "cpu" else mn.DEVICE_ALGORITHMS
    dev = torch.device("cuda", torch.cuda.current_device()) if args.device == "cuda" else torch.device("cpu")
    if pg.rank == 0:
        print(f"world_size={W} device={dev}\n{'bytes':>12} " + " ".join(f"{a:>14}" for a in algos), flush=True)
    size = 1024
    while size <= args.max_mib << 20:
        cells = []
        for algo in algos:
            t = torch.ones(size // 4, device=dev)
            mn.all_reduce(t, algorithm=algo)  # warm-up
            if dev.type == "cuda":
                torch.cuda.synchronize()
            mn.barrier()
            t0 = time.perf_counter()
            for _ in range(args.iters):
                mn.all_reduce(t, algorithm=algo)
            if dev.type == "cuda":
                torch.cuda.synchronize()
            dt = (time.perf_counter() - t0) / args.iters
            worst = torch.tensor([dt], dtype=torch.float64)
            mn.all_reduce(worst, op="max")
            busbw = size / worst.item() * 2 * (W - 1) / W / 1e9
            cells.append(f"{worst.item() * 1e3:8.3f}ms/{busbw:5.1f}")
        if pg.rank == 0:
            print(f"{size:>12} " + " ".join(f"{c:>14}" for c in cells), flush=True)
        size *= 4
    mn.destroy_process_group()


if __name__ == "__main__":
    main()
