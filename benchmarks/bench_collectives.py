#!/usr/bin/env python
"""Collective sweep on GPUs: this library's peer-memory kernels vs NCCL.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \\
        --master-addr 127.0.0.1 --master-port 29700 benchmarks/bench_collectives.py \\
        --min-bytes 4096 --max-bytes 1073741824 --out results/collectives_w8.csv

For every op (all_reduce per algorithm, reduce_scatter, all_gather,
broadcast, all_to_all), dtype (fp32, bf16, and fp32 with a bf16 wire) and
message size (powers of ``--size-factor``, default 2), each rank times
``--iters`` back-to-back calls with CUDA events after ``--warmup`` calls;
the reported time is the **max over ranks** and bus bandwidth follows nccl-tests
(``busbw = algbw * 2(W-1)/W`` for all-reduce, ``(W-1)/W`` for reduce-scatter,
all-gather and all-to-all, ``1`` for broadcast).  Messages are larger than L2
above 128 MiB; below that the same buffer is reused (as nccl-tests does).
NCCL runs through torch.distributed on the same tensors.  ``--reference``
adds the reference's own GPU entry point (``mini_nccl.device.all_reduce_staged``
from baseline/_ref) for all-reduce up to ``--reference-max-bytes``.
``two_shot_sym`` is the two-shot all-reduce on a tensor in symmetric memory
(every peer has it mapped, like a DDP gradient bucket): results are stored
straight into every rank's copy, with no copy-out (NCCL's counterpart is a
registered user buffer).  ``nvls`` reduces through the NVSwitch (multimem
loads and stores) via a staging buffer; ``nvls_sym`` does it in place on a
tensor bound to the multicast object (how DDP's buckets are reduced).
Reduce-scatter, all-gather and broadcast are timed on both of this
library's paths: ``direct`` (peer stores) and ``nvls``.
Rank 0 prints one JSON line per measurement and writes the CSV.
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import collectives as C  # noqa: E402

BUS = {"all_reduce": lambda W: 2 * (W - 1) / W, "reduce_scatter": lambda W: (W - 1) / W,
       "all_gather": lambda W: (W - 1) / W, "all_to_all": lambda W: (W - 1) / W, "broadcast": lambda W: 1.0}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--min-bytes", type=int, default=4096)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--size-factor", type=int, default=2, help="ratio of consecutive message sizes")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--ops", default="all_reduce,reduce_scatter,all_gather,broadcast,all_to_all")
    ap.add_argument("--algorithms", default="auto,one_shot,two_shot,two_shot_sym,nvls,nvls_sym,ring,tree,halving,naive")
    ap.add_argument("--dtypes", default="float32,bfloat16,float32+bf16wire")
    ap.add_argument("--no-nccl", action="store_true")
    ap.add_argument("--reference", action="store_true")
    ap.add_argument("--reference-max-bytes", type=int, default=64 << 20)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = mn.init_process_group(rank, world, device=dev, op_timeout=120.0)
    if not args.no_nccl:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    ref_pg = None
    if args.reference:
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        import mini_nccl as rmn  # the unmodified reference package
        from mini_nccl import device as rdev

        ports = [p for p in C.all_gather(pg, torch.tensor([mn.launcher._free_ports(1)[0]]))]
        ref_pg = rmn.ProcessGroup(rank, world, addrs=[("127.0.0.1", int(p.item())) for p in ports])

    def reduce_max(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64)
        C.all_reduce(pg, t, op="max")
        return float(t.item())

    def time_it(fn) -> float:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        C.barrier(pg)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return reduce_max(s.elapsed_time(e) / args.iters)

    rows = []
    sym_bufs: dict = {}
    dc = pg.device_comm()
    nvls_paths = ("direct", "nvls") if dc.nvls else ("direct",)
    if rank == 0:
        print(json.dumps({"nvls": dc.nvls, "nvls_reason": dc.nvls_reason}), flush=True)

    def sym_view(dtype, n, nvls=False):
        key = (dtype, nvls)
        buf = sym_bufs.get(key)
        if buf is None:
            numel = args.max_bytes // torch.empty(0, dtype=dtype).element_size()
            buf = sym_bufs[key] = dc.symmetric_zeros(numel, dtype, nvls=nvls)
        return buf[:n]

    def record(op, impl, algo, dtype, nbytes, ms):
        algbw = nbytes / (ms / 1e3) / 1e9
        row = {"op": op, "impl": impl, "algorithm": algo, "dtype": dtype, "bytes": nbytes, "world": world,
               "ms": round(ms, 5), "algbw_GBs": round(algbw, 2), "busbw_GBs": round(algbw * BUS[op](world), 2)}
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)

    dtypes = {"float32": (torch.float32, None), "bfloat16": (torch.bfloat16, None),
              "float32+bf16wire": (torch.float32, torch.bfloat16)}
    ops = args.ops.split(",")
    size = args.min_bytes
    while size <= args.max_bytes:
        for dname in args.dtypes.split(","):
            dtype, wire = dtypes[dname]
            n = size // torch.empty(0, dtype=dtype).element_size()
            n -= n % world
            if n == 0:
                continue
            x = torch.randn(n, device=dev).to(dtype)
            for op in ops:
                if wire is not None and op != "all_reduce":
                    continue
                if op == "all_reduce":
                    for algo in args.algorithms.split(","):
                        if algo in ("nvls", "nvls_sym") and (not dc.nvls or wire is not None):
                            continue
                        if algo in ("two_shot_sym", "nvls_sym"):
                            if wire is None:
                                sv = sym_view(dtype, n, nvls=algo == "nvls_sym")
                                sv.copy_(x)
                                a = algo[: -len("_sym")]
                                record(op, "ours", algo, dname, size,
                                       time_it(lambda a=a: dc.all_reduce(sv, algorithm=a)))
                            continue
                        if algo == "halving" and world & (world - 1):
                            continue
                        if algo in ("ring", "tree", "halving", "naive") and size > (256 << 20):
                            continue  # step-by-step parity schedules: keep the sweep bounded
                        record(op, "ours", algo, dname, size,
                               time_it(lambda a=algo: C.all_reduce(pg, x, algorithm=a, wire_dtype=wire)))
                    if not args.no_nccl and wire is None:
                        record(op, "nccl", "nccl", dname, size, time_it(lambda: dist.all_reduce(x)))
                    if ref_pg is not None and wire is None and size <= args.reference_max_bytes:
                        record(op, "reference", "staged-ring", dname, size,
                               time_it(lambda: rdev.all_reduce_staged(ref_pg, x)))
                elif op == "reduce_scatter":
                    for path in nvls_paths:
                        record(op, "ours", path, dname, size,
                               time_it(lambda p=path: dc.reduce_scatter(x, algorithm=p)))
                    if not args.no_nccl:
                        o = torch.empty(n // world, dtype=dtype, device=dev)
                        record(op, "nccl", "nccl", dname, size,
                               time_it(lambda: dist.reduce_scatter_tensor(o, x)))
                elif op == "all_gather":
                    shard = x[: n // world]
                    out = torch.empty(n, dtype=dtype, device=dev)
                    for path in nvls_paths:
                        if path == "nvls" and (shard.numel() * shard.element_size()) % 16:
                            continue
                        record(op, "ours", path, dname, size,
                               time_it(lambda p=path: dc.all_gather(shard, out.view(world, -1), algorithm=p)))
                    if not args.no_nccl:
                        record(op, "nccl", "nccl", dname, size,
                               time_it(lambda: dist.all_gather_into_tensor(out, shard)))
                elif op == "broadcast":
                    for path in nvls_paths:
                        if path == "nvls" and size % 16:
                            continue
                        record(op, "ours", path, dname, size,
                               time_it(lambda p=path: dc.broadcast(x, src=0, algorithm=p)))
                    if not args.no_nccl:
                        record(op, "nccl", "nccl", dname, size, time_it(lambda: dist.broadcast(x, src=0)))
                elif op == "all_to_all":
                    record(op, "ours", "direct", dname, size, time_it(lambda: C.all_to_all(pg, x)))
                    if not args.no_nccl:
                        o = torch.empty_like(x)
                        record(op, "nccl", "nccl", dname, size, time_it(lambda: dist.all_to_all_single(o, x)))
            del x
        size *= args.size_factor
    pg.device_comm().synchronize()
    if rank == 0 and args.out:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        with open(args.out, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=list(rows[0]))
            w.writeheader()
            w.writerows(rows)
    if not args.no_nccl:
        dist.destroy_process_group()
    if ref_pg is not None:
        ref_pg.close()
    mn.destroy_process_group()


if __name__ == "__main__":
    main()
