#!/usr/bin/env python
"""Fused GEMM + collective kernels vs the same work unfused, and vs cuBLAS + NCCL.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29710 benchmarks/bench_fused_tp.py --out results/fused_tp_w2.jsonl
    python benchmarks/bench_fused_tp.py --single --iters 1 --warmup 1   # one GPU (ncu capture)

Shapes are the tensor-parallel GEMMs of the 3D config (GPT d_model 4096,
32 heads, micro-batch 2 x seq 2048 = 4096 tokens, TP=W):

* ``rs_proj`` / ``rs_fc2``: row-parallel GEMM -> reduce-scatter
  (x [4096, 4096/W or 16384/W] @ W^T -> this rank's [4096/W, 4096]);
* ``ag_qkv`` / ``ag_fc1``: all-gather -> column-parallel GEMM
  (x_shard [4096/W, 4096] -> gathered [4096, 4096] @ W^T, N = 12288/W or 16384/W).

Three implementations per shape, timed with CUDA events over back-to-back
calls (warm-up; an L2 flush enqueued before every call and its time
subtracted), max over ranks:

* ``fused``   : one kernel (``DeviceComm.gemm_reduce_scatter`` / ``all_gather_gemm``);
* ``ours``    : our GEMM kernel and our collective kernel, back to back;
* ``nccl``    : ``torch.matmul`` (cuBLAS) and NCCL through torch.distributed.

The roofline of a fused call is the slower of its FLOPs at the measured
bf16 GEMM peak and the bytes it must move over NVLink per rank at the
measured 770 GB/s per direction: achieved = target / measured time.
``--single`` runs the fused kernels on one GPU (the collective degenerates to
a local copy), which is what an ncu capture can see.
"""

from __future__ import annotations

import argparse
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
from mini_nccl_b200.ops import kernels as K  # noqa: E402

NVLINK_GBS = 770.0


def peak_tflops() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    return float(json.loads(p.read_text())["bf16_tflops"]) if p.exists() else 1590.0


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--width", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--cases", default="rs_proj,rs_fc2,ag_qkv,ag_fc1")
    ap.add_argument("--single", action="store_true", help="one GPU, fused kernels only")
    ap.add_argument("--shape-world", type=int, default=0,
                    help="size the GEMMs as for this TP degree (default: the real world size)")
    ap.add_argument("--out")
    args = ap.parse_args()

    if args.single:
        rank, world = 0, 1
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        pg = mn.init_process_group(0, 1, device=dev)
    else:
        rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
        torch.cuda.set_device(dev)
        pg = mn.init_process_group(rank, world, device=dev, op_timeout=120.0)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    dc = pg.device_comm()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    bf = torch.bfloat16
    M, C = args.tokens, args.width
    W = world
    SW = args.shape_world or world  # TP degree the shapes are cut for

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev) * scale).to(bf)

    local_ms: list[float] = []

    def reduce_max(v: float) -> float:
        local_ms.append(v)
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        mn.collectives.all_reduce(pg, t, op="max")
        return float(t.item())

    def reduce_min(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        mn.collectives.all_reduce(pg, t, op="min")
        return float(t.item())

    def timed(fn) -> float:
        """Back-to-back calls on the stream with an L2 flush enqueued before each
        (no host synchronisation in between, as nccl-tests times); the flushes,
        timed alone the same way, are subtracted.  Max over ranks."""
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            mn.collectives.barrier(pg)

        def run(with_fn: bool) -> float:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.iters):
                flush.zero_()
                if with_fn:
                    fn()
            e.record()
            torch.cuda.synchronize()
            return s.elapsed_time(e)

        flush_only = run(False)
        both = run(True)
        return reduce_max(max(0.0, both - flush_only) / args.iters)

    peak = peak_tflops()
    rows = []
    for case in args.cases.split(","):
        if case.startswith("rs"):
            Kl = (C if case == "rs_proj" else 4 * C) // SW
            N = C
            x, w, bias = rnd(M, Kl, scale=0.5), rnd(N, Kl, scale=0.02), rnd(N)
            resid = rnd(M // W, N)
            flops = 2.0 * M * N * Kl
            nvlink = (W - 1) / W * M * N * 2
            impls = {"fused": lambda: dc.gemm_reduce_scatter(x, w, bias=bias, resid=resid, force_kernel=True)}
            if world == 1:
                impls["gemm_only"] = lambda: K.gemm(x, w, bias=bias)
            if world > 1:
                def ours():
                    y = K.gemm(x, w)
                    part = dc.reduce_scatter(y.view(-1)).view(M // W, N)
                    return part + bias + resid

                def nccl():
                    y = torch.matmul(x, w.t())
                    part = torch.empty(M // W, N, dtype=bf, device=dev)
                    dist.reduce_scatter_tensor(part, y)
                    return part + bias + resid

                impls.update(ours=ours, nccl=nccl)
        else:
            N = (3 * C if case == "ag_qkv" else 4 * C) // SW
            Kd = C
            xs, w, bias = rnd(M // W, Kd, scale=0.5), rnd(N, Kd, scale=0.02), rnd(N)
            gathered = torch.empty(M, Kd, dtype=bf, device=dev)
            flops = 2.0 * M * N * Kd
            nvlink = (W - 1) / W * M * Kd * 2
            impls = {"fused": lambda: dc.all_gather_gemm(xs, w, bias=bias, gathered=gathered, force_kernel=True)}
            if world == 1:
                impls["gemm_only"] = lambda: K.gemm(xs, w, bias=bias)
            if world > 1:
                def ours():
                    full = dc.all_gather(xs.view(-1)).view(M, Kd)
                    return K.gemm(full, w, bias=bias)

                def nccl():
                    dist.all_gather_into_tensor(gathered, xs)
                    return torch.addmm(bias, gathered, w.t())

                impls.update(ours=ours, nccl=nccl)
        target_ms = max(flops / (peak * 1e12), nvlink / (NVLINK_GBS * 1e9)) * 1e3
        for name, fn in impls.items():
            ms = timed(fn)
            fastest = reduce_min(local_ms[-1])
            row = {"case": case, "impl": name, "world": world, "M": M, "N": N, "K": Kl if case.startswith("rs") else Kd,
                   "ms": round(ms, 4), "ms_fastest_rank": round(fastest, 4), "tflops": round(flops / ms / 1e9, 1),
                   "nvlink_GB_per_rank": round(nvlink / 1e9, 4), "roofline_ms": round(target_ms, 4),
                   "frac_of_roofline": round(target_ms / ms, 3),
                   "peaks": f"bf16 {peak} TFLOP/s (measured), NVLink {NVLINK_GBS} GB/s per direction (measured)"}
            if name == "fused" and case.startswith("rs"):
                # five back-to-back calls (flush between) with phase stamps:
                # per call [start - previous call's end, tiles done, all tiles seen, reduced] in us
                st = torch.zeros(5, 4, dtype=torch.int64, device=dev)
                torch.cuda.synchronize()
                if world > 1:
                    mn.collectives.barrier(pg)
                for i in range(5):
                    flush.zero_()
                    dc.gemm_reduce_scatter(x, w, bias=bias, resid=resid, force_kernel=True, stamps=st[i])
                torch.cuda.synchronize()
                t = st.cpu().tolist()
                phases = []
                for i in range(5):
                    gap = (t[i][0] - t[i - 1][3]) / 1e3 if i else 0.0
                    phases += [round(gap, 1)] + [round((t[i][k] - t[i][0]) / 1e3, 1) for k in (1, 2, 3)]
                allp = mn.collectives.all_gather(pg, torch.tensor(phases)) if world > 1 else [torch.tensor(phases)]
                row["phases_us_per_rank"] = [p.view(5, 4).tolist() for p in allp]
            rows.append(row)
            if rank == 0:
                print(json.dumps(row), flush=True)
    dc.synchronize()
    K.check_status(dev)
    if rank == 0 and args.out:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        with open(args.out, "w") as fh:
            for r in rows:
                fh.write(json.dumps(r) + "\n")
    if world > 1:
        dist.destroy_process_group()
    mn.destroy_process_group()


if __name__ == "__main__":
    main()
