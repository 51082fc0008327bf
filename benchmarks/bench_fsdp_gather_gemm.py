#!/usr/bin/env python
"""FSDP's parameter all-gather fused into the unit's first GEMM, vs unfused and vs NCCL + cuBLAS.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29720 benchmarks/bench_fsdp_gather_gemm.py --out results/fsdp_gather_gemm_w8.jsonl

Shapes are one transformer block of the FSDP config (d_model 2048, micro-
batch 4 x seq 2048 = 8192 tokens): the block's 2-D weights flattened
(12 d^2 = 50.3 M bf16 parameters; its 1-D parameters stay whole on every
rank in the fused mode), sharded W ways, and the QKV projection
x [8192, 2048] @ W_qkv^T, W_qkv = the first [6144, 2048] of the buffer.

* ``fused`` : one kernel, ``DeviceComm.gather_weight_gemm`` (gather warps copy
  the buffer in, QKV rows first; tiles start as their rows arrive);
* ``ours``  : this library's all-gather kernel, then its GEMM kernel;
* ``nccl``  : NCCL all-gather (torch.distributed), then ``torch.matmul`` (cuBLAS).

``--single`` runs the fused kernel on one GPU (the gather copies the own
shard only), which is what an ncu capture can see:

    python benchmarks/bench_fsdp_gather_gemm.py --single --iters 1 --warmup 1

Each is timed with CUDA events over ``--iters`` calls after ``--warmup``,
with a >126 MB L2 flush enqueued before every call and its own time
subtracted; the reported time is the max over ranks.  The roofline target is
the slower of the GEMM at the measured bf16 peak and the (W-1)/W of the
buffer that must arrive over NVLink at the measured 770 GB/s per direction.
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
    ap.add_argument("--width", type=int, default=2048)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impls", default="fused,ours,nccl")
    ap.add_argument("--single", action="store_true", help="one GPU, the fused kernel only (for ncu)")
    ap.add_argument("--out")
    args = ap.parse_args()

    if args.single:
        os.environ.update(RANK="0", WORLD_SIZE="1", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=os.environ.get("MASTER_PORT", "29731"))
        args.impls = "fused"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    pg = mn.init_process_group(rank, world, device=dev, op_timeout=120.0)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    dc = pg.device_comm()

    C = args.width
    flat_n = 12 * C * C
    quantum = 8 * world
    flat_n = -(-flat_n // quantum) * quantum
    shard_n = flat_n // world
    N = 3 * C
    g = torch.Generator().manual_seed(rank)
    shard = dc.symmetric_zeros(shard_n, torch.bfloat16)
    shard.copy_((torch.randn(shard_n, generator=g) * 0.02).to(torch.bfloat16))
    plain_shard = shard.clone()
    x = torch.randn(args.tokens, C, generator=g).to(dev, torch.bfloat16)
    bias = torch.zeros(N, dtype=torch.bfloat16, device=dev)
    flat = torch.empty(flat_n, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def fused():
        return dc.gather_weight_gemm(x, shard, flat, 0, N, bias=bias)

    def ours():
        dc.all_gather(shard, flat.view(world, -1))
        return K.gemm(x, flat[: N * C].view(N, C), bias=bias)

    def nccl():
        dist.all_gather_into_tensor(flat, plain_shard)
        return torch.addmm(bias, x, flat[: N * C].view(N, C).t())

    def reduce_max(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_it(fn) -> float:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.iters):
            flush.fill_(1)
        e0.record()
        torch.cuda.synchronize()
        flush_ms = s0.elapsed_time(e0) / args.iters
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            flush.fill_(1)
            fn()
        e.record()
        torch.cuda.synchronize()
        return reduce_max(s.elapsed_time(e) / args.iters - flush_ms)

    want = nccl()
    got = fused()
    torch.cuda.synchronize()
    err = (got.float() - want.float()).abs().max().item()
    flops = 2.0 * args.tokens * N * C
    arrive_bytes = (world - 1) / world * flat_n * 2
    target_ms = max(flops / (peak_tflops() * 1e12), arrive_bytes / (NVLINK_GBS * 1e9)) * 1e3
    rows = []
    for impl in args.impls.split(","):
        ms = time_it({"fused": fused, "ours": ours, "nccl": nccl}[impl])
        row = {"case": "fsdp_gather_qkv", "impl": impl, "world": world, "tokens": args.tokens, "width": C,
               "ms": round(ms, 4), "tflops": round(flops / (ms / 1e3) / 1e12, 1),
               "roofline_ms": round(target_ms, 4), "frac_of_roofline": round(target_ms / ms, 3),
               "max_abs_err_vs_nccl": err}
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    if rank == 0 and args.out:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        Path(args.out).write_text("".join(json.dumps(r) + "\n" for r in rows))
    dc.synchronize()
    dist.destroy_process_group()
    mn.destroy_process_group()


if __name__ == "__main__":
    main()
