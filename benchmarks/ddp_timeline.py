#!/usr/bin/env python
"""Where a DDP step's gradient all-reduces sit relative to backward, per bucket.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29730 benchmarks/ddp_timeline.py --out results/ddp_timeline_w2.json

The GPT of the DDP configuration (12 layers, d_model 768, T 1024, micro-batch
16 per GPU, 25 MB buckets) runs a few warm-up steps; then one step is traced
on the GPU's own clock (``%globaltimer``):

* a stamp kernel on the compute stream marks the step start, the start of
  backward, each bucket's readiness (its last gradient written; stamped where
  DDP launches its all-reduce) and the end of backward;
* the device event ring gives each bucket all-reduce's kernel start and end.

For every rank it reports, in microseconds from the start of backward: when
each bucket became ready, when its all-reduce ran, and how long after the
end of backward the last one finished (the exposed communication).  Rank 0
prints one JSON document (every rank's table) and writes it to ``--out``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import collectives as C  # noqa: E402
from mini_nccl_b200.models.gpt import GPT  # noqa: E402
from mini_nccl_b200.ops.kernels import FusedAdamW, ext  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--micro-batch", type=int, default=16)
    ap.add_argument("--bucket-mb", type=float, default=25.0)
    ap.add_argument("--out")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    pg = mn.init_process_group(rank, world, device=dev, op_timeout=120.0)
    torch.manual_seed(0)
    model = GPT(50304, 1024, 12, 12, 768).to(dev, torch.bfloat16)
    ddp = mn.DistributedDataParallel(model, pg, bucket_cap_mb=args.bucket_mb, overlap=True, algorithm="auto")
    opt = FusedAdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    g = torch.Generator().manual_seed(1000 + rank)
    x = torch.randint(0, 50304, (args.micro_batch, 1024), generator=g).to(dev)
    y = torch.randint(0, 50304, (args.micro_batch, 1024), generator=g).to(dev)
    stamps = torch.zeros(256, dtype=torch.int64, device=dev)
    STEP, BWD, BWD_END, SYNCED = 250, 251, 252, 253

    def step(trace: bool) -> None:
        if trace:
            ext().stamp(stamps, STEP)
        ddp.zero_grad()
        _, loss = ddp(x, y)
        if trace:
            ext().stamp(stamps, BWD)
        loss.backward()
        if trace:
            ext().stamp(stamps, BWD_END)
        ddp.sync()
        if trace:
            ext().stamp(stamps, SYNCED)
        opt.step()

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    C.barrier(pg)
    ddp.timeline, ddp.timeline_seqs = stamps, []
    step(True)
    torch.cuda.synchronize()
    ddp.timeline = None
    t = stamps.cpu().tolist()
    dc = pg.device_comm()
    ring = {e["seq"]: e for e in dc.device_events()}
    t0 = t[BWD]
    us = lambda ns: round((ns - t0) / 1e3, 1)  # noqa: E731
    buckets = []
    for b, seq in zip(ddp._buckets, ddp.timeline_seqs, strict=True):
        ev = ring.get(seq, {})
        buckets.append({"bucket": b.index, "mb": round(b.nbytes / 2**20, 2), "ready_us": us(t[b.index]),
                        "ar_start_us": us(ev["start_ns"]) if ev else None,
                        "ar_end_us": us(ev["end_ns"]) if ev.get("end_ns") else None,
                        "algorithm": "nvls" if dc.impl.is_nvls(b.buffer) else "two_shot"})
    last_end = max((bk["ar_end_us"] or 0.0) for bk in buckets) if buckets else 0.0
    mine = {"rank": rank, "forward_us": round((t[BWD] - t[STEP]) / 1e3, 1), "backward_us": us(t[BWD_END]),
            "sync_done_us": us(t[SYNCED]), "exposed_after_backward_us": round(max(0.0, last_end - us(t[BWD_END])), 1),
            "buckets": buckets}
    blob = torch.frombuffer(bytearray(json.dumps(mine).encode()), dtype=torch.uint8)
    size = torch.tensor([blob.numel()])
    sizes = C.all_gather(pg, size)
    n = int(max(s.item() for s in sizes))
    padded = torch.zeros(n, dtype=torch.uint8)
    padded[: blob.numel()] = blob
    parts = C.all_gather(pg, padded)
    if rank == 0:
        ranks = [json.loads(bytes(p[: int(s.item())].tolist()).decode()) for p, s in zip(parts, sizes)]
        doc = {"world": world, "nvls": dc.nvls, "bucket_mb": args.bucket_mb, "ranks": ranks,
               "max_exposed_after_backward_us": max(r["exposed_after_backward_us"] for r in ranks)}
        print(json.dumps(doc), flush=True)
        if args.out:
            Path(args.out).parent.mkdir(parents=True, exist_ok=True)
            Path(args.out).write_text(json.dumps(doc, indent=1))
    dc.synchronize()
    mn.destroy_process_group()


if __name__ == "__main__":
    main()
