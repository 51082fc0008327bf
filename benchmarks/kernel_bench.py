#!/usr/bin/env python
"""Time one sm_100a kernel in isolation (CUDA events, warm-up, L2 flush).

    python benchmarks/kernel_bench.py gemm --m 16384 --n 2304 --k 768
    python benchmarks/kernel_bench.py gemm --m 16384 --n 3072 --k 768 --epi gelu
    python benchmarks/kernel_bench.py attn_fwd --b 16 --h 12 --t 1024 --d 64
    python benchmarks/kernel_bench.py attn_bwd --b 16 --h 12 --t 1024 --d 64
    python benchmarks/kernel_bench.py layernorm --m 16384 --n 768
    python benchmarks/kernel_bench.py layernorm_bwd --m 16384 --n 768
    python benchmarks/kernel_bench.py xent --m 16384 --n 50304
    python benchmarks/kernel_bench.py adamw --numel 124000000

Prints one JSON line: time per launch and the achieved fraction of the
measured peaks in ``MEASURED_PEAKS.json`` (bf16 TFLOP/s for tensor-core
kernels, HBM GB/s for the rest), falling back to 1.59 PFLOP/s and 6.65 TB/s.
``--iters 1 --warmup 1`` is the setting for an ncu capture of one launch.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from mini_nccl_b200.ops import kernels as K  # noqa: E402


def peaks() -> tuple[float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


def timed(fn, iters: int, warmup: int, flush: torch.Tensor) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.zero_()  # > L2: every timed launch starts cold
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("kernel", choices=["gemm", "attn_fwd", "attn_bwd", "layernorm", "layernorm_bwd", "xent", "adamw"])
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=2304)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--layout", choices=["tn", "dgrad", "wgrad"], default="tn")
    ap.add_argument("--epi", choices=["none", "bias", "gelu", "gelu_grad", "resid"], default="none")
    ap.add_argument("--splits", type=int, default=0, help="GEMM split-K factor (0: the library's choice)")
    ap.add_argument("--b", type=int, default=16)
    ap.add_argument("--h", type=int, default=12)
    ap.add_argument("--t", type=int, default=1024)
    ap.add_argument("--d", type=int, default=64)
    ap.add_argument("--numel", type=int, default=124_000_000)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    tflops_peak, hbm_peak, src = peaks()
    bf = torch.bfloat16
    r = lambda *s: torch.randn(*s, device=dev).to(bf)  # noqa: E731
    flops = bytes_ = 0.0
    if args.kernel == "gemm":
        M, N, Kd = args.m, args.n, args.k
        if args.layout == "tn":
            a, b = r(M, Kd), r(N, Kd)
            kw = {}
        elif args.layout == "dgrad":
            a, b = r(M, Kd), r(Kd, N)
            kw = {"b_mn": True}
        else:
            a, b = r(Kd, M), r(Kd, N)
            kw = {"a_mn": True, "b_mn": True}
        out = torch.empty(M, N, dtype=bf, device=dev)
        if args.epi == "bias":
            kw["bias"] = r(N)
        elif args.epi == "gelu":
            kw["bias"] = r(N)
            kw["gelu_out_aux"] = torch.empty(M, N, dtype=bf, device=dev)
        elif args.epi == "gelu_grad":
            kw["gelu_grad_aux"] = r(M, N)
        elif args.epi == "resid":
            kw["resid"] = r(M, N)
        if args.splits > 0:
            kw["splits"] = args.splits
        fn = lambda: K.gemm(a, b, out, **kw)  # noqa: E731
        flops = 2.0 * M * N * Kd
    elif args.kernel in ("attn_fwd", "attn_bwd"):
        B, H, T, D = args.b, args.h, args.t, args.d
        qkv = r(B, T, 3 * H * D).requires_grad_(args.kernel == "attn_bwd")
        if args.kernel == "attn_fwd":
            fn = lambda: K.FlashAttention.apply(qkv, H)  # noqa: E731
            flops = 4.0 * B * H * T * T * D / 2
        else:
            y = K.FlashAttention.apply(qkv, H)
            go = torch.randn_like(y)
            fn = lambda: torch.autograd.grad(y, qkv, go, retain_graph=True)  # noqa: E731
            flops = 2.5 * 4.0 * B * H * T * T * D / 2
    elif args.kernel == "layernorm":
        x, w, bb = r(args.m, args.n), r(args.n), r(args.n)
        fn = lambda: K.LayerNorm.apply(x, w, bb, 1e-5)  # noqa: E731
        bytes_ = 2.0 * 2 * args.m * args.n
    elif args.kernel == "layernorm_bwd":
        # the backward kernel alone (dx, dgamma, dbeta), outputs preallocated
        x, w, bb, gy = r(args.m, args.n), r(args.n), r(args.n), r(args.m, args.n)
        y, dx = torch.empty_like(x), torch.empty_like(x)
        dw, db = torch.empty_like(w), torch.empty_like(w)
        mean = torch.empty(args.m, dtype=torch.float32, device=dev)
        rstd = torch.empty(args.m, dtype=torch.float32, device=dev)
        K.ext().layernorm_fwd(x, w, bb, y, mean, rstd, 1e-5)
        acc = K.fold_accumulator(dev, 2 * args.n)
        fn = lambda: K.ext().layernorm_bwd(gy, x, w, mean, rstd, dx, dw, db, acc, False)  # noqa: E731
        bytes_ = 3.0 * 2 * args.m * args.n
    elif args.kernel == "xent":
        z = r(args.m, args.n)
        t = torch.randint(0, args.n, (args.m,), device=dev)
        loss = torch.empty(args.m, dtype=torch.float32, device=dev)
        fn = lambda: K.ext().xent_fwd_bwd(z, t, loss, 1.0 / args.m, -100)  # noqa: E731
        bytes_ = 2.0 * 2 * args.m * args.n
    else:
        p = torch.nn.Parameter(r(args.numel))
        p.grad = r(args.numel)
        opt = K.FusedAdamW([p], lr=1e-4)
        fn = opt.step
        bytes_ = 28.0 * args.numel
    ms = timed(fn, args.iters, args.warmup, flush)
    out = {"kernel": args.kernel, "ms": round(ms, 4), "args": vars(args)}
    if flops:
        tf = flops / (ms / 1e3) / 1e12
        out.update(tflops=round(tf, 1), frac_of_peak=round(tf / tflops_peak, 3), peak=f"{tflops_peak} TFLOP/s ({src})")
    if bytes_:
        gbs = bytes_ / (ms / 1e3) / 1e9
        out.update(gbs=round(gbs, 1), frac_of_peak=round(gbs / hbm_peak, 3), peak=f"{hbm_peak} GB/s ({src})")
    print(json.dumps(out))
    if not math.isfinite(ms):
        raise SystemExit(1)


if __name__ == "__main__":
    main()
