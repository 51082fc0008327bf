#!/usr/bin/env python
"""Fit the alpha-beta cost model ``t = steps*alpha + bytes_moved*beta`` per algorithm.

    python benchmarks/fit_cost_model.py results/allreduce.csv --world 4

Reads a sweep written by bench_allreduce.py (or bench_collectives.py for the
device path) and fits, per algorithm, the per-step latency alpha and the
per-byte cost beta by least squares on *relative* error, so small messages
weigh as much as large ones (reference: benchmarks/fit_cost_model.py:48-242).
Step counts and payload multipliers follow each algorithm's schedule.
"""

from __future__ import annotations

import argparse
import csv
import math

import numpy as np


def model_terms(algorithm: str, W: int) -> tuple[float, float]:
    """(number of latency steps, bytes moved per rank as a multiple of n)."""
    lg = math.ceil(math.log2(W))
    return {
        "ring": (2 * (W - 1), 2 * (W - 1) / W),
        "tree": (2 * lg, 2 * lg),
        "halving": (2 * lg, 2 * (W - 1) / W),
        "naive": (2 * (W - 1), 2 * (W - 1)),
        "one_shot": (1, W - 1),
        "two_shot": (2, 2 * (W - 1) / W),
    }.get(algorithm, (1, 1))


def fit(rows: list[dict], W: int):
    out = {}
    for algo in sorted({r["algorithm"] for r in rows}):
        pts = [(float(r["bytes"]), float(r["ms"]) / 1e3) for r in rows if r["algorithm"] == algo
               and int(r.get("world", W)) == W]
        if len(pts) < 2:
            continue
        steps, mult = model_terms(algo, W)
        A = np.array([[steps / t, mult * b / t] for b, t in pts])
        y = np.ones(len(pts))
        (alpha, beta), *_ = np.linalg.lstsq(A, y, rcond=None)
        pred = A @ np.array([alpha, beta])
        out[algo] = {"alpha_us": alpha * 1e6, "beta_ns_per_byte": beta * 1e9,
                     "implied_GBs": (1 / beta / 1e9) if beta > 0 else float("inf"),
                     "mean_rel_err": float(np.mean(np.abs(pred - 1)))}
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("csv")
    ap.add_argument("--world", type=int, default=4)
    args = ap.parse_args()
    rows = list(csv.DictReader(open(args.csv)))
    for algo, f in fit(rows, args.world).items():
        print(f"{algo:10s} alpha {f['alpha_us']:9.2f} us/step  beta {f['beta_ns_per_byte']:8.4f} ns/B  "
              f"({f['implied_GBs']:8.2f} GB/s)  mean rel err {f['mean_rel_err']:.1%}")


if __name__ == "__main__":
    main()
