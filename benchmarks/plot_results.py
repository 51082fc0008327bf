#!/usr/bin/env python
"""Plot benchmark CSVs as standalone SVG line charts (no plotting library needed).

    python benchmarks/plot_results.py results/collectives_w8.csv --x bytes --y busbw_GBs \\
        --series impl,algorithm --filter op=all_reduce --filter dtype=bfloat16 --out docs/img/ar_w8.svg

Log-scaled x axis (message sizes), linear y, one line per distinct value of
the ``--series`` columns (reference: benchmarks/plot_results.py:72-131 draws
the same charts with matplotlib, which this image does not have).
"""

from __future__ import annotations

import argparse
import csv
import math
from pathlib import Path

COLORS = ["#1f77b4", "#d62728", "#2ca02c", "#ff7f0e", "#9467bd", "#8c564b", "#e377c2", "#17becf", "#7f7f7f"]


def human_bytes(v: float) -> str:
    for unit, div in (("GiB", 1 << 30), ("MiB", 1 << 20), ("KiB", 1 << 10)):
        if v >= div:
            return f"{v / div:g}{unit}"
    return f"{v:g}B"


def render(series: dict[str, list[tuple[float, float]]], xlabel: str, ylabel: str, title: str) -> str:
    W, H, L, R, T, B = 760, 440, 70, 200, 40, 60
    xs = [x for pts in series.values() for x, _ in pts if x > 0]
    ys = [y for pts in series.values() for _, y in pts]
    x0, x1 = math.log2(min(xs)), math.log2(max(xs))
    y1 = max(ys) * 1.05 if ys else 1.0
    sx = lambda x: L + (math.log2(x) - x0) / max(1e-9, x1 - x0) * (W - L - R)  # noqa: E731
    sy = lambda y: H - B - y / y1 * (H - T - B)  # noqa: E731
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" font-family="sans-serif" font-size="11">',
           f'<rect width="{W}" height="{H}" fill="white"/>',
           f'<text x="{W / 2 - R / 2}" y="22" text-anchor="middle" font-size="14">{title}</text>',
           f'<line x1="{L}" y1="{H - B}" x2="{W - R}" y2="{H - B}" stroke="black"/>',
           f'<line x1="{L}" y1="{T}" x2="{L}" y2="{H - B}" stroke="black"/>']
    for k in range(int(x0), int(x1) + 1, 2):
        x = sx(2.0 ** k)
        out.append(f'<line x1="{x:.1f}" y1="{H - B}" x2="{x:.1f}" y2="{H - B + 5}" stroke="black"/>')
        out.append(f'<text x="{x:.1f}" y="{H - B + 18}" text-anchor="middle">{human_bytes(2.0 ** k)}</text>')
    for i in range(6):
        yv = y1 * i / 5
        y = sy(yv)
        out.append(f'<line x1="{L - 5}" y1="{y:.1f}" x2="{W - R}" y2="{y:.1f}" stroke="#ddd"/>')
        out.append(f'<text x="{L - 8}" y="{y + 4:.1f}" text-anchor="end">{yv:.0f}</text>')
    out.append(f'<text x="{(L + W - R) / 2}" y="{H - 15}" text-anchor="middle">{xlabel}</text>')
    out.append(f'<text x="18" y="{(T + H - B) / 2}" text-anchor="middle" transform="rotate(-90 18 {(T + H - B) / 2})">'
               f'{ylabel}</text>')
    for n, (name, pts) in enumerate(sorted(series.items())):
        c = COLORS[n % len(COLORS)]
        pts = sorted(pts)
        path = " ".join(f"{'M' if i == 0 else 'L'}{sx(x):.1f},{sy(y):.1f}" for i, (x, y) in enumerate(pts))
        out.append(f'<path d="{path}" fill="none" stroke="{c}" stroke-width="2"/>')
        for x, y in pts:
            out.append(f'<circle cx="{sx(x):.1f}" cy="{sy(y):.1f}" r="2.5" fill="{c}"/>')
        ly = T + 16 * n
        out.append(f'<line x1="{W - R + 12}" y1="{ly}" x2="{W - R + 32}" y2="{ly}" stroke="{c}" stroke-width="2"/>')
        out.append(f'<text x="{W - R + 38}" y="{ly + 4}">{name}</text>')
    out.append("</svg>")
    return "\n".join(out)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("csv")
    ap.add_argument("--x", default="bytes")
    ap.add_argument("--y", default="busbw_GBs")
    ap.add_argument("--series", default="impl,algorithm")
    ap.add_argument("--filter", action="append", default=[], help="column=value (repeatable)")
    ap.add_argument("--title", default="")
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    keys = args.series.split(",")
    filters = [f.split("=", 1) for f in args.filter]
    series: dict[str, list[tuple[float, float]]] = {}
    for row in csv.DictReader(open(args.csv)):
        if any(row.get(k) != v for k, v in filters):
            continue
        name = "/".join(row[k] for k in keys)
        series.setdefault(name, []).append((float(row[args.x]), float(row[args.y])))
    if not series:
        raise SystemExit("no rows matched")
    Path(args.out).parent.mkdir(parents=True, exist_ok=True)
    Path(args.out).write_text(render(series, args.x, args.y, args.title or Path(args.csv).stem))
    print(f"wrote {args.out} ({len(series)} series)")


if __name__ == "__main__":
    main()
