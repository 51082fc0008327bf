"""What a desynchronised job looks like, and how the flight recorder finds it.

    python examples/desync_demo.py

Rank 2 skips the second all-reduce (the classic "conditional collective"
bug).  The survivors time out instead of hanging, every rank dumps its
flight recorder, and ``diagnose`` names the divergence (reference:
examples/desync_demo.py:33-75).
"""

from __future__ import annotations

import subprocess
import sys
import tempfile
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import mini_nccl_b200 as mn  # noqa: E402
from mini_nccl_b200 import collectives  # noqa: E402


def buggy_worker(pg):
    t = torch.ones(1024)
    collectives.all_reduce(pg, t)
    if pg.rank != 2:  # rank 2 "forgets" this one
        collectives.all_reduce(pg, t)
    collectives.barrier(pg)


def main():
    trace_dir = Path(tempfile.mkdtemp(prefix="mnb-desync-"))
    try:
        mn.run(buggy_worker, 4, op_timeout=5.0, timeout=120.0, trace_dir=trace_dir)
    except RuntimeError as exc:
        first = str(exc).splitlines()
        print("job failed as expected:\n  " + "\n  ".join(line for line in first if "Error" in line)[:2000])
    print(f"\n$ python -m mini_nccl_b200.diagnose {trace_dir}\n", flush=True)
    out = subprocess.run([sys.executable, "-m", "mini_nccl_b200.diagnose", str(trace_dir)],
                         capture_output=True, text=True)
    print(out.stdout)


if __name__ == "__main__":
    main()
