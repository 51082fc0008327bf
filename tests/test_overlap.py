"""Mechanism checks for overlap and straggler diagnosis.

What is asserted is deterministic: the reduction is *dispatched* before
backward returns when overlap is on, and not when it is off.  Whether the
communication thread then wins CPU time before backward ends is up to the OS
and is only reported (the reference's lesson, tests/test_overlap.py:1-25).
"""

from __future__ import annotations

import json
import subprocess
import sys
import time

import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200 import collectives as C
from mini_nccl_b200.ddp import DistributedDataParallel
from mini_nccl_b200.launcher import run


def deep() -> nn.Module:
    torch.manual_seed(5)
    layers: list[nn.Module] = []
    for _ in range(8):
        layers += [nn.Linear(256, 256), nn.Tanh()]
    return nn.Sequential(*layers, nn.Linear(256, 1))


def _measure(pg, overlap: bool) -> dict:
    pg.recorder.enabled = True
    ddp = DistributedDataParallel(deep(), pg, bucket_cap_mb=0.05, overlap=overlap)
    x, y = torch.randn(64, 256), torch.randn(64, 1)
    for _ in range(2):
        ddp.zero_grad()
        F.mse_loss(ddp(x), y).backward()
        ddp.sync()
    ddp.zero_grad()
    loss = F.mse_loss(ddp(x), y)
    t0 = time.perf_counter_ns()
    loss.backward()
    t1 = time.perf_counter_ns()
    submitted = ddp.reduce_submitted_ns
    ddp.sync()
    buckets = [e for e in pg.recorder.events() if e.op.startswith("ddp_bucket") and e.start_ns >= t0]
    first = min((e.start_ns for e in buckets), default=None)
    return {
        "rank": pg.rank,
        "n_buckets": len(ddp._buckets),
        "n_events": len(buckets),
        "dispatch_rel_us": None if submitted is None else (submitted - t1) / 1e3,
        "first_rel_us": None if first is None else (first - t1) / 1e3,
        "backward_us": (t1 - t0) / 1e3,
    }


def test_overlap_dispatches_the_reduction_during_backward() -> None:
    for rep in run(_measure, 2, True):
        assert rep["n_buckets"] > 1 and rep["n_events"] > 0, rep
        assert rep["dispatch_rel_us"] is not None and rep["dispatch_rel_us"] < 0, rep
        print(f"rank {rep['rank']}: dispatched {rep['dispatch_rel_us']:.0f}us, first reduction "
              f"{rep['first_rel_us']:.0f}us relative to a {rep['backward_us']:.0f}us backward")


def test_without_overlap_nothing_is_dispatched_during_backward() -> None:
    for rep in run(_measure, 2, False):
        assert rep["dispatch_rel_us"] is None, rep
        assert rep["first_rel_us"] is not None and rep["first_rel_us"] > 0, rep


def _straggle(pg, slow: int) -> None:
    for _ in range(12):
        if pg.rank == slow:
            time.sleep(0.02)
        C.all_reduce(pg, torch.ones(4096))
    C.barrier(pg)


def test_diagnose_names_a_straggler(tmp_path) -> None:
    trace = tmp_path / "trace"
    run(_straggle, 4, 2, trace_dir=trace, timeout=180.0)
    proc = subprocess.run([sys.executable, "-m", "mini_nccl_b200.diagnose", str(trace)],
                          capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout
    assert "all ranks agree" in proc.stdout
    assert "STRAGGLER: rank 2" in proc.stdout, proc.stdout
    med = {}
    for path in sorted(trace.glob("rank*.json")):
        st = json.loads(path.read_text())
        d = sorted(e["dur_us"] for e in st["events"] if e["op"] == "all_reduce" and e["dur_us"] is not None)
        med[st["rank"]] = d[len(d) // 2]
    assert med[2] < max(med.values()), med
