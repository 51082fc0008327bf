"""A broken job must fail loudly and quickly, with a diagnosis.

Faults are made on the host only (a rank that exits hard, a rank that skips a
collective); nothing here touches a GPU.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import time

import pytest
import torch

from mini_nccl_b200 import collectives as C
from mini_nccl_b200.errors import CollectiveTimeoutError, PeerClosedError
from mini_nccl_b200.launcher import run


def diagnose(*args: str) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, "-m", "mini_nccl_b200.diagnose", *args],
                          capture_output=True, text=True)


def _dies(pg) -> None:
    if pg.rank == 1:
        os._exit(9)
    for _ in range(50):
        C.all_reduce(pg, torch.ones(50_000))


def test_dead_rank_fails_fast() -> None:
    t0 = time.perf_counter()
    with pytest.raises(RuntimeError) as info:
        run(_dies, 3, timeout=60.0, op_timeout=20.0)
    assert "rank 1 exited with code" in str(info.value), str(info.value)
    assert time.perf_counter() - t0 < 30.0


def _peer_closed(pg) -> str:
    if pg.rank == 1:
        os._exit(3)
    try:
        C.all_reduce(pg, torch.ones(1 << 20), algorithm="ring")
    except PeerClosedError as exc:
        return f"peer closed: {exc}"
    return "no error"


def test_survivor_sees_peer_closed() -> None:
    with pytest.raises(RuntimeError) as info:
        run(_peer_closed, 2, timeout=60.0, op_timeout=20.0)
    assert "rank 1 exited with code 3" in str(info.value)


def _skips(pg) -> None:
    t = torch.ones(1000)
    C.all_reduce(pg, t)
    if pg.rank != 1:
        C.all_reduce(pg, t)  # rank 1 never joins this one
    C.barrier(pg)


def test_desync_times_out_with_diagnosis(tmp_path) -> None:
    trace = tmp_path / "trace"
    t0 = time.perf_counter()
    with pytest.raises(RuntimeError) as info:
        run(_skips, 3, timeout=90.0, op_timeout=3.0, trace_dir=trace)
    msg = str(info.value)
    assert "CollectiveTimeoutError" in msg, msg
    assert "collectives in identical order" in msg, msg
    assert time.perf_counter() - t0 < 45.0
    dumps = sorted(trace.glob("rank*.json"))
    assert len(dumps) == 3
    second = {}
    for path in dumps:
        state = json.loads(path.read_text())
        order = sorted((e for e in state["events"] if e["channel"] == -1), key=lambda e: e["seq"])
        second[state["rank"]] = order[1]["op"] if len(order) > 1 else None
    assert second[1] == "barrier" and second[0] == "all_reduce", second
    proc = diagnose(str(trace), "--trace", str(tmp_path / "merged.json"))
    assert "DESYNC at collective #1" in proc.stdout, proc.stdout
    assert "rank 1: barrier" in proc.stdout, proc.stdout
    assert proc.returncode == 1
    assert (tmp_path / "merged.json").exists()


def _bounded(pg) -> None:
    pg.recorder.enabled = True
    pg.recorder.resize(8)
    for _ in range(40):
        C.all_reduce(pg, torch.ones(64))
    assert len(pg.recorder.events()) == 8
    assert pg.recorder.dropped > 0
    assert pg.recorder.next_seq(-1) >= 40


def test_recorder_ring_buffer_bounds_memory() -> None:
    run(_bounded, 2, op_timeout=30.0)


def _late_skip(pg) -> None:
    pg.recorder.resize(6)
    t = torch.ones(128)
    for _ in range(20):
        C.all_reduce(pg, t)
    if pg.rank != 1:
        C.all_reduce(pg, t)
    C.barrier(pg)


def test_desync_found_even_when_log_truncated(tmp_path) -> None:
    trace = tmp_path / "trace"
    with pytest.raises(RuntimeError):
        run(_late_skip, 3, timeout=90.0, op_timeout=3.0, trace_dir=trace)
    proc = diagnose(str(trace))
    assert "dropped" in proc.stdout, proc.stdout
    assert "DESYNC at collective #20" in proc.stdout, proc.stdout
    assert "rank 1: barrier" in proc.stdout, proc.stdout


def _healthy(pg) -> None:
    for _ in range(3):
        C.all_reduce(pg, torch.ones(4096))
    C.barrier(pg)


def test_healthy_run_traces_clean(tmp_path) -> None:
    trace = tmp_path / "trace"
    run(_healthy, 2, trace_dir=trace)
    proc = diagnose(str(trace))
    assert proc.returncode == 0, proc.stdout
    assert "all ranks agree" in proc.stdout
    state = json.loads((trace / "rank0.json").read_text())
    ops = [e["op"] for e in state["events"]]
    assert ops.count("all_reduce") == 3 and "barrier" in ops
    assert all(e["dur_us"] is not None for e in state["events"])


def _timeout_error_type(pg) -> str:
    pg.set_op_timeout(1.0)
    if pg.rank == 0:
        try:
            pg.recv(torch.empty(4), src=1)  # rank 1 never sends
        except CollectiveTimeoutError as exc:
            assert isinstance(exc, TimeoutError)
            return "timeout"
        return "none"
    time.sleep(2.5)
    return "idle"


def test_op_timeout_is_adjustable_and_typed() -> None:
    assert run(_timeout_error_type, 2, op_timeout=300.0)[0] == "timeout"


def test_device_log_records_reach_diagnose(tmp_path) -> None:
    """Kernel-level records (as the device ring writes them) are compared per rank."""
    from mini_nccl_b200.recorder import Recorder

    for rank, status in ((0, 0), (1, 1)):
        rec = Recorder(rank, 2, enabled=True)
        rec.attach_device_log(lambda s=status: [
            {"seq": 0, "op": "all_reduce", "nbytes": 64, "end_ns": 10, "status": 0},
            {"seq": 1, "op": "all_reduce", "nbytes": 64, "end_ns": 20, "status": s},
        ])
        rec.dump(tmp_path)
    proc = diagnose(str(tmp_path))
    assert "device progress" in proc.stdout
    assert "DEVICE ERROR on rank 1" in proc.stdout, proc.stdout
    assert proc.returncode == 1
