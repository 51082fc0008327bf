"""Pipeline schedules: whole-model parity, the 1F1B depth bound, tracing, validation."""

from __future__ import annotations

import json
import subprocess
import sys

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200.launcher import run
from mini_nccl_b200.pipeline import PIPELINE_CHANNEL, PipelineParallel

WIDTH, PER_STAGE = 8, 2


def layers_for(n_stages: int) -> list[nn.Module]:
    torch.manual_seed(4)
    return [nn.Sequential(nn.Linear(WIDTH, WIDTH), nn.Tanh()) for _ in range(n_stages * PER_STAGE)]


def my_stage(layers, rank: int) -> nn.Module:
    return nn.Sequential(*layers[rank * PER_STAGE : (rank + 1) * PER_STAGE])


def _parity(pg, schedule: str, n_micro: int, batch: int) -> None:
    layers = layers_for(pg.world_size)
    whole = nn.Sequential(*layers)
    stage = my_stage(layers, pg.rank)
    pp = PipelineParallel(stage, pg, (batch // n_micro, WIDTH), loss_fn=F.mse_loss, schedule=schedule)
    g = torch.Generator().manual_seed(19)
    x = torch.randn(batch, WIDTH, generator=g)
    y = torch.randn(batch, WIDTH, generator=g)
    for p in whole.parameters():
        p.grad = None
    loss = pp.step(x if pg.rank == 0 else None, y if pg.rank == pg.world_size - 1 else None, n_micro)
    got = [p.grad.clone() for p in stage.parameters()]
    for p in whole.parameters():
        p.grad = None
    ref_loss = F.mse_loss(whole(x), y)
    ref_loss.backward()
    for i, p in enumerate(stage.parameters()):
        torch.testing.assert_close(got[i], p.grad, rtol=1e-4, atol=1e-6)
    if pg.rank == pg.world_size - 1:
        torch.testing.assert_close(torch.tensor(loss), ref_loss.detach(), rtol=1e-5, atol=1e-6)


def test_1f1b_matches_single_process_two_stages() -> None:
    run(_parity, 2, "1f1b", 4, 16)


def test_1f1b_matches_single_process_four_stages() -> None:
    run(_parity, 4, "1f1b", 8, 16)


def test_gpipe_matches_single_process() -> None:
    run(_parity, 4, "gpipe", 8, 16)


def test_1f1b_fewer_microbatches_than_stages() -> None:
    run(_parity, 4, "1f1b", 2, 16)


def test_single_microbatch_degenerates_cleanly() -> None:
    run(_parity, 3, "1f1b", 1, 12)


def _depth(pg, schedule: str, n_micro: int) -> dict:
    stage = my_stage(layers_for(pg.world_size), pg.rank)
    pp = PipelineParallel(stage, pg, (2, WIDTH), loss_fn=F.mse_loss, schedule=schedule)
    g = torch.Generator().manual_seed(23)
    b = 2 * n_micro
    pp.step(torch.randn(b, WIDTH, generator=g) if pg.rank == 0 else None,
            torch.randn(b, WIDTH, generator=g) if pg.rank == pg.world_size - 1 else None, n_micro)
    return {"rank": pg.rank, "peak": pp.in_flight_peak}


def test_1f1b_bounds_in_flight_microbatches() -> None:
    W, M = 4, 12
    peaks = {r["rank"]: r["peak"] for r in run(_depth, W, "1f1b", M)}
    for rank, peak in peaks.items():
        assert peak <= W - rank and peak < M, peaks
    assert peaks[0] > peaks[W - 1] and peaks[W - 1] == 1, peaks


def test_gpipe_holds_every_microbatch() -> None:
    for rep in run(_depth, 4, "gpipe", 12):
        assert rep["peak"] == 12, rep


def _traced(pg) -> None:
    stage = nn.Sequential(nn.Linear(WIDTH, WIDTH), nn.Tanh())
    pp = PipelineParallel(stage, pg, (2, WIDTH), loss_fn=F.mse_loss)
    for _ in range(2):
        pp.step(torch.randn(8, WIDTH) if pg.rank == 0 else None,
                torch.randn(8, WIDTH) if pg.rank == pg.world_size - 1 else None, 4)


def test_pipeline_traced_without_faking_a_desync(tmp_path) -> None:
    trace = tmp_path / "trace"
    run(_traced, 4, trace_dir=trace, timeout=180.0)
    proc = subprocess.run([sys.executable, "-m", "mini_nccl_b200.diagnose", str(trace)],
                          capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout
    assert "all ranks agree" in proc.stdout and "'pipeline':" in proc.stdout, proc.stdout
    st = json.loads((trace / "rank0.json").read_text())
    ops = [e["op"] for e in st["events"]]
    assert "pp_forward" in ops and "pp_backward" in ops
    assert all(e["channel"] == PIPELINE_CHANNEL for e in st["events"] if e["op"].startswith("pp_"))


def _rejects(pg) -> None:
    stage = nn.Linear(WIDTH, WIDTH)
    with pytest.raises(ValueError, match="unknown schedule"):
        PipelineParallel(stage, pg, (2, WIDTH), loss_fn=F.mse_loss, schedule="zigzag")
    with pytest.raises(ValueError, match="needs loss_fn"):
        PipelineParallel(stage, pg, (2, WIDTH), loss_fn=None)
    pp = PipelineParallel(stage, pg, (2, WIDTH), loss_fn=F.mse_loss)
    with pytest.raises(ValueError, match="needs inputs"):
        pp.step(None, torch.zeros(4, WIDTH), 2)
    with pytest.raises(ValueError, match="needs targets"):
        pp.step(torch.zeros(4, WIDTH), None, 2)
    with pytest.raises(ValueError, match="not divisible"):
        pp.step(torch.zeros(5, WIDTH), torch.zeros(5, WIDTH), 2)
    with pytest.raises(ValueError, match="at least 1"):
        pp.step(torch.zeros(4, WIDTH), torch.zeros(4, WIDTH), 0)


def test_argument_errors_are_clear() -> None:
    run(_rejects, 1)
