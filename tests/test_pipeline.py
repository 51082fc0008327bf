"""Pipeline schedules on CPU ranks: gradients equal one process, depth, tracing.

This library's own scenarios: a stack of pre-norm residual MLP blocks split
evenly over the stages, a classification head with cross-entropy on the last
stage, and per-case seeds; every stage's parameter gradients and the last
stage's loss must equal what one process computes on the whole model and the
whole batch.
"""

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

HIDDEN, CLASSES, BLOCKS_PER_STAGE = 12, 5, 2


class ResidualMLP(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(HIDDEN)
        self.up = nn.Linear(HIDDEN, 2 * HIDDEN)
        self.down = nn.Linear(2 * HIDDEN, HIDDEN)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.down(F.gelu(self.up(self.norm(x))))


class Head(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(HIDDEN)
        self.out = nn.Linear(HIDDEN, CLASSES)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.out(self.norm(x))


def build_stages(n_stages: int, seed: int) -> list[nn.Sequential]:
    """The whole model, already cut into stages (the last one ends in the head)."""
    torch.manual_seed(seed)
    stages = [nn.Sequential(*(ResidualMLP() for _ in range(BLOCKS_PER_STAGE))) for _ in range(n_stages)]
    stages[-1].append(Head())
    return stages


def _matches_one_process(pg, schedule: str, n_micro: int, batch: int, seed: int) -> float | None:
    stages = build_stages(pg.world_size, seed)
    whole = nn.Sequential(*stages)
    mine = stages[pg.rank]
    pp = PipelineParallel(mine, pg, (batch // n_micro, HIDDEN), loss_fn=F.cross_entropy, schedule=schedule)
    data = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(batch, HIDDEN, generator=data)
    y = torch.randint(0, CLASSES, (batch,), generator=data)
    last = pg.rank == pg.world_size - 1
    whole.zero_grad(set_to_none=True)
    loss = pp.step(x if pg.rank == 0 else None, y if last else None, n_micro)
    piped = [p.grad.clone() for p in mine.parameters()]
    whole.zero_grad(set_to_none=True)
    want = F.cross_entropy(whole(x), y)
    want.backward()
    for got, p in zip(piped, mine.parameters(), strict=True):
        torch.testing.assert_close(got, p.grad, rtol=1e-5, atol=1e-6)
    if last:
        assert abs(float(loss) - want.item()) <= 1e-5 * max(1.0, abs(want.item()))
        return float(loss)
    return None


@pytest.mark.parametrize("world,schedule,n_micro,batch,seed", [
    (2, "1f1b", 6, 18, 3),   # more microbatches than stages
    (4, "1f1b", 4, 16, 5),   # exactly one microbatch per stage
    (4, "1f1b", 3, 12, 7),   # fewer microbatches than stages: warm-up is cut short
    (3, "gpipe", 5, 15, 11),
    (2, "1f1b", 1, 6, 13),   # one microbatch: no steady state at all
])
def test_gradients_match_one_process(world, schedule, n_micro, batch, seed) -> None:
    losses = run(_matches_one_process, world, schedule, n_micro, batch, seed)
    assert losses[-1] is not None and all(v is None for v in losses[:-1])


def _peak_depth(pg, schedule: str, n_micro: int) -> int:
    stage = build_stages(pg.world_size, 17)[pg.rank]
    pp = PipelineParallel(stage, pg, (3, HIDDEN), loss_fn=F.cross_entropy, schedule=schedule)
    data = torch.Generator().manual_seed(18)
    n = 3 * n_micro
    x = torch.randn(n, HIDDEN, generator=data)
    y = torch.randint(0, CLASSES, (n,), generator=data)
    pp.step(x if pg.rank == 0 else None, y if pg.rank == pg.world_size - 1 else None, n_micro)
    return pp.in_flight_peak


def test_1f1b_bounds_in_flight_microbatches() -> None:
    W, M = 4, 10
    peaks = run(_peak_depth, W, "1f1b", M)
    assert peaks == [W - s for s in range(W)], peaks  # stage s holds at most W - s, the last one 1


def test_gpipe_holds_every_microbatch() -> None:
    assert run(_peak_depth, 3, "gpipe", 7) == [7, 7, 7]


def _two_traced_steps(pg) -> None:
    stage = build_stages(pg.world_size, 21)[pg.rank]
    pp = PipelineParallel(stage, pg, (2, HIDDEN), loss_fn=F.cross_entropy)
    for k in range(2):
        data = torch.Generator().manual_seed(100 + k)
        x = torch.randn(6, HIDDEN, generator=data)
        y = torch.randint(0, CLASSES, (6,), generator=data)
        pp.step(x if pg.rank == 0 else None, y if pg.rank == pg.world_size - 1 else None, 3)


def test_stage_dependent_schedules_do_not_read_as_a_desync(tmp_path) -> None:
    trace = tmp_path / "trace"
    run(_two_traced_steps, 3, trace_dir=trace, timeout=180.0)
    proc = subprocess.run([sys.executable, "-m", "mini_nccl_b200.diagnose", str(trace)],
                          capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout
    assert "all ranks agree" in proc.stdout and "'pipeline':" in proc.stdout, proc.stdout
    for rank in range(3):
        events = json.loads((trace / f"rank{rank}.json").read_text())["events"]
        pipe = [e for e in events if e["op"].startswith("pp_")]
        assert {e["op"] for e in pipe} == {"pp_forward", "pp_backward"}
        assert all(e["channel"] == PIPELINE_CHANNEL for e in pipe)
        assert sum(e["op"] == "pp_forward" for e in pipe) == 6  # 2 steps x 3 microbatches


def _bad_arguments(pg) -> None:
    stage = nn.Linear(HIDDEN, HIDDEN)
    with pytest.raises(ValueError, match="unknown schedule"):
        PipelineParallel(stage, pg, (2, HIDDEN), loss_fn=F.mse_loss, schedule="interleaved")
    with pytest.raises(ValueError, match="needs loss_fn"):
        PipelineParallel(stage, pg, (2, HIDDEN))
    pp = PipelineParallel(stage, pg, (3, HIDDEN), loss_fn=F.mse_loss)
    with pytest.raises(ValueError, match="needs inputs"):
        pp.step(None, torch.zeros(6, HIDDEN), 2)
    with pytest.raises(ValueError, match="needs targets"):
        pp.step(torch.zeros(6, HIDDEN), None, 2)
    with pytest.raises(ValueError, match="not divisible"):
        pp.step(torch.zeros(7, HIDDEN), torch.zeros(7, HIDDEN), 2)
    with pytest.raises(ValueError, match="at least 1"):
        pp.step(torch.zeros(6, HIDDEN), torch.zeros(6, HIDDEN), 0)


def test_argument_errors_are_raised_before_any_traffic() -> None:
    run(_bad_arguments, 1)
