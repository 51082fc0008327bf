"""Sub-groups and mesh composition (2D and 3D parity with one process)."""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200 import collectives as C
from mini_nccl_b200.communicator import Communicator
from mini_nccl_b200.ddp import DistributedDataParallel, average_gradients
from mini_nccl_b200.launcher import run
from mini_nccl_b200.mesh import ParallelMesh, SubGroup
from mini_nccl_b200.pipeline import PipelineParallel
from mini_nccl_b200.tensor_parallel import ParallelMLP

WIDTH = 12


def _layout(pg) -> dict:
    m = ParallelMesh(pg, dp=2, tp=2)
    return {"rank": pg.rank, "dp": m.coordinate("dp"), "tp": m.coordinate("tp"),
            "tp_ranks": m.ranks_along("tp"), "dp_ranks": m.ranks_along("dp")}


def test_mesh_layout_last_dimension_fastest() -> None:
    reps = {r["rank"]: r for r in run(_layout, 4)}
    assert reps[0]["tp_ranks"] == [0, 1] and reps[2]["tp_ranks"] == [2, 3]
    assert reps[0]["dp_ranks"] == [0, 2] and reps[1]["dp_ranks"] == [1, 3]
    for rank, rep in reps.items():
        assert rep["dp"] * 2 + rep["tp"] == rank


def _orthogonal(pg) -> None:
    m = ParallelMesh(pg, dp=2, pp=2, tp=2)
    groups = [set(m.ranks_along(n)) for n in ("dp", "pp", "tp")]
    assert set.intersection(*groups) == {pg.rank}
    for a in range(3):
        for b in range(a + 1, 3):
            assert groups[a] & groups[b] == {pg.rank}


def test_three_dimensional_groups_are_orthogonal() -> None:
    run(_orthogonal, 8)


def _errors(pg) -> None:
    with pytest.raises(ValueError, match="has 6 slots"):
        ParallelMesh(pg, dp=3, tp=2)
    with pytest.raises(ValueError, match="at least 1"):
        ParallelMesh(pg, dp=0, tp=4)
    with pytest.raises(ValueError, match="give at least one"):
        ParallelMesh(pg)
    with pytest.raises(KeyError, match="no dimension"):
        ParallelMesh(pg, dp=4).ranks_along("tp")
    with pytest.raises(ValueError, match="duplicate"):
        SubGroup(pg, [pg.rank, pg.rank])
    other = [r for r in range(pg.world_size) if r != pg.rank][:1]
    with pytest.raises(ValueError, match="not a member"):
        SubGroup(pg, other)


def test_mesh_errors_are_clear() -> None:
    run(_errors, 4)


def _subgroup_collectives(pg) -> None:
    m = ParallelMesh(pg, dp=2, tp=2)
    tp, dp = m.group("tp"), m.group("dp")
    assert isinstance(tp, Communicator)
    t = torch.full((1000,), float(pg.rank))
    C.all_reduce(tp, t)
    members = m.ranks_along("tp")
    assert torch.all(t == float(sum(members)))
    got = C.all_gather(dp, torch.tensor([float(pg.rank)]))
    assert [g.item() for g in got] == [float(r) for r in m.ranks_along("dp")]
    nested = tp.subgroup([tp.rank])
    one = torch.ones(3)
    C.all_reduce(nested, one)
    assert torch.all(one == 1)
    assert nested.global_ranks == [pg.rank]
    C.barrier(dp)


def test_collectives_on_subgroups() -> None:
    run(_subgroup_collectives, 4)


def _size_one(pg) -> None:
    m = ParallelMesh(pg, dp=1, tp=pg.world_size)
    g = m.group("dp")
    assert g.world_size == 1
    t = torch.arange(5.0)
    C.all_reduce(g, t)
    torch.testing.assert_close(t, torch.arange(5.0))


def test_size_one_dimension_is_a_noop() -> None:
    run(_size_one, 2)


def _two_d(pg) -> None:
    """TP inside DP: grads equal the single-process gradients of the whole batch."""
    m = ParallelMesh(pg, dp=2, tp=2)
    tp, dp = m.group("tp"), m.group("dp")
    torch.manual_seed(3)
    ref = nn.Sequential(nn.Linear(WIDTH, 4 * WIDTH), nn.GELU(), nn.Linear(4 * WIDTH, WIDTH))
    par = ParallelMLP(WIDTH, tp)
    par.up.load_full_weight(ref[0].weight.detach(), ref[0].bias.detach())
    par.down.load_full_weight(ref[2].weight.detach(), ref[2].bias.detach())
    ddp = DistributedDataParallel(par, dp)
    g = torch.Generator().manual_seed(8)
    x = torch.randn(8, WIDTH, generator=g)
    y = torch.randn(8, WIDTH, generator=g)
    mine = slice(m.coordinate("dp") * 4, (m.coordinate("dp") + 1) * 4)
    F.mse_loss(ddp(x[mine]), y[mine]).backward()
    ddp.sync()
    F.mse_loss(ref(x), y).backward()
    a, b = par.up.shard_start, par.up.shard_start + par.up.shard_size
    torch.testing.assert_close(par.up.weight.grad, ref[0].weight.grad[a:b], rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(par.down.bias.grad, ref[2].bias.grad, rtol=1e-4, atol=1e-6)


def test_two_dimensional_parity() -> None:
    run(_two_d, 4)


def _three_d(pg) -> dict:
    """dp2 x pp2 x tp2: every rank's slice of every gradient matches one process."""
    m = ParallelMesh(pg, dp=2, pp=2, tp=2)
    tp, pp, dp = m.group("tp"), m.group("pp"), m.group("dp")
    torch.manual_seed(5)
    full = [nn.Sequential(nn.Linear(WIDTH, 4 * WIDTH), nn.GELU(), nn.Linear(4 * WIDTH, WIDTH))
            for _ in range(2)]
    ref = nn.Sequential(*copy.deepcopy(full))
    s = m.coordinate("pp")
    stage = ParallelMLP(WIDTH, tp)
    stage.up.load_full_weight(full[s][0].weight.detach(), full[s][0].bias.detach())
    stage.down.load_full_weight(full[s][2].weight.detach(), full[s][2].bias.detach())
    pipe = PipelineParallel(stage, pp, (2, WIDTH), loss_fn=F.mse_loss)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(8, WIDTH, generator=g)
    y = torch.randn(8, WIDTH, generator=g)
    mine = slice(m.coordinate("dp") * 4, (m.coordinate("dp") + 1) * 4)
    loss = pipe.step(x[mine] if s == 0 else None, y[mine] if s == 1 else None, 2)
    average_gradients(dp, list(stage.parameters()))
    F.mse_loss(ref(x), y).backward()
    a, b = stage.up.shard_start, stage.up.shard_start + stage.up.shard_size
    torch.testing.assert_close(stage.up.weight.grad, ref[s][0].weight.grad[a:b], rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(stage.down.bias.grad, ref[s][2].bias.grad, rtol=1e-4, atol=1e-6)
    return {"rank": pg.rank, "loss": loss, "tp": m.coordinate("tp"), "pp": s, "dp": m.coordinate("dp")}


def test_three_dimensional_parity() -> None:
    reps = run(_three_d, 8)
    last = [r for r in reps if r["pp"] == 1]
    for dpc in (0, 1):
        pair = [r["loss"] for r in last if r["dp"] == dpc]
        assert pair[0] == pair[1], pair  # the tp pair agrees exactly
