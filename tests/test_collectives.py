"""Every host collective against results each rank recomputes from seeds.

Rank ``r``'s input is a pure function of ``(r, numel, dtype)``, so any rank
can rebuild every input and the exact expected output without a golden file
or a cross-process oracle (the reference's strategy,
tests/test_collectives.py:28-47).  One worker runs the whole battery inside a
single process group; the test is parametrised over the world size.
"""

from __future__ import annotations

import pytest
import torch

from mini_nccl_b200 import collectives as C
from mini_nccl_b200.launcher import run

NUMELS = (1, 3, 1024, 262_147)  # one element, fewer than ranks, odd, many socket buffers


def seeded(rank: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
    g = torch.Generator().manual_seed(7000 + rank)
    if dtype.is_floating_point:
        return torch.randn(numel, generator=g, dtype=dtype)
    return torch.randint(-40, 40, (numel,), generator=g, dtype=dtype)


def expected(world: int, numel: int, dtype: torch.dtype, op: str) -> torch.Tensor:
    parts = [seeded(r, numel, dtype) for r in range(world)]
    out = parts[0].clone()
    for p in parts[1:]:
        if op == "sum":
            out = out + p
        elif op == "prod":
            out = out * p
        elif op == "max":
            out = torch.maximum(out, p)
        else:
            out = torch.minimum(out, p)
    return out


def _battery(pg) -> None:
    W, r = pg.world_size, pg.rank
    for algorithm in C.ALGORITHMS:
        for op in ("sum", "max", "min", "prod"):
            for dtype in (torch.float32, torch.int64):
                for numel in NUMELS:
                    if op == "prod" and numel > 1024:
                        continue
                    t = seeded(r, numel, dtype)
                    C.all_reduce(pg, t, op=op, algorithm=algorithm)
                    torch.testing.assert_close(
                        t, expected(W, numel, dtype, op), rtol=1e-4, atol=1e-4,
                        msg=lambda m, a=algorithm, o=op, d=dtype, n=numel: f"{a}/{o}/{d}/{n}: {m}",
                    )
    for numel in (16, 1_000_000):  # auto: tree below the threshold, ring above
        t = seeded(r, numel, torch.float32)
        C.all_reduce(pg, t)
        torch.testing.assert_close(t, expected(W, numel, torch.float32, "sum"), rtol=1e-4, atol=1e-4)
    for src in range(W):
        t = seeded(r, 4097, torch.float32)
        C.broadcast(pg, t, src=src)
        torch.testing.assert_close(t, seeded(src, 4097, torch.float32))
    shaped = seeded(r, 6 * 13, torch.float32).view(6, 13)
    got = C.all_gather(pg, shaped)
    assert len(got) == W
    for i, g in enumerate(got):
        torch.testing.assert_close(g, seeded(i, 6 * 13, torch.float32).view(6, 13))
    n = 10 * W
    t = seeded(r, n, torch.float32)
    before = t.clone()
    mine = C.reduce_scatter(pg, t)
    torch.testing.assert_close(mine, expected(W, n, torch.float32, "sum").view(W, -1)[r], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(t, before)  # input untouched
    n = 7 * W
    out = C.all_to_all(pg, seeded(r, n, torch.float32))
    for src in range(W):
        torch.testing.assert_close(out.view(W, -1)[src], seeded(src, n, torch.float32).view(W, -1)[r])
    C.barrier(pg)


@pytest.mark.parametrize("world_size", [2, 3, 4])
def test_collective_battery(world_size: int) -> None:
    run(_battery, world_size)


def _multichannel(pg) -> None:
    assert pg.n_channels == 4
    numel = 1_000_003  # divisible by neither the channels nor the ranks
    assert C._n_channels_for(pg, numel * 4) == 4, "must exercise every channel"
    for algorithm in ("ring", "halving"):
        t = seeded(pg.rank, numel, torch.float32)
        C.all_reduce(pg, t, algorithm=algorithm)
        torch.testing.assert_close(t, expected(pg.world_size, numel, torch.float32, "sum"), rtol=1e-4, atol=1e-3)


def test_multichannel_large_allreduce(monkeypatch) -> None:
    monkeypatch.setenv("MINI_NCCL_CHANNEL_MIN_BYTES", str(64 * 1024))
    run(_multichannel, 4, n_channels=4)


def _sliced(pg) -> None:
    assert C.MAX_SLICES == 8
    numel = 300_001
    for algorithm in ("ring", "halving"):
        t = seeded(pg.rank, numel, torch.float32)
        C.all_reduce(pg, t, algorithm=algorithm)
        torch.testing.assert_close(t, expected(pg.world_size, numel, torch.float32, "sum"), rtol=1e-4, atol=1e-3)


def test_sliced_reduction_overlap(monkeypatch) -> None:
    """Reduce-while-receiving (slices) gives the same answer."""
    monkeypatch.setenv("MINI_NCCL_MAX_SLICES", "8")
    run(_sliced, 2)


def _single_channel(pg) -> None:
    assert pg.n_channels == 1
    t = seeded(pg.rank, 1_000_001, torch.float32)
    C.all_reduce(pg, t, algorithm="ring")
    torch.testing.assert_close(t, expected(2, 1_000_001, torch.float32, "sum"), rtol=1e-4, atol=1e-3)


def test_single_channel_still_correct() -> None:
    run(_single_channel, 2, n_channels=1)


def _raises_on_rank1(pg) -> None:
    if pg.rank == 1:
        raise ValueError("deliberate failure on rank 1")
    C.barrier(pg)


def test_worker_errors_propagate() -> None:
    with pytest.raises(RuntimeError, match="deliberate failure on rank 1"):
        run(_raises_on_rank1, 2, timeout=60.0, op_timeout=10.0)


def test_world_size_one_is_identity() -> None:
    from mini_nccl_b200.process_group import ProcessGroup

    with ProcessGroup(0, 1) as pg:
        t = torch.arange(8, dtype=torch.float32)
        C.all_reduce(pg, t)
        torch.testing.assert_close(t, torch.arange(8, dtype=torch.float32))
        assert C.reduce_scatter(pg, t).data_ptr() != t.data_ptr()
        C.barrier(pg)


def test_argument_validation() -> None:
    from mini_nccl_b200.process_group import ProcessGroup

    with ProcessGroup(0, 1) as pg:
        with pytest.raises(ValueError, match="unknown op"):
            C.all_reduce(pg, torch.ones(2), op="mean")
    with pytest.raises(ValueError, match="contiguous"):
        C._flat(torch.zeros(4, 4).t())
    assert [p.numel() for p in C._split(torch.arange(10), 3)] == [4, 3, 3]
