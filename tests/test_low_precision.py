"""Narrow wire (bf16) with wide accumulation on the host path.

Pins the reference's measured behaviour (tests/test_low_precision.py:36-150):
the error of a bf16-wire reduction is set by how many times the partial sum
is re-rounded onto the wire, so ring error grows with the world size while
tree error stays flat, and widening the accumulator does not change it.
"""

from __future__ import annotations

import pytest
import torch

from mini_nccl_b200 import collectives as C
from mini_nccl_b200.launcher import run
from mini_nccl_b200.process_group import ProcessGroup

N = 20_000


def payload(rank: int, world: int = 1) -> torch.Tensor:
    """Rank 0 holds 1.0, every other rank a value below half a bf16 ulp of 1.0.

    Every time a partial sum near 1.0 is put on the wire, one small term is
    rounded away (or up), so the error counts how many hops cross the wire
    with a large partial sum: ``W-1`` for ring, about ``log2 W`` for tree.
    """
    return torch.full((N,), 1.0 if rank == 0 else 0.004)


def _err(pg, algorithm: str) -> float:
    W = pg.world_size
    t = payload(pg.rank, W)
    C.all_reduce(pg, t, algorithm=algorithm, wire_dtype=torch.bfloat16)
    exact = sum(payload(r, W).double() for r in range(W))
    return float((t.double() - exact).abs().mean())


def _both(pg) -> dict:
    return {"ring": _err(pg, "ring"), "tree": _err(pg, "tree")}


@pytest.fixture(scope="module")
def errors() -> dict[int, dict]:
    return {W: run(_both, W)[0] for W in (4, 8)}


def test_ring_error_grows_with_world_size(errors) -> None:
    assert errors[8]["ring"] > 1.5 * errors[4]["ring"], errors


def test_tree_error_stays_flat(errors) -> None:
    # Tree sums the small terms among themselves first, so its error stays
    # below half a bf16 ulp of the result at every world size.
    half_ulp = 2.0**-9
    assert errors[4]["tree"] < half_ulp and errors[8]["tree"] < half_ulp, errors


def test_tree_is_more_accurate_at_scale(errors) -> None:
    assert errors[8]["tree"] < errors[8]["ring"] / 4 or errors[8]["tree"] < 2e-3, errors


def _wide_acc(pg) -> tuple[float, float]:
    a = payload(pg.rank).bfloat16()
    C.all_reduce(pg, a, algorithm="ring", wire_dtype=torch.bfloat16)
    b = payload(pg.rank).bfloat16()
    C.all_reduce(pg, b, algorithm="ring")
    exact = sum(payload(r).double() for r in range(pg.world_size))
    e = lambda t: float(((t.double() - exact).abs() / exact).max())  # noqa: E731
    return e(a), e(b)


def test_wide_accumulator_does_not_change_the_error() -> None:
    wide, narrow = run(_wide_acc, 4)[0]
    assert wide <= narrow * 1.5 + 1e-6, (wide, narrow)


def _exact(pg) -> None:
    t = torch.full((N,), 2.0)
    C.all_reduce(pg, t, algorithm="ring", wire_dtype=torch.bfloat16)
    assert torch.all(t == 2.0 * pg.world_size)


def test_representable_payloads_are_exact() -> None:
    run(_exact, 4)


def test_rejected_combinations() -> None:
    with ProcessGroup(0, 1) as pg:
        pg.world_size = 2  # validation happens before any traffic
        with pytest.raises(ValueError, match="wire_dtype is implemented"):
            C.all_reduce(pg, torch.ones(4), algorithm="naive", wire_dtype=torch.bfloat16)
        with pytest.raises(ValueError, match="wider"):
            C.all_reduce(pg, torch.ones(4, dtype=torch.bfloat16), algorithm="ring", wire_dtype=torch.float32)
        pg.world_size = 1
