"""Pull-form all-reduce schedules of the device communicator, checked on CPU.

The device executor runs ring / tree / halving / naive as a list of
per-rank steps (read a peer's range, fold or copy it into ours) separated by
barriers.  Simulating those tables on CPU tensors proves every schedule
computes the exact sum on every rank before any GPU runs it.
"""

from __future__ import annotations

import pytest
import torch


def test_schedule_tables_are_consistent():
    """Pull schedules (CPU-only check): every read targets data the peer has finished."""
    from mini_nccl_b200.device import schedule_steps

    for W in (2, 3, 4, 8):
        for alg in ("ring", "tree", "naive") + (("halving",) if W & (W - 1) == 0 else ()):
            tables = [schedule_steps(alg, W, r, 1000) for r in range(W)]
            assert len({len(t) for t in tables}) == 1, (alg, W)
            for t in tables:
                for peer, src, dst, count, mode in t:
                    assert 0 <= peer < W and count >= 0 and mode in (0, 1, 2)
                    assert 0 <= src and src + count <= 1000 and 0 <= dst and dst + count <= 1000


def _simulate(alg: str, W: int, n: int = 37):
    """Run the pull schedules on CPU tensors to prove they compute the sum."""
    from mini_nccl_b200.device import schedule_steps

    bufs = [torch.arange(n, dtype=torch.float64) * (r + 1) + r for r in range(W)]
    want = sum(b.clone() for b in bufs)
    tables = [schedule_steps(alg, W, r, n) for r in range(W)]
    for s in range(len(tables[0])):
        snap = [b.clone() for b in bufs]  # every rank reads peers' state from before the step
        for r in range(W):
            peer, src, dst, count, mode = tables[r][s]
            if mode == 1:
                bufs[r][dst : dst + count] += snap[peer][src : src + count]
            elif mode == 2:
                bufs[r][dst : dst + count] = snap[peer][src : src + count]
    for r in range(W):
        assert torch.equal(bufs[r], want), (alg, W, r)


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_pull_schedules_compute_the_sum(W):
    for alg in ("ring", "tree", "naive") + (("halving",) if W & (W - 1) == 0 else ()):
        _simulate(alg, W)
