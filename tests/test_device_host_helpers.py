"""Host-side helpers of the device communicator that run without a GPU."""

from __future__ import annotations

from mini_nccl_b200.device import all_gather_blobs, schedule_steps
from mini_nccl_b200.launcher import run


def _blobs(pg) -> list[bytes]:
    # different lengths per rank, and an empty one (what a "no error" or a
    # "supported" answer looks like)
    mine = b"" if pg.rank == 1 else f"rank-{pg.rank}-".encode() * (pg.rank + 1)
    return all_gather_blobs(pg, mine)


def test_all_gather_blobs_handles_ragged_and_empty_blobs() -> None:
    for got in run(_blobs, 3):
        assert got == [b"rank-0-", b"", b"rank-2-rank-2-rank-2-"]


def _all_empty(pg) -> list[bytes]:
    return all_gather_blobs(pg, b"")


def test_all_gather_blobs_all_empty() -> None:
    assert run(_all_empty, 2) == [[b"", b""], [b"", b""]]


def test_ring_schedule_visits_each_foreign_block_once_per_phase() -> None:
    W, n = 4, 1003
    for r in range(W):
        steps = schedule_steps("ring", W, r, n)
        assert len(steps) == 2 * (W - 1)
        reduce, gather = steps[: W - 1], steps[W - 1:]
        assert {s[4] for s in reduce} == {1} and {s[4] for s in gather} == {2}
        assert len({s[1] for s in reduce}) == W - 1 and len({s[1] for s in gather}) == W - 1
        assert sum(s[3] for s in reduce) < n and sum(s[3] for s in gather) < n


def test_auto_all_reduce_follows_the_measured_cut_overs() -> None:
    from mini_nccl_b200.device import NVLS_MIN_BYTES, ONE_SHOT_MAX_BYTES, auto_all_reduce_algorithm

    KiB, MiB = 1 << 10, 1 << 20
    # two ranks: the switch moves more bytes per GPU than the peer kernels
    assert auto_all_reduce_algorithm(64 * KiB, 2, True, False) == "one_shot"
    assert auto_all_reduce_algorithm(ONE_SHOT_MAX_BYTES, 2, True, False) == "one_shot"
    assert auto_all_reduce_algorithm(ONE_SHOT_MAX_BYTES + 16, 2, True, False) == "two_shot"
    assert auto_all_reduce_algorithm(256 * MiB, 2, True, False) == "two_shot"
    # eight ranks: one-shot below NVLS_MIN_BYTES, the switch from there on
    assert auto_all_reduce_algorithm(1 * MiB, 8, True, False) == "one_shot"
    assert auto_all_reduce_algorithm(NVLS_MIN_BYTES, 8, True, False) == "nvls"
    assert auto_all_reduce_algorithm(1 << 30, 8, True, False) == "nvls"
    # no usable switch path: peer kernels at every size
    assert auto_all_reduce_algorithm(1 << 30, 8, False, False) == "two_shot"
    # a tensor bound to the multicast object is reduced in place at any size
    assert auto_all_reduce_algorithm(4 * KiB, 2, True, True) == "nvls"
