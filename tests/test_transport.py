"""Native TCP transport: point-to-point, full duplex, rendezvous cleanup."""

from __future__ import annotations

import socket

import pytest
import torch

from mini_nccl_b200.errors import RendezvousError
from mini_nccl_b200.launcher import _free_ports, run
from mini_nccl_b200.transport import Mesh, byte_view


def _pingpong(pg) -> None:
    data = torch.arange(20_000, dtype=torch.float64)
    if pg.rank == 0:
        pg.send(data, dst=1)
        back = torch.empty_like(data)
        pg.recv(back, src=1)
        torch.testing.assert_close(back, data * 3)
    else:
        got = torch.empty_like(data)
        pg.recv(got, src=0)
        pg.send(got * 3, dst=0)


def test_send_recv_pingpong() -> None:
    run(_pingpong, 2)


def _rotate(pg) -> None:
    W, r = pg.world_size, pg.rank
    mine = torch.full((1 << 20,), float(r))  # 4 MiB: larger than the socket buffers
    inbox = torch.empty_like(mine)
    pg.send_recv(mine, (r + 1) % W, inbox, (r - 1) % W)
    assert torch.all(inbox == float((r - 1) % W))


def test_full_duplex_ring_rotation_does_not_deadlock() -> None:
    run(_rotate, 3)


def _slices(pg) -> None:
    peer = 1 - pg.rank
    out = torch.arange(100_003, dtype=torch.float32) + pg.rank
    inbox = torch.empty_like(out)
    seen: list[tuple[int, int]] = []
    pg.send_recv_sliced(out, peer, inbox, peer, 7, lambda a, b: seen.append((a, b)))
    assert seen[0][0] == 0 and seen[-1][1] == inbox.numel()
    assert all(a == b for (_, a), (b, _) in zip(seen, seen[1:]))  # contiguous, ordered
    assert len(seen) == 7
    torch.testing.assert_close(inbox, torch.arange(100_003, dtype=torch.float32) + peer)


def test_sliced_exchange_reports_every_slice_in_order() -> None:
    run(_slices, 2)


def test_failed_rendezvous_frees_the_port() -> None:
    mine, absent = _free_ports(2)
    addrs = [("127.0.0.1", mine), ("127.0.0.1", absent)]
    for _ in range(2):  # the second attempt only binds if the first released it
        with pytest.raises(RendezvousError, match=r"no contact with ranks \[1\]"):
            Mesh(0, 2, addrs, n_channels=1, timeout=1.0)
    probe = socket.create_server(("127.0.0.1", mine))
    probe.close()


def test_byte_view_rejects_non_contiguous() -> None:
    with pytest.raises(ValueError, match="contiguous"):
        byte_view(torch.zeros(3, 5).t())


def test_byte_view_is_zero_copy() -> None:
    t = torch.zeros(4, dtype=torch.float32)
    v = byte_view(t)
    assert len(v) == 16
    v[0] = 1
    assert t[0] != 0
