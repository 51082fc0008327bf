"""The interface all collectives and strategies are written against.

Mirrors the nine-member protocol of the reference
(mini_nccl/communicator.py:27-70): ``rank``, ``world_size``, ``n_channels``,
``recorder``, ``send``, ``recv``, ``send_recv``, ``send_recv_sliced`` and
``run_per_channel``.  :class:`~mini_nccl_b200.process_group.ProcessGroup` and
:class:`~mini_nccl_b200.mesh.SubGroup` both satisfy it, which is what lets DP,
TP and PP compose on sub-groups unchanged.

The GPU data path needs one more thing that the host protocol does not carry:
the set of *global* ranks a communicator spans, so a sub-group can build a
device context over exactly its members' peer memory.  That is exposed as the
optional ``global_ranks`` attribute (see :func:`global_ranks_of`) rather than
as a tenth protocol member, so third-party communicators written against the
nine-member protocol still type-check.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Protocol, runtime_checkable

import torch

from .recorder import Recorder


@runtime_checkable
class Communicator(Protocol):
    """What a collective needs from whatever it communicates over."""

    #: This participant's index within the group, ``0 .. world_size-1``.
    rank: int
    #: Number of participants.
    world_size: int
    #: Independent connections (host) or CTA groups (device) per peer.
    n_channels: int
    #: Flight recorder the collectives log themselves to.
    recorder: Recorder

    def send(self, tensor: torch.Tensor, dst: int, channel: int = 0) -> None: ...

    def recv(self, tensor: torch.Tensor, src: int, channel: int = 0) -> None: ...

    def send_recv(
        self,
        send_tensor: torch.Tensor,
        dst: int,
        recv_tensor: torch.Tensor,
        src: int,
        channel: int = 0,
    ) -> None:
        """Send to ``dst`` and receive from ``src`` at the same time."""
        ...

    def send_recv_sliced(
        self,
        send_tensor: torch.Tensor,
        dst: int,
        recv_tensor: torch.Tensor,
        src: int,
        n_slices: int,
        on_slice: Callable[[int, int], None],
        channel: int = 0,
    ) -> None:
        """Like ``send_recv`` but report each received slice as it lands."""
        ...

    def run_per_channel(self, fns: list[Callable[[], None]]) -> None:
        """Run one callable per channel concurrently; re-raise the first error."""
        ...


def global_ranks_of(comm: Communicator) -> list[int]:
    """Global (root process group) ranks of ``comm``'s members, in local order."""
    ranks = getattr(comm, "global_ranks", None)
    if ranks is None:
        return list(range(comm.world_size))
    return list(ranks)
