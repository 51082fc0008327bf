"""Host transport: Python face of the native TCP full mesh.

The sockets, rendezvous, full-duplex progress engine and timeouts live in
C++ (``csrc/host/tcp_mesh.cpp``); this module only validates tensors, turns
native exceptions into :mod:`mini_nccl_b200.errors` types, and keeps the
reference's module surface (``byte_view``, ``Mesh``, ``DEFAULT_OP_TIMEOUT``;
mini_nccl/transport.py:49-216).

CPU tensors only: a CUDA tensor never crosses this transport on the hot path
(device collectives use peer memory, pipeline p2p uses NCCL).
"""

from __future__ import annotations

import torch

from ._build import host_ext
from .errors import PeerClosedError, RendezvousError

DEFAULT_OP_TIMEOUT = 300.0


def byte_view(tensor: torch.Tensor) -> memoryview:
    """The tensor's storage as a flat writable byte view, without copying."""
    if not tensor.is_contiguous():
        raise ValueError("transport requires contiguous tensors")
    if tensor.device.type != "cpu":
        raise ValueError("transport requires CPU tensors (device tensors use peer memory)")
    return tensor.detach().reshape(-1).view(torch.uint8).numpy().data


def tensor_span(tensor: torch.Tensor) -> tuple[int, int]:
    """(address, nbytes) of a contiguous CPU tensor, validated like ``byte_view``."""
    if not tensor.is_contiguous():
        raise ValueError("transport requires contiguous tensors")
    if tensor.device.type != "cpu":
        raise ValueError("transport requires CPU tensors (device tensors use peer memory)")
    return tensor.data_ptr(), tensor.numel() * tensor.element_size()


class Mesh:
    """All ``n_channels`` connections from this rank to every peer."""

    def __init__(
        self,
        rank: int,
        world_size: int,
        addrs: list[tuple[str, int]],
        n_channels: int = 1,
        timeout: float = 60.0,
        op_timeout: float | None = DEFAULT_OP_TIMEOUT,
    ) -> None:
        ext = host_ext()
        self.rank = rank
        self.world_size = world_size
        self.n_channels = n_channels
        try:
            self.native = ext.TcpMesh(
                rank,
                world_size,
                [(h, int(p)) for h, p in addrs] if world_size > 1 else [],
                n_channels,
                float(timeout),
                -1.0 if op_timeout is None else float(op_timeout),
            )
        except ext.TransportRendezvous as exc:
            raise RendezvousError(str(exc)) from None

    def set_op_timeout(self, op_timeout: float | None) -> None:
        self.native.set_op_timeout(-1.0 if op_timeout is None else float(op_timeout))

    def close(self) -> None:
        self.native.close()


def native_errors():
    """(timeout_exc, peer_closed_exc) classes raised by the native transport."""
    ext = host_ext()
    return ext.TransportTimeout, ext.TransportPeerClosed


__all__ = ["DEFAULT_OP_TIMEOUT", "Mesh", "PeerClosedError", "byte_view", "tensor_span"]
