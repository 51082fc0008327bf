"""Sub-group communicators and the named parallelism mesh.

API and layout follow the reference (mini_nccl/mesh.py:50-207):
``SubGroup(parent, ranks)`` is a rank-translating *view* over the parent's
connections (nothing reconnects) that implements the whole communicator
protocol and can be nested; ``ParallelMesh(pg, dp=2, pp=2, tp=2)`` factors the
world with the **last dimension fastest**, so tensor-parallel groups are runs
of consecutive ranks (on one HGX board: GPUs that are neighbours on NVSwitch,
which is every GPU).

On the GPU path a sub-group also owns a *device* communicator over just its
members: built lazily on its first CUDA collective, with the handle exchange
carried over this same view, so the tp, pp and dp groups of a 3D mesh each get
their own peer mappings and signal pads.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence

import torch

from .communicator import Communicator, global_ranks_of


class SubGroup:
    """A communicator over a subset of a parent communicator's ranks."""

    def __init__(self, parent: Communicator, global_ranks: Sequence[int], name: str = "") -> None:
        ranks = list(global_ranks)
        repeated = sorted({r for r in ranks if ranks.count(r) > 1})
        if repeated:
            raise ValueError(f"subgroup {ranks} names ranks {repeated} more than once (duplicate members)")
        if parent.rank not in ranks:
            raise ValueError(f"this process (rank {parent.rank}) is not a member of {ranks}: "
                             "only the members construct a SubGroup")
        outside = [r for r in ranks if not 0 <= r < parent.world_size]
        if outside:
            raise ValueError(f"ranks {outside} are outside the parent group of {parent.world_size}")
        self.parent = parent
        self.name = name
        #: Members in *parent* numbering (what ``SubGroup(parent, ranks)`` was given).
        self.parent_ranks = ranks
        parent_globals = global_ranks_of(parent)
        #: Members in *root* numbering, for device contexts.
        self.global_ranks = [parent_globals[r] for r in ranks]
        self.rank = ranks.index(parent.rank)
        self.world_size = len(ranks)
        self.n_channels = parent.n_channels
        self.recorder = parent.recorder
        self.device = getattr(parent, "device", None)
        self._device_comm = None

    def _up(self, local: int) -> int:
        return self.parent_ranks[local]

    # ---- the protocol --------------------------------------------------------------

    def send(self, tensor: torch.Tensor, dst: int, channel: int = 0) -> None:
        self.parent.send(tensor, self._up(dst), channel)

    def recv(self, tensor: torch.Tensor, src: int, channel: int = 0) -> None:
        self.parent.recv(tensor, self._up(src), channel)

    def send_recv(self, send_tensor, dst, recv_tensor, src, channel: int = 0) -> None:
        self.parent.send_recv(send_tensor, self._up(dst), recv_tensor, self._up(src), channel)

    def send_recv_sliced(
        self, send_tensor, dst, recv_tensor, src, n_slices: int,
        on_slice: Callable[[int, int], None], channel: int = 0,
    ) -> None:
        self.parent.send_recv_sliced(
            send_tensor, self._up(dst), recv_tensor, self._up(src), n_slices, on_slice, channel
        )

    def run_per_channel(self, fns: list[Callable[[], None]]) -> None:
        self.parent.run_per_channel(fns)

    # ---- extras ----------------------------------------------------------------------

    @property
    def nccl_group(self):
        return getattr(self.parent, "nccl_group", None)

    def device_comm(self):
        """Device communicator over this sub-group's members (collective on first use)."""
        if self._device_comm is None:
            from .device import DeviceComm

            self._device_comm = DeviceComm(self, self.global_ranks)
        return self._device_comm

    def subgroup(self, ranks: Sequence[int], name: str = "") -> SubGroup:
        """Nest a subgroup; ``ranks`` are in *this* group's numbering."""
        return SubGroup(self, ranks, name)

    def close(self) -> None:
        if self._device_comm is not None:
            self._device_comm.close()
            self._device_comm = None

    def __repr__(self) -> str:
        label = f" {self.name!r}" if self.name else ""
        return f"<SubGroup{label} rank {self.rank}/{self.world_size} global={self.global_ranks}>"


class ParallelMesh:
    """Name the dimensions of the world: ``ParallelMesh(pg, dp=2, tp=2)``.

    Dimensions are listed outermost first; the last varies fastest.
    """

    def __init__(self, pg: Communicator, **dims: int) -> None:
        if not dims:
            raise ValueError("give at least one dimension, e.g. ParallelMesh(pg, tp=2)")
        too_small = {name: size for name, size in dims.items() if size < 1}
        if too_small:
            raise ValueError(f"every mesh dimension must be at least 1, got {too_small}")
        slots = math.prod(dims.values())
        if slots != pg.world_size:
            raise ValueError(f"mesh {dims} has {slots} slots but the group has {pg.world_size} ranks")
        self.pg = pg
        self.dims = dict(dims)
        self.names = list(dims)
        sizes = list(dims.values())
        # row-major: a dimension's stride is the product of the sizes after it
        self.strides: dict[str, int] = {n: math.prod(sizes[i + 1:]) for i, n in enumerate(self.names)}
        self.coords = {n: (pg.rank // self.strides[n]) % self.dims[n] for n in self.names}
        self._groups: dict[str, SubGroup] = {}

    def ranks_along(self, name: str) -> list[int]:
        """Ranks that differ from this one only in dimension ``name``."""
        if name not in self.dims:
            raise KeyError(f"no dimension {name!r}; mesh has {self.names}")
        origin = self.pg.rank - self.coords[name] * self.strides[name]
        return [origin + i * self.strides[name] for i in range(self.dims[name])]

    def group(self, name: str) -> SubGroup:
        """This rank's communicator along ``name`` (a size-1 axis is a no-op group)."""
        if name not in self._groups:
            self._groups[name] = SubGroup(self.pg, self.ranks_along(name), name)
        return self._groups[name]

    def coordinate(self, name: str) -> int:
        return self.coords[name]

    def size(self, name: str) -> int:
        return self.dims[name]

    def describe(self) -> str:
        body = " ".join(f"{n}={self.coords[n]}/{self.dims[n]}" for n in self.names)
        return f"rank {self.pg.rank}: {body}"

    def __repr__(self) -> str:
        return f"<ParallelMesh {self.dims} rank {self.pg.rank}>"
