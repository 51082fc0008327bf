"""mini_nccl_b200: a collectives-and-parallelism library for NVIDIA B200.

Same public API as mini-nccl (mini_nccl/__init__.py:49-181): process groups,
the ``ring``/``tree``/``halving``/``naive`` all-reduce family with a narrow
wire option, reduce-scatter, all-gather, broadcast, all-to-all, barrier, DDP,
FSDP, tensor and pipeline parallelism, ``ParallelMesh`` sub-groups, the flight
recorder and its ``diagnose`` CLI, and the spawn launcher.

Underneath, CUDA tensors never touch a socket: every group maps its peers'
symmetric buffers once (CUDA IPC) and hand-written sm_100a kernels move and
reduce data over NVLink 5 / NVSwitch, fused with the compute around them.
CPU tensors use a native C++ TCP mesh.

Inside a worker::

    import mini_nccl_b200 as mn

    pg = mn.init_process_group()          # RANK / WORLD_SIZE from the env
    mn.all_reduce(tensor)                  # CUDA tensor -> peer-memory kernel
    mn.destroy_process_group()

or spawn locally::

    mn.run(worker_fn, world_size=8, devices="cuda")
"""

from __future__ import annotations

import os

import torch

from . import collectives as _c
from .collectives import ALGORITHMS, DEVICE_ALGORITHMS
from .errors import (
    CollectiveTimeoutError,
    DeviceCommError,
    MiniNcclError,
    PeerClosedError,
    RendezvousError,
)
from .launcher import run
from .mesh import ParallelMesh, SubGroup
from .parallel.ddp import DistributedDataParallel, average_gradients
from .parallel.fsdp import FullyShardedDataParallel
from .parallel.pipeline import PipelineParallel
from .process_group import DEFAULT_N_CHANNELS, ProcessGroup
from .recorder import Recorder

__all__ = [
    "ALGORITHMS",
    "DEFAULT_N_CHANNELS",
    "DEVICE_ALGORITHMS",
    "CollectiveTimeoutError",
    "DeviceCommError",
    "DistributedDataParallel",
    "FullyShardedDataParallel",
    "MiniNcclError",
    "ParallelMesh",
    "PeerClosedError",
    "PipelineParallel",
    "ProcessGroup",
    "Recorder",
    "RendezvousError",
    "SubGroup",
    "all_gather",
    "all_reduce",
    "all_to_all",
    "average_gradients",
    "barrier",
    "broadcast",
    "destroy_process_group",
    "get_group",
    "init_process_group",
    "reduce_scatter",
    "run",
]

__version__ = "0.1.0"

_group: ProcessGroup | None = None


def _hosts_from_env() -> list[tuple[str, int]] | None:
    """Parse ``MINI_NCCL_HOSTS`` = ``host:port,host:port,...`` (multi-node contract)."""
    raw = os.environ.get("MINI_NCCL_HOSTS")
    if not raw:
        return None
    out: list[tuple[str, int]] = []
    for item in raw.split(","):
        item = item.strip()
        if not item:
            continue
        host, sep, port = item.rpartition(":")
        if not sep or not host:
            raise ValueError(f"MINI_NCCL_HOSTS entry {item!r} must be host:port")
        out.append((host, int(port)))
    return out


def _hosts_via_store(rank: int, world_size: int) -> list[tuple[str, int]]:
    """Exchange listening ports through the launcher's TCP store (torchrun).

    Under torchrun the agent already runs a key-value store at
    ``MASTER_ADDR:MASTER_PORT``; each rank picks a free local port, publishes
    it there and reads everyone else's.  That avoids colliding with the store's
    own port, which a ``MASTER_PORT + rank`` scheme would.
    """
    from datetime import timedelta

    import torch.distributed as dist

    from .launcher import _free_ports

    master = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ["MASTER_PORT"])
    store = dist.TCPStore(master, port, world_size, is_master=False, timeout=timedelta(seconds=120))
    host = os.environ.get("MINI_NCCL_LISTEN_HOST", "127.0.0.1")
    mine = _free_ports(1)[0]
    run_id = os.environ.get("TORCHELASTIC_RUN_ID", "job")
    store.set(f"mnb/{run_id}/addr/{rank}", f"{host}:{mine}")
    addrs = []
    for r in range(world_size):
        key = f"mnb/{run_id}/addr/{r}"
        store.wait([key])
        h, _, p = store.get(key).decode().rpartition(":")
        addrs.append((h, int(p)))
    return addrs


def init_process_group(
    rank: int | None = None,
    world_size: int | None = None,
    addrs: list[tuple[str, int]] | None = None,
    base_port: int | None = None,
    n_channels: int | None = None,
    device: torch.device | str | int | None = None,
    nccl_p2p: bool = False,
    **kwargs,
) -> ProcessGroup:
    """Create the default process group.

    Missing arguments come from the environment: ``RANK``/``WORLD_SIZE``,
    ``MASTER_PORT`` (base port), ``MINI_NCCL_CHANNELS`` and ``MINI_NCCL_HOSTS``.
    Under torchrun (``TORCHELASTIC_RUN_ID`` set) addresses are exchanged through
    the launcher's store instead.  With CUDA available and ``LOCAL_RANK`` set,
    the group is bound to ``cuda:LOCAL_RANK``.  ``nccl_p2p=True`` also brings up
    a torch.distributed NCCL group used for CUDA tensors at pipeline
    boundaries.
    """
    global _group
    if _group is not None:
        raise RuntimeError("default process group already initialized")
    if rank is None:
        rank = int(os.environ["RANK"])
    if world_size is None:
        world_size = int(os.environ["WORLD_SIZE"])
    if n_channels is None:
        n_channels = int(os.environ.get("MINI_NCCL_CHANNELS", DEFAULT_N_CHANNELS))
    if addrs is None:
        addrs = _hosts_from_env()
    if addrs is None and world_size > 1 and os.environ.get("TORCHELASTIC_RUN_ID"):
        addrs = _hosts_via_store(rank, world_size)
    if base_port is None:
        base_port = int(os.environ.get("MASTER_PORT", "29500"))
    if device is None and torch.cuda.is_available() and "LOCAL_RANK" in os.environ:
        device = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    if device is not None:
        device = torch.device(device)
        if device.type == "cuda":
            torch.cuda.set_device(device)
    _group = ProcessGroup(
        rank, world_size, addrs=addrs, base_port=base_port, n_channels=n_channels,
        device=device, **kwargs,
    )
    if nccl_p2p and world_size > 1:
        import torch.distributed as dist

        if not dist.is_initialized():
            dist.init_process_group("nccl", rank=rank, world_size=world_size, device_id=device)
        _group.attach_nccl(dist.group.WORLD)
    return _group


def get_group() -> ProcessGroup:
    if _group is None:
        raise RuntimeError("call init_process_group() first")
    return _group


def destroy_process_group() -> None:
    global _group
    if _group is not None:
        _group.close()
        _group = None


def all_reduce(
    tensor: torch.Tensor,
    op: str = "sum",
    algorithm: str = "auto",
    wire_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    return _c.all_reduce(get_group(), tensor, op=op, algorithm=algorithm, wire_dtype=wire_dtype)


def broadcast(tensor: torch.Tensor, src: int = 0) -> torch.Tensor:
    return _c.broadcast(get_group(), tensor, src=src)


def all_gather(tensor: torch.Tensor) -> list[torch.Tensor]:
    return _c.all_gather(get_group(), tensor)


def reduce_scatter(tensor: torch.Tensor, op: str = "sum") -> torch.Tensor:
    return _c.reduce_scatter(get_group(), tensor, op=op)


def all_to_all(tensor: torch.Tensor) -> torch.Tensor:
    return _c.all_to_all(get_group(), tensor)


def barrier() -> None:
    _c.barrier(get_group())
