"""Process group: the point-to-point layer every collective is built on.

Same constructor, members and error behaviour as the reference
(mini_nccl/process_group.py:42-196), on a different engine:

* CPU tensors go over the native TCP mesh.  ``send_recv`` is a single native
  call that drives both directions from one poll() loop (no send thread), and
  ``send_recv_sliced`` gets a callback per landed slice from that same loop.
* CUDA tensors handed to ``send``/``recv``/``send_recv`` (pipeline stage
  boundaries) go over NCCL point-to-point when a NCCL group is attached
  (``attach_nccl``), otherwise they are staged through host memory.
* CUDA tensors handed to *collectives* never come here: collectives use the
  device communicator returned by :meth:`device_comm`, which maps every peer's
  symmetric buffers into this process once and then moves data with kernels.

A timeout anywhere becomes :class:`CollectiveTimeoutError` carrying the
flight recorder's context and the likely cause.
"""

from __future__ import annotations

from collections.abc import Callable
from concurrent.futures import ThreadPoolExecutor

import torch

from .errors import CollectiveTimeoutError, PeerClosedError
from .recorder import Recorder, trace_enabled_by_env
from .transport import DEFAULT_OP_TIMEOUT, Mesh, native_errors, tensor_span

DEFAULT_BASE_PORT = 29500

# Two channels measured best on loopback TCP in the reference's ablation
# (mini_nccl/process_group.py:32-35); on the GPU path a "channel" is a group
# of CTAs and the count is chosen per message size instead.
DEFAULT_N_CHANNELS = 2


def default_addrs(world_size: int, base_port: int = DEFAULT_BASE_PORT) -> list[tuple[str, int]]:
    return [("127.0.0.1", base_port + r) for r in range(world_size)]


class ProcessGroup:
    """All ranks of one job, connected pairwise over ``n_channels`` channels."""

    def __init__(
        self,
        rank: int,
        world_size: int,
        addrs: list[tuple[str, int]] | None = None,
        base_port: int = DEFAULT_BASE_PORT,
        timeout: float = 60.0,
        n_channels: int = DEFAULT_N_CHANNELS,
        op_timeout: float | None = DEFAULT_OP_TIMEOUT,
        trace: bool | None = None,
        device: torch.device | str | int | None = None,
    ) -> None:
        if not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} out of range for world_size {world_size}")
        if n_channels < 1:
            raise ValueError("n_channels must be >= 1")
        self.rank = rank
        self.world_size = world_size
        self.n_channels = n_channels
        self.global_ranks = list(range(world_size))
        self.op_timeout = op_timeout
        self.recorder = Recorder(
            rank, world_size, enabled=trace_enabled_by_env() if trace is None else bool(trace)
        )
        if addrs is None:
            addrs = default_addrs(world_size, base_port)
        if world_size > 1 and len(addrs) != world_size:
            raise ValueError("need one (host, port) address per rank")
        self._mesh = Mesh(rank, world_size, addrs, n_channels, timeout, op_timeout)
        self._native = self._mesh.native
        self._timeout_exc, self._closed_exc = native_errors()
        self._channel_pool = (
            ThreadPoolExecutor(max_workers=n_channels, thread_name_prefix=f"mnb-chan-r{rank}")
            if n_channels > 1
            else None
        )
        self.device = None if device is None else torch.device(device)
        self._device_comm = None
        self.nccl_group = None
        self._closed = False

    # ---- point to point -------------------------------------------------------

    def _translate(self, exc: BaseException, what: str, peer: int, channel: int) -> BaseException:
        if isinstance(exc, self._timeout_exc):
            return self._timeout_error(what, peer, channel, str(exc))
        if isinstance(exc, self._closed_exc):
            return PeerClosedError(f"rank {self.rank}: {exc}")
        return exc

    def send(self, tensor: torch.Tensor, dst: int, channel: int = 0) -> None:
        if tensor.is_cuda:
            self._device_send(tensor, dst)
            return
        ptr, n = tensor_span(tensor)
        try:
            self._native.send(dst, channel, ptr, n)
        except (self._timeout_exc, self._closed_exc) as exc:
            raise self._translate(exc, "send", dst, channel) from None

    def recv(self, tensor: torch.Tensor, src: int, channel: int = 0) -> None:
        if tensor.is_cuda:
            self._device_recv(tensor, src)
            return
        ptr, n = tensor_span(tensor)
        try:
            self._native.recv(src, channel, ptr, n)
        except (self._timeout_exc, self._closed_exc) as exc:
            raise self._translate(exc, "recv", src, channel) from None

    def send_recv(
        self,
        send_tensor: torch.Tensor,
        dst: int,
        recv_tensor: torch.Tensor,
        src: int,
        channel: int = 0,
    ) -> None:
        """Full-duplex exchange: both directions progress in one native loop."""
        if send_tensor.is_cuda or recv_tensor.is_cuda:
            self._device_send_recv(send_tensor, dst, recv_tensor, src)
            return
        sp, sn = tensor_span(send_tensor)
        rp, rn = tensor_span(recv_tensor)
        try:
            self._native.exchange(dst, sp, sn, src, rp, rn, channel, 0, None)
        except (self._timeout_exc, self._closed_exc) as exc:
            raise self._translate(exc, "send_recv", src, channel) from None

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
        """As ``send_recv``; ``on_slice(start, end)`` (elements) runs per landed slice."""
        n = recv_tensor.numel()
        if n_slices <= 1 or n < n_slices or recv_tensor.is_cuda:
            self.send_recv(send_tensor, dst, recv_tensor, src, channel)
            on_slice(0, n)
            return
        item = recv_tensor.element_size()
        per = -(-n // n_slices)
        sp, sn = tensor_span(send_tensor)
        rp, rn = tensor_span(recv_tensor)

        def landed(lo: int, hi: int) -> None:
            on_slice(lo // item, hi // item)

        try:
            self._native.exchange(dst, sp, sn, src, rp, rn, channel, per * item, landed)
        except (self._timeout_exc, self._closed_exc) as exc:
            raise self._translate(exc, "send_recv", src, channel) from None

    def run_per_channel(self, fns: list[Callable[[], None]]) -> None:
        """Drive one callable per channel concurrently (native calls drop the GIL)."""
        if len(fns) == 1 or self._channel_pool is None:
            for fn in fns:
                fn()
            return
        futures = [self._channel_pool.submit(fn) for fn in fns]
        first: BaseException | None = None
        for fut in futures:
            try:
                fut.result()
            except BaseException as exc:  # collect all, re-raise the first
                first = first or exc
        if first is not None:
            raise first

    # ---- CUDA tensors at p2p boundaries ----------------------------------------

    def attach_nccl(self, group) -> None:
        """Use a torch.distributed NCCL group (same rank numbering) for device p2p."""
        self.nccl_group = group

    def _device_send(self, tensor: torch.Tensor, dst: int) -> None:
        if self.nccl_group is not None:
            import torch.distributed as dist

            dist.send(tensor.contiguous(), dst=self._nccl_rank(dst), group=self.nccl_group)
            return
        self.send(tensor.detach().contiguous().cpu(), dst)

    def _device_recv(self, tensor: torch.Tensor, src: int) -> None:
        if self.nccl_group is not None:
            import torch.distributed as dist

            dist.recv(tensor, src=self._nccl_rank(src), group=self.nccl_group)
            return
        host = torch.empty(tensor.shape, dtype=tensor.dtype)
        self.recv(host, src)
        tensor.copy_(host)

    def _device_send_recv(self, send_tensor, dst, recv_tensor, src) -> None:
        if self.nccl_group is not None:
            import torch.distributed as dist

            ops = [
                dist.P2POp(dist.isend, send_tensor.contiguous(), self._nccl_rank(dst), self.nccl_group),
                dist.P2POp(dist.irecv, recv_tensor, self._nccl_rank(src), self.nccl_group),
            ]
            for work in dist.batch_isend_irecv(ops):
                work.wait()
            return
        host_out = send_tensor.detach().contiguous().cpu()
        host_in = torch.empty(recv_tensor.shape, dtype=recv_tensor.dtype)
        self.send_recv(host_out, dst, host_in, src)
        recv_tensor.copy_(host_in)

    def _nccl_rank(self, rank: int) -> int:
        import torch.distributed as dist

        try:
            return dist.get_global_rank(self.nccl_group, rank)
        except Exception:
            return rank

    # ---- device communicator ------------------------------------------------------

    def device_comm(self):
        """The device communicator over all ranks (built collectively on first use)."""
        if self._device_comm is None:
            from .device import DeviceComm

            self._device_comm = DeviceComm(self, self.global_ranks)
        return self._device_comm

    # ---- diagnostics ------------------------------------------------------------------

    def _timeout_error(self, direction: str, peer: int, channel: int, why: str = "") -> CollectiveTimeoutError:
        return CollectiveTimeoutError(
            f"rank {self.rank}: {direction} on channel {channel} to/from rank {peer} "
            f"exceeded {self.op_timeout}s{' (' + why + ')' if why else ''}.\n"
            f"  local state: {self.recorder.context()}\n"
            f"  likely cause: rank {peer} is dead, stuck, or issuing a different "
            f"collective (ranks must call collectives in identical order)."
        )

    def set_op_timeout(self, op_timeout: float | None) -> None:
        self.op_timeout = op_timeout
        self._mesh.set_op_timeout(op_timeout)
        if self._device_comm is not None:
            self._device_comm.set_timeout(op_timeout)

    # ---- lifecycle ------------------------------------------------------------------------

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        if self._device_comm is not None:
            self._device_comm.close()
            self._device_comm = None
        if self._channel_pool is not None:
            self._channel_pool.shutdown(wait=True)
        self._mesh.close()

    def __enter__(self) -> ProcessGroup:
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __repr__(self) -> str:
        return f"<ProcessGroup rank {self.rank}/{self.world_size} channels={self.n_channels}>"
