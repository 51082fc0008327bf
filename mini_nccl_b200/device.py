"""Device communicator: collectives on CUDA tensors as peer-memory kernels.

Replaces the reference's pinned-host staging path (mini_nccl/device.py:
1-320, TCP + D2H/H2D copies) with the B200 design:

1. **Bootstrap, once.**  Each rank allocates a staging buffer and a signal pad
   and exports CUDA IPC handles; the handles are all-gathered over the host
   communicator this device communicator was built from (so a
   :class:`~mini_nccl_b200.mesh.SubGroup` gets a context over exactly its
   members) and every rank maps every peer's memory.
2. **Every collective is one kernel** (``csrc/cuda/comm.cu``) that reads and
   writes peer HBM over NVLink directly, with cross-GPU release/acquire
   signalling and ``%globaltimer`` deadlines; no host round trip, no staging
   through host memory.
3. **Symmetric tensors** (:meth:`symmetric_zeros`): memory every peer has
   mapped.  DDP buckets and FSDP shards live there, so their collectives are
   zero-copy (the two-shot all-reduce runs in place on the bucket).

Algorithm names: ``auto`` picks ``one_shot`` for small messages (one round of
peer reads; lowest latency) and ``two_shot`` (reduce-scatter + all-gather;
bandwidth-optimal) above :data:`ONE_SHOT_MAX_BYTES`.  ``ring``, ``tree``,
``halving`` and ``naive`` run the reference's schedules step by step over
peer memory (for parity and the narrow-wire precision study).

A kernel that waits past the op timeout records the stuck peer in a
host-mapped status block; :meth:`check` turns that into
:class:`~mini_nccl_b200.errors.CollectiveTimeoutError`.
"""

from __future__ import annotations

import os

import torch

from . import collectives as _hostc
from .errors import CollectiveTimeoutError, DeviceCommError

#: Below this many bytes ``auto`` uses the one-shot all-reduce.
ONE_SHOT_MAX_BYTES = int(os.environ.get("MINI_NCCL_ONE_SHOT_MAX_BYTES", 512 << 10))
#: Initial staging buffer per rank (grows on demand, collectively).
STAGING_BYTES = int(os.environ.get("MINI_NCCL_STAGING_BYTES", 64 << 20))
#: CTAs a collective may use (the device meaning of "channels").
MAX_BLOCKS = int(os.environ.get("MINI_NCCL_DEVICE_BLOCKS", 32))

_OPS = {"sum": 0, "prod": 1, "max": 2, "min": 3}
OPNAMES = ["all_reduce", "reduce_scatter", "all_gather", "broadcast", "all_to_all", "barrier", "all_reduce_stepped"]


def _ext():
    from ._build import cuda_ext

    return cuda_ext()


class DeviceComm:
    """Peer-memory collectives among the ranks of one host communicator."""

    def __init__(self, comm, global_ranks: list[int], staging_bytes: int | None = None) -> None:
        if not torch.cuda.is_available():
            raise DeviceCommError("CUDA is not available")
        self.comm = comm
        self.global_ranks = list(global_ranks)
        self.rank = comm.rank
        self.world_size = comm.world_size
        dev = getattr(comm, "device", None)
        self.device = torch.device("cuda", torch.cuda.current_device()) if dev is None or dev.type != "cuda" else dev
        from .utils.launches import CountingProxy

        self.impl = CountingProxy(_ext().DeviceCommImpl(self.rank, self.world_size, self.device.index,
                                                        int(staging_bytes or STAGING_BYTES)))
        timeout = getattr(comm, "op_timeout", None)
        if timeout is None:
            timeout = getattr(getattr(comm, "parent", None), "op_timeout", 300.0) or 300.0
        self.impl.set_timeout(float(timeout))
        if self.world_size > 1:
            self.impl.open_signals(self._all_gather_bytes(bytes(self.impl.signal_handle())))
            self._open(self.impl.staging_segment())
        self.staging_bytes = self.impl.segment_bytes(self.impl.staging_segment())
        self._schedules: dict[tuple, torch.Tensor] = {}
        recorder = getattr(comm, "recorder", None)
        if recorder is not None:
            recorder.attach_device_log(self.device_events)
        self._closed = False

    # ---- bootstrap ------------------------------------------------------------------

    def _all_gather_bytes(self, blob: bytes) -> list[bytes]:
        t = torch.frombuffer(bytearray(blob), dtype=torch.uint8).clone()
        parts = _hostc.all_gather(self.comm, t)
        return [bytes(p.numpy().tobytes()) for p in parts]

    def _open(self, seg: int) -> None:
        handles = self._all_gather_bytes(bytes(self.impl.segment_handle(seg)))
        self.impl.open_segment(seg, handles)

    def _new_segment(self, nbytes: int) -> int:
        seg = self.impl.add_segment(int(nbytes))
        if self.world_size > 1:
            self._open(seg)
        return seg

    def symmetric_zeros(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zeroed tensor every peer has mapped (collective: same size on all ranks).

        The memory belongs to this communicator and stays valid until
        :meth:`close`.
        """
        nbytes = max(16, numel * torch.empty(0, dtype=dtype).element_size())
        seg = self._new_segment((nbytes + 255) // 256 * 256)
        return self.impl.segment_tensor(seg, numel, dtype)

    def scratch_zeros(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zeroed tensor inside the staging buffer's tail is not safe to hand out
        (collectives reuse it), so scratch is ordinary device memory."""
        return torch.zeros(numel, dtype=dtype, device=self.device)

    def _ensure_staging(self, nbytes: int) -> None:
        if nbytes <= self.staging_bytes:
            return
        torch.cuda.current_stream(self.device).synchronize()
        size = max(nbytes, 2 * self.staging_bytes)
        seg = self._new_segment(size)
        self.impl.set_staging(seg)
        self.staging_bytes = size

    # ---- status -----------------------------------------------------------------------

    def set_timeout(self, seconds: float | None) -> None:
        self.impl.set_timeout(1e9 if seconds is None else float(seconds))

    def check(self) -> None:
        """Raise if any kernel of this communicator gave up waiting on a peer."""
        code, peer, block, seq = self.impl.status()
        if code == 0:
            return
        self.impl.clear_status()
        recorder = getattr(self.comm, "recorder", None)
        context = recorder.context() if recorder is not None else ""
        if code == 1:
            raise CollectiveTimeoutError(
                f"rank {self.rank}: device collective #{seq} (block {block}) timed out waiting "
                f"for rank {peer}.\n  local state: {context}\n  likely cause: rank {peer} is dead, "
                f"stuck, or issuing a different collective (ranks must call collectives in "
                f"identical order)."
            )
        raise DeviceCommError(f"rank {self.rank}: device collective #{seq} failed with status {code}")

    def synchronize(self) -> None:
        torch.cuda.current_stream(self.device).synchronize()
        self.check()

    def device_events(self) -> list[dict]:
        out = []
        for e in self.impl.events(4096):
            code = int(e["opcode"])
            e = dict(e)
            e["op"] = OPNAMES[code] if 0 <= code < len(OPNAMES) else str(code)
            out.append(e)
        return out

    # ---- collectives ------------------------------------------------------------------

    def _record(self, name: str, algorithm: str, nbytes: int, **detail):
        rec = getattr(self.comm, "recorder", None)
        return rec.start(name, algorithm, channel=-1, nbytes=nbytes, device=True, **detail) if rec is not None else None

    def _finish(self, ev) -> None:
        rec = getattr(self.comm, "recorder", None)
        if rec is not None:
            rec.finish(ev)

    def all_reduce(
        self,
        tensor: torch.Tensor,
        op: str = "sum",
        algorithm: str = "auto",
        wire_dtype: torch.dtype | None = None,
        scale: float = 1.0,
    ) -> torch.Tensor:
        if op not in _OPS:
            raise ValueError(f"unknown op {op!r}; expected one of {sorted(_OPS)}")
        if not tensor.is_contiguous():
            raise ValueError("collectives require contiguous tensors")
        if self.world_size == 1:
            if scale != 1.0:
                tensor.mul_(scale)
            return tensor
        nbytes = tensor.numel() * tensor.element_size()
        if algorithm == "auto":
            algorithm = "one_shot" if nbytes <= ONE_SHOT_MAX_BYTES else "two_shot"
        if algorithm == "halving" and (self.world_size & (self.world_size - 1)):
            algorithm = "ring"
        wire_bf16 = 0
        if wire_dtype is not None:
            if wire_dtype.itemsize > tensor.element_size():
                raise ValueError(f"wire_dtype {wire_dtype} is wider than the tensor's {tensor.dtype}")
            if wire_dtype not in (torch.bfloat16, tensor.dtype):
                raise ValueError("the device wire type must be bfloat16")
            wire_bf16 = int(wire_dtype == torch.bfloat16)
        ev = self._record("all_reduce", algorithm, nbytes, op=op,
                          wire=str(wire_dtype) if wire_dtype else "native")
        try:
            if algorithm in ("one_shot", "two_shot"):
                wire_bf16 = wire_bf16 if tensor.dtype == torch.float32 else 0
                step_bytes = tensor.numel() * (2 if wire_bf16 else tensor.element_size())
                zero_copy = algorithm == "two_shot" and not wire_bf16 and self.impl.is_symmetric(tensor)
                if not zero_copy:
                    self._ensure_staging(step_bytes)
                self.impl.all_reduce(tensor, tensor, _OPS[op], 1 if algorithm == "two_shot" else 0,
                                     wire_bf16, float(scale), MAX_BLOCKS)
            elif algorithm in ("ring", "tree", "halving", "naive"):
                self._ensure_staging(tensor.numel() * max(4, tensor.element_size()))
                steps = self._schedule(algorithm, tensor.numel())
                self.impl.stepped_all_reduce(tensor, tensor, steps, _OPS[op], wire_bf16, float(scale))
            else:
                raise ValueError(f"unknown algorithm {algorithm!r}")
        finally:
            self._finish(ev)
        return tensor

    def reduce_scatter(self, flat: torch.Tensor, op: str = "sum", scale: float = 1.0) -> torch.Tensor:
        W = self.world_size
        if flat.numel() % W:
            raise ValueError(f"numel {flat.numel()} not divisible by world_size {W}")
        out = torch.empty(flat.numel() // W, dtype=flat.dtype, device=flat.device)
        if W == 1:
            out.copy_(flat)
            return out.mul_(scale) if scale != 1.0 else out
        nbytes = flat.numel() * flat.element_size()
        if not self.impl.is_symmetric(flat):
            self._ensure_staging(nbytes)
        ev = self._record("reduce_scatter", "direct", nbytes, op=op)
        try:
            self.impl.reduce_scatter(flat, out, _OPS[op], float(scale), min(MAX_BLOCKS, 512 // W))
        finally:
            self._finish(ev)
        return out

    def all_gather(self, shard: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        W = self.world_size
        if out is None:
            out = torch.empty((W, shard.numel()), dtype=shard.dtype, device=shard.device)
        if W == 1:
            out.view(-1).copy_(shard.reshape(-1))
            return out
        nbytes = shard.numel() * shard.element_size()
        if not self.impl.is_symmetric(shard):
            self._ensure_staging(nbytes)
        ev = self._record("all_gather", "direct", nbytes)
        try:
            self.impl.move(shard.contiguous(), out, 0, 0, min(MAX_BLOCKS, 512 // W))
        finally:
            self._finish(ev)
        return out

    def broadcast(self, tensor: torch.Tensor, src: int = 0) -> torch.Tensor:
        if self.world_size == 1:
            return tensor
        nbytes = tensor.numel() * tensor.element_size()
        if not self.impl.is_symmetric(tensor):
            self._ensure_staging(nbytes)
        ev = self._record("broadcast", "direct", nbytes, root=src)
        try:
            self.impl.move(tensor, tensor, 1, int(src), min(MAX_BLOCKS, 512 // self.world_size))
        finally:
            self._finish(ev)
        return tensor

    def all_to_all(self, flat: torch.Tensor) -> torch.Tensor:
        W = self.world_size
        out = torch.empty_like(flat)
        if W == 1:
            return out.copy_(flat)
        nbytes = flat.numel() * flat.element_size()
        if not self.impl.is_symmetric(flat):
            self._ensure_staging(nbytes)
        ev = self._record("all_to_all", "direct", nbytes)
        try:
            self.impl.move(flat, out, 2, 0, min(MAX_BLOCKS, 512 // W))
        finally:
            self._finish(ev)
        return out

    def barrier(self) -> None:
        if self.world_size > 1:
            ev = self._record("barrier", "device", 0)
            try:
                self.impl.barrier()
            finally:
                self._finish(ev)

    def all_reduce_multi(self, tensors: list[torch.Tensor], scale: float = 1.0) -> int:
        """Average a list of same-dtype tensors with one collective."""
        if not tensors:
            return 0
        flat = torch.cat([t.reshape(-1) for t in tensors])
        self.all_reduce(flat, scale=scale)
        at = 0
        for t in tensors:
            n = t.numel()
            t.copy_(flat[at : at + n].view_as(t))
            at += n
        return flat.numel() * flat.element_size()

    # ---- parity schedules -------------------------------------------------------------

    def _schedule(self, algorithm: str, n: int) -> torch.Tensor:
        key = (algorithm, n)
        hit = self._schedules.get(key)
        if hit is None:
            rows = schedule_steps(algorithm, self.world_size, self.rank, n)
            hit = torch.tensor(rows if rows else [[0, 0, 0, 0, 0]], dtype=torch.int64).to(self.device)
            if not rows:
                hit = hit[:0]
            self._schedules[key] = hit
        return hit

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self.impl.close()


def _split_bounds(n: int, parts: int) -> list[int]:
    q, extra = divmod(n, parts)
    bounds = [0]
    for i in range(parts):
        bounds.append(bounds[-1] + q + (1 if i < extra else 0))
    return bounds


def schedule_steps(algorithm: str, W: int, r: int, n: int) -> list[list[int]]:
    """Pull-form steps ``[peer, src_off, dst_off, count, mode]`` for this rank.

    Mode 1 folds the peer's range into ours, mode 2 copies it, mode 0 idles
    (every rank still joins the step's barrier).  Each schedule is the pull
    formulation of the host algorithm of the same name, so it performs the
    same additions in the same order and rounds onto the wire at each hop.
    """
    steps: list[list[int]] = []
    idle = [0, 0, 0, 0, 0]
    if algorithm == "ring":
        b = _split_bounds(n, W)
        left = (r - 1) % W
        for s in range(W - 1):  # reduce-scatter
            i = (r - s - 1) % W
            steps.append([left, b[i], b[i], b[i + 1] - b[i], 1])
        for s in range(W - 1):  # all-gather
            i = (r - s) % W
            steps.append([left, b[i], b[i], b[i + 1] - b[i], 2])
    elif algorithm == "tree":
        step = 1
        while step < W:  # binomial reduce onto rank 0
            if r % (2 * step) == 0 and r + step < W:
                steps.append([r + step, 0, 0, n, 1])
            else:
                steps.append(idle)
            step <<= 1
        top = 1 << ((W - 1).bit_length() - 1) if W > 1 else 0
        m = top
        while m:  # binomial broadcast from rank 0
            if r & (2 * m - 1) == m:
                steps.append([r - m, 0, 0, n, 2])
            else:
                steps.append(idle)
            m >>= 1
    elif algorithm == "halving":
        lo, hi = 0, n
        # pad-free halving on element ranges: halves are computed identically on partners
        mask = W >> 1
        ranges = []
        while mask:
            partner = r ^ mask
            mid = (lo + hi) // 2
            lo, hi = (mid, hi) if r & mask else (lo, mid)
            steps.append([partner, lo, lo, hi - lo, 1])
            ranges.append((mask, lo, hi))
            mask >>= 1
        for mask, _, _ in reversed(ranges):  # doubling: fetch the partner's owned range
            partner = r ^ mask
            plo, phi = _owned_after_halving(W, partner, n, mask)
            steps.append([partner, plo, plo, phi - plo, 2])
    elif algorithm == "naive":
        for src in range(1, W):
            steps.append([src, 0, 0, n, 1] if r == 0 else idle)
        steps.append(idle if r == 0 else [0, 0, 0, n, 2])
    else:
        raise ValueError(f"unknown algorithm {algorithm!r}")
    return steps


def _owned_after_halving(W: int, rank: int, n: int, stop_mask: int) -> tuple[int, int]:
    """Range ``rank`` owns in the doubling phase once masks above ``stop_mask`` merged.

    Walk the halving phase down to ``stop_mask`` (inclusive) for ``rank``:
    that is the range it holds fully reduced *at the doubling level* just
    before exchanging with the partner across ``stop_mask``.
    """
    lo, hi = 0, n
    mask = W >> 1
    while mask:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if rank & mask else (lo, mid)
        if mask == stop_mask:
            break
        mask >>= 1
    # Doubling below stop_mask has already widened the range back up to the
    # block covered at level stop_mask, which is exactly (lo, hi) above.
    return lo, hi
