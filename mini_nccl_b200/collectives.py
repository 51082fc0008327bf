"""Collective operations.

Public surface and semantics match the reference (mini_nccl/collectives.py:
112-562): ``all_reduce`` with the ``ring`` / ``tree`` / ``halving`` / ``naive``
algorithms and an optional narrow ``wire_dtype``, ``broadcast``,
``all_gather`` (returns a list indexed by rank), ``reduce_scatter`` (returns
this rank's chunk, input untouched), ``all_to_all`` and ``barrier``; ops
``sum``/``prod``/``max``/``min``.

Two engines sit behind that surface:

* **CUDA tensors** go to the group's device communicator
  (:mod:`mini_nccl_b200.device`): one sm_100a kernel per collective that
  loads and stores peer HBM over NVLink directly.  On the device the same
  algorithm names select the same *schedules* over peer memory, plus
  ``one_shot`` / ``two_shot`` (peer stores; every peer is one hop away on a
  switch) and ``nvls`` (the NVSwitch adds the ranks' copies itself;
  multimem loads and stores).  ``auto`` picks among the last three.
* **CPU tensors** run the schedules below over the host TCP mesh.  They are
  the parity/testing path and what multi-host CPU runs use.

Every rank must issue collectives in the same order (per communicator).
"""

from __future__ import annotations

import os
from collections.abc import Callable

import torch

from .communicator import Communicator

#: Message size at which ``auto`` switches from the latency-optimal tree to the
#: bandwidth-optimal ring on the host path (the reference measured 1 MiB on
#: loopback TCP, mini_nccl/collectives.py:43-47).
RING_THRESHOLD_BYTES = 1 << 20

#: A ring segment per channel only pays once each channel carries this much.
CHANNEL_MIN_BYTES = int(os.environ.get("MINI_NCCL_CHANNEL_MIN_BYTES", 8 << 20))

#: Receive-slice size for overlapping the reduction with the transfer.
SLICE_TARGET_BYTES = 256 << 10
MAX_SLICES = int(os.environ.get("MINI_NCCL_MAX_SLICES", "1"))

#: Host-path algorithms, in the order benchmarks report them.
ALGORITHMS = ("ring", "tree", "halving", "naive")
#: Extra schedules only the device path implements.
DEVICE_ALGORITHMS = ALGORITHMS + ("one_shot", "two_shot", "nvls")

#: Dtypes too narrow to accumulate many terms in.
LOW_PRECISION = (torch.bfloat16, torch.float16)


def _acc_sum(acc: torch.Tensor, x: torch.Tensor) -> None:
    acc.add_(x)


def _acc_prod(acc: torch.Tensor, x: torch.Tensor) -> None:
    acc.mul_(x)


def _acc_max(acc: torch.Tensor, x: torch.Tensor) -> None:
    torch.maximum(acc, x, out=acc)


def _acc_min(acc: torch.Tensor, x: torch.Tensor) -> None:
    torch.minimum(acc, x, out=acc)


#: In-place ``acc = acc (op) other`` for each reduction op.
_OPS: dict[str, Callable[[torch.Tensor, torch.Tensor], None]] = {
    "sum": _acc_sum,
    "prod": _acc_prod,
    "max": _acc_max,
    "min": _acc_min,
}


def _check_op(op: str) -> None:
    if op not in _OPS:
        raise ValueError(f"unknown op {op!r}; expected one of {sorted(_OPS)}")


def _flat(tensor: torch.Tensor) -> torch.Tensor:
    if not tensor.is_contiguous():
        raise ValueError("collectives require contiguous tensors")
    return tensor.view(-1)


def _n_channels_for(pg: Communicator, nbytes: int) -> int:
    """Channel count from the message size alone, so every rank derives the same."""
    return max(1, min(pg.n_channels, nbytes // CHANNEL_MIN_BYTES))


def _n_slices_for(nbytes: int) -> int:
    return max(1, min(MAX_SLICES, nbytes // SLICE_TARGET_BYTES))


def _split(flat: torch.Tensor, parts: int) -> list[torch.Tensor]:
    """Deterministic contiguous split; the first ``n % parts`` pieces get one extra."""
    n = flat.numel()
    q, extra = divmod(n, parts)
    sizes = [q + (i < extra) for i in range(parts)]
    return list(torch.split(flat, sizes))


def _padded_blocks(flat: torch.Tensor, world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(padded flat buffer, its [world, chunk] view); no copy when it divides."""
    chunk = -(-flat.numel() // world)
    if chunk * world == flat.numel():
        return flat, flat.view(world, chunk)
    buf = torch.zeros(chunk * world, dtype=flat.dtype, device=flat.device)
    buf[: flat.numel()].copy_(flat)
    return buf, buf.view(world, chunk)


def _device_comm(pg: Communicator):
    getter = getattr(pg, "device_comm", None)
    return getter() if callable(getter) else None


# ============================================================================
# all_reduce
# ============================================================================


def all_reduce(
    pg: Communicator,
    tensor: torch.Tensor,
    op: str = "sum",
    algorithm: str = "auto",
    wire_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Reduce ``tensor`` across all ranks, in place, and return it.

    ``wire_dtype`` separates what travels between ranks from what the sum is
    accumulated in (reference semantics, mini_nccl/collectives.py:119-141):
    a float32 tensor with ``wire_dtype=torch.bfloat16`` halves the bytes while
    every addition stays float32.  On the host path the partial sum is
    re-rounded at every hop, so ring error grows with the world size and tree
    error stays flat; the device kernels accumulate every peer's contribution
    in float32 registers and round once, which is at least as accurate.
    """
    _check_op(op)
    if pg.world_size == 1:
        return tensor
    if tensor.is_cuda:
        dc = _device_comm(pg)
        if dc is not None:
            return dc.all_reduce(tensor, op=op, algorithm=algorithm, wire_dtype=wire_dtype)
        host = tensor.detach().cpu().contiguous()
        all_reduce(pg, host, op=op, algorithm=algorithm, wire_dtype=wire_dtype)
        tensor.copy_(host)
        return tensor

    nbytes = tensor.numel() * tensor.element_size()
    if algorithm == "auto":
        algorithm = "tree" if nbytes <= RING_THRESHOLD_BYTES else "ring"
    elif algorithm in ("one_shot", "two_shot", "nvls"):
        # Device-only schedules; on the host their closest analogues.
        algorithm = "naive" if algorithm == "one_shot" else "ring"
    if algorithm == "halving" and (pg.world_size & (pg.world_size - 1)):
        algorithm = "ring"  # power-of-two only; ring is the honest fallback
    if algorithm not in ALGORITHMS:
        raise ValueError(f"unknown algorithm {algorithm!r}")

    if wire_dtype is not None:
        if algorithm not in ("ring", "tree"):
            raise ValueError(f"wire_dtype is implemented for ring and tree, not {algorithm!r}")
        if wire_dtype.itemsize > tensor.element_size():
            raise ValueError(f"wire_dtype {wire_dtype} is wider than the tensor's {tensor.dtype}")
        nbytes = tensor.numel() * wire_dtype.itemsize

    ev = pg.recorder.start(
        "all_reduce", algorithm, channel=-1, nbytes=nbytes, op=op,
        wire=str(wire_dtype) if wire_dtype else "native",
    )
    try:
        flat = _flat(tensor)
        work = flat.float() if (wire_dtype is not None and flat.dtype in LOW_PRECISION) else flat
        if algorithm == "ring":
            segments = _split(work, _n_channels_for(pg, nbytes))
            pg.run_per_channel(
                [
                    (lambda seg=seg, ch=ch: _ring_all_reduce(pg, seg, op, ch, wire_dtype))
                    for ch, seg in enumerate(segments)
                ]
            )
        elif algorithm == "tree":
            _tree_reduce(pg, work, op, root=0, wire_dtype=wire_dtype)
            _tree_broadcast(pg, work, root=0, wire_dtype=wire_dtype)
        elif algorithm == "halving":
            _halving_doubling(pg, work, op)
        else:
            _naive_all_reduce(pg, work, op)
        if work is not flat:
            flat.copy_(work)
    finally:
        pg.recorder.finish(ev)
    return tensor


class _Wire:
    """Cast-down send buffer and cast-up receive buffer for a narrow wire."""

    def __init__(self, numel: int, dtype: torch.dtype | None) -> None:
        self.dtype = dtype
        if dtype is not None:
            self.out = torch.empty(numel, dtype=dtype)
            self.inc = torch.empty(numel, dtype=dtype)

    def pack(self, x: torch.Tensor) -> torch.Tensor:
        if self.dtype is None:
            return x
        view = self.out[: x.numel()]
        view.copy_(x)
        return view


def _ring_all_reduce(
    pg: Communicator,
    segment: torch.Tensor,
    op: str,
    channel: int,
    wire_dtype: torch.dtype | None = None,
) -> None:
    """Reduce-scatter then all-gather around the ring, all on one channel."""
    W, r = pg.world_size, pg.rank
    nbytes = segment.numel() * segment.element_size()
    ev = pg.recorder.start("ring_segment", "ring", channel=channel, nbytes=nbytes)
    try:
        padded, blocks = _padded_blocks(segment, W)
        chunk = blocks.shape[1]
        right, left = (r + 1) % W, (r - 1) % W
        acc = _OPS[op]
        landing = torch.empty(chunk, dtype=segment.dtype)
        wire = _Wire(chunk, wire_dtype)
        slices = _n_slices_for(chunk * segment.element_size())

        # Reduce-scatter: at step s forward the block just accumulated and fold
        # the incoming partial into the next one.  After W-1 steps this rank
        # owns the fully reduced block (r + 1) % W.
        for s in range(W - 1):
            out_b = blocks[(r - s) % W]
            in_b = blocks[(r - s - 1) % W]
            if wire_dtype is None:
                pg.send_recv_sliced(
                    out_b, right, landing, left, slices,
                    lambda lo, hi, t=in_b: acc(t[lo:hi], landing[lo:hi]),
                    channel,
                )
            else:
                pg.send_recv(wire.pack(out_b), right, wire.inc, left, channel)
                if op == "sum":
                    in_b.add_(wire.inc)  # widened inside the add
                else:
                    landing.copy_(wire.inc)
                    acc(in_b, landing)

        # All-gather: circulate the finished blocks.
        for s in range(W - 1):
            out_b = blocks[(r + 1 - s) % W]
            in_b = blocks[(r - s) % W]
            if wire_dtype is None:
                pg.send_recv(out_b, right, in_b, left, channel)
            else:
                pg.send_recv(wire.pack(out_b), right, wire.inc, left, channel)
                in_b.copy_(wire.inc)

        if padded.data_ptr() != segment.data_ptr():
            segment.copy_(padded[: segment.numel()])
    finally:
        pg.recorder.finish(ev)


def _halving_doubling(pg: Communicator, tensor: torch.Tensor, op: str) -> None:
    """Recursive-halving reduce-scatter then recursive-doubling all-gather.

    Partners are ``rank ^ mask`` from the highest bit down, so after the
    halving phase rank ``r`` owns segment ``r`` of the reduced vector and the
    doubling phase retraces the same exchanges in reverse.
    """
    W, r = pg.world_size, pg.rank
    flat = _flat(tensor)
    padded, _ = _padded_blocks(flat, W)
    acc = _OPS[op]
    landing = torch.empty(padded.numel() // 2, dtype=flat.dtype)
    lo, hi = 0, padded.numel()
    bit = W >> 1
    while bit:
        peer = r ^ bit
        mid = (lo + hi) // 2
        upper = bool(r & bit)
        keep = padded[mid:hi] if upper else padded[lo:mid]
        give = padded[lo:mid] if upper else padded[mid:hi]
        inbox = landing[: keep.numel()]
        pg.send_recv_sliced(
            give, peer, inbox, peer, _n_slices_for(keep.numel() * flat.element_size()),
            lambda a, b, k=keep, ib=inbox: acc(k[a:b], ib[a:b]),
        )
        lo, hi = (mid, hi) if upper else (lo, mid)
        bit >>= 1
    bit = 1
    while bit < W:
        peer = r ^ bit
        width = hi - lo
        if r & bit:
            pg.send_recv(padded[lo:hi], peer, padded[lo - width : lo], peer)
            lo -= width
        else:
            pg.send_recv(padded[lo:hi], peer, padded[hi : hi + width], peer)
            hi += width
        bit <<= 1
    if padded.data_ptr() != flat.data_ptr():
        flat.copy_(padded[: flat.numel()])


def _tree_reduce(
    pg: Communicator,
    tensor: torch.Tensor,
    op: str,
    root: int,
    wire_dtype: torch.dtype | None = None,
) -> None:
    """Binomial-tree reduction onto ``root`` (any world size).

    In virtual-rank space (root = 0) a node with lowest set bit ``b`` receives
    from ``v + 2^k`` for every ``2^k < b`` and then sends once to ``v - b``.
    """
    W, r = pg.world_size, pg.rank
    v = (r - root) % W
    flat = _flat(tensor)
    acc = _OPS[op]
    landing = torch.empty_like(flat)
    wire = torch.empty(flat.numel(), dtype=wire_dtype) if wire_dtype is not None else None
    step = 1
    while step < W:
        if v & step:
            parent = (v - step + root) % W
            if wire is None:
                pg.send(flat, parent)
            else:
                wire.copy_(flat)
                pg.send(wire, parent)
            return
        child = v + step
        if child < W:
            src = (child + root) % W
            if wire is None:
                pg.recv(landing, src)
                acc(flat, landing)
            else:
                pg.recv(wire, src)
                if op == "sum":
                    flat.add_(wire)
                else:
                    landing.copy_(wire)
                    acc(flat, landing)
        step <<= 1


def _tree_broadcast(
    pg: Communicator,
    tensor: torch.Tensor,
    root: int,
    wire_dtype: torch.dtype | None = None,
) -> None:
    """Binomial-tree broadcast from ``root``: receive once, then fan out."""
    W, r = pg.world_size, pg.rank
    if W == 1:
        return
    flat = _flat(tensor)
    v = (r - root) % W
    wire = torch.empty(flat.numel(), dtype=wire_dtype) if wire_dtype is not None else None
    if v:
        low = v & -v
        parent = (v - low + root) % W
        if wire is None:
            pg.recv(flat, parent)
        else:
            pg.recv(wire, parent)
            flat.copy_(wire)
        step = low >> 1
    else:
        step = 1 << ((W - 1).bit_length() - 1)
    payload = flat
    if wire is not None:
        wire.copy_(flat)
        payload = wire
    while step:
        if v + step < W:
            pg.send(payload, (v + step + root) % W)
        step >>= 1


def _naive_all_reduce(pg: Communicator, tensor: torch.Tensor, op: str) -> None:
    """Parameter-server baseline: everyone to rank 0, rank 0 back to everyone."""
    W, r = pg.world_size, pg.rank
    flat = _flat(tensor)
    if r:
        pg.send(flat, 0)
        pg.recv(flat, 0)
        return
    acc = _OPS[op]
    landing = torch.empty_like(flat)
    for src in range(1, W):
        pg.recv(landing, src)
        acc(flat, landing)
    for dst in range(1, W):
        pg.send(flat, dst)


# ============================================================================
# the other collectives
# ============================================================================


def broadcast(pg: Communicator, tensor: torch.Tensor, src: int = 0) -> torch.Tensor:
    """Overwrite ``tensor`` on every rank with rank ``src``'s copy."""
    if pg.world_size == 1:
        return tensor
    if tensor.is_cuda:
        dc = _device_comm(pg)
        if dc is not None:
            return dc.broadcast(tensor, src=src)
        host = tensor.detach().cpu().contiguous()
        broadcast(pg, host, src)
        tensor.copy_(host)
        return tensor
    nbytes = tensor.numel() * tensor.element_size()
    ev = pg.recorder.start("broadcast", "tree", channel=-1, nbytes=nbytes, root=src)
    try:
        _tree_broadcast(pg, tensor, root=src)
    finally:
        pg.recorder.finish(ev)
    return tensor


def all_gather(pg: Communicator, tensor: torch.Tensor) -> list[torch.Tensor]:
    """Every rank's ``tensor``, as a list indexed by rank."""
    W, r = pg.world_size, pg.rank
    if tensor.is_cuda and W > 1:
        dc = _device_comm(pg)
        if dc is not None:
            out = dc.all_gather(tensor.contiguous())
            return [out[i].view(tensor.shape) for i in range(W)]
        host = [t.to(tensor.device) for t in all_gather(pg, tensor.detach().cpu())]
        return host
    flat = tensor.contiguous().view(-1)
    table = torch.empty((W, flat.numel()), dtype=flat.dtype, device=flat.device)
    table[r].copy_(flat)
    if W > 1:
        ev = pg.recorder.start(
            "all_gather", "ring", channel=-1, nbytes=flat.numel() * flat.element_size()
        )
        try:
            right, left = (r + 1) % W, (r - 1) % W
            for s in range(W - 1):
                pg.send_recv(table[(r - s) % W], right, table[(r - s - 1) % W], left)
        finally:
            pg.recorder.finish(ev)
    return [table[i].view(tensor.shape) for i in range(W)]


def all_gather_into(pg: Communicator, out: torch.Tensor, tensor: torch.Tensor) -> torch.Tensor:
    """Gather into a preallocated ``[world_size * numel]`` buffer (no list, no copies)."""
    W = pg.world_size
    if out.numel() != W * tensor.numel():
        raise ValueError("output must hold world_size * numel elements")
    if tensor.is_cuda and W > 1:
        dc = _device_comm(pg)
        if dc is not None:
            dc.all_gather(tensor.contiguous(), out=out.view(W, -1))
            return out
    parts = all_gather(pg, tensor)
    out.view(W, -1).copy_(torch.stack([p.reshape(-1) for p in parts]))
    return out


def reduce_scatter(pg: Communicator, tensor: torch.Tensor, op: str = "sum") -> torch.Tensor:
    """Return this rank's ``1/W`` chunk of the reduced tensor; the input is untouched.

    ``tensor.numel()`` must be divisible by the world size.
    """
    _check_op(op)
    W, r = pg.world_size, pg.rank
    flat = _flat(tensor)
    if flat.numel() % W:
        raise ValueError(f"numel {flat.numel()} not divisible by world_size {W}")
    if W == 1:
        return flat.clone()
    if tensor.is_cuda:
        dc = _device_comm(pg)
        if dc is not None:
            return dc.reduce_scatter(flat, op=op)
        host = reduce_scatter(pg, flat.detach().cpu(), op)
        return host.to(tensor.device)
    chunk = flat.numel() // W
    blocks = flat.clone().view(W, chunk)
    landing = torch.empty(chunk, dtype=flat.dtype)
    right, left = (r + 1) % W, (r - 1) % W
    acc = _OPS[op]
    ev = pg.recorder.start(
        "reduce_scatter", "ring", channel=-1, nbytes=flat.numel() * flat.element_size(), op=op
    )
    try:
        # The ring reduce-scatter phase, rotated by one block so the block a
        # rank finishes with is its own index.
        for s in range(W - 1):
            pg.send_recv(blocks[(r - s - 1) % W], right, landing, left)
            acc(blocks[(r - s - 2) % W], landing)
    finally:
        pg.recorder.finish(ev)
    return blocks[r].clone()


def all_to_all(pg: Communicator, tensor: torch.Tensor) -> torch.Tensor:
    """Chunk ``j`` goes to rank ``j``; output chunk ``i`` is what rank ``i`` sent here."""
    W, r = pg.world_size, pg.rank
    flat = _flat(tensor)
    if flat.numel() % W:
        raise ValueError(f"numel {flat.numel()} not divisible by world_size {W}")
    if tensor.is_cuda and W > 1:
        dc = _device_comm(pg)
        if dc is not None:
            return dc.all_to_all(flat).view(tensor.shape)
        return all_to_all(pg, flat.detach().cpu()).to(tensor.device).view(tensor.shape)
    chunk = flat.numel() // W
    out = torch.empty_like(flat)
    mine = slice(r * chunk, (r + 1) * chunk)
    out[mine] = flat[mine]
    if W > 1:
        ev = pg.recorder.start(
            "all_to_all", "pairwise", channel=-1, nbytes=flat.numel() * flat.element_size()
        )
        try:
            # Distance-ordered pairs: at distance d every rank sends to r+d and
            # receives from r-d, so no rank is ever a hotspot.
            for d in range(1, W):
                to, frm = (r + d) % W, (r - d) % W
                pg.send_recv(
                    flat[to * chunk : (to + 1) * chunk], to,
                    out[frm * chunk : (frm + 1) * chunk], frm,
                )
        finally:
            pg.recorder.finish(ev)
    return out.view(tensor.shape)


def barrier(pg: Communicator) -> None:
    """Return only once every rank has entered the barrier.

    Host path: a dissemination barrier, ``ceil(log2 W)`` rounds in which rank
    ``r`` signals ``r + 2^k`` and waits for ``r - 2^k``.
    """
    if pg.world_size == 1:
        return
    W, r = pg.world_size, pg.rank
    ev = pg.recorder.start("barrier", "dissemination", channel=-1, nbytes=0)
    try:
        token_out = torch.zeros(1, dtype=torch.uint8)
        token_in = torch.zeros(1, dtype=torch.uint8)
        dist = 1
        while dist < W:
            pg.send_recv(token_out, (r + dist) % W, token_in, (r - dist) % W)
            dist <<= 1
    finally:
        pg.recorder.finish(ev)
