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

4. **NVLS (NVLink SHARP)**, where the GPUs and the driver support multicast
   objects: at set-up the ranks build a multicast object over NVSwitch (rank
   0 creates it and hands it to the others as a file descriptor over a Unix
   socket; each rank binds its own memory), and sum reductions run as
   ``multimem.ld_reduce`` (the switch adds every rank's copy and returns the
   sum) plus ``multimem.st`` (one store reaches every rank).  A tensor made by
   :meth:`symmetric_zeros` with ``nvls=True`` (DDP's buckets) is reduced in
   place; other tensors go through an NVLS staging buffer.

Algorithm names: ``auto`` picks ``one_shot`` for small messages (one round of
peer stores; lowest latency), ``nvls`` for sum all-reduces of fp32 / bf16 /
fp16 from :data:`NVLS_MIN_BYTES` on at :data:`NVLS_MIN_WORLD` ranks or more
(and always for tensors that live in NVLS memory), and ``two_shot``
(reduce-scatter + all-gather by peer stores) for the rest above
:data:`ONE_SHOT_MAX_BYTES`.  Reduce-scatter, all-gather and broadcast take
the switch only for tensors already in multicast memory: on other tensors
the staging copy leaves the direct peer-store kernels ahead.  ``ring``, ``tree``, ``halving``
and ``naive`` run the reference's schedules step by step over peer memory
(for parity and the narrow-wire precision study).  The cut-over sizes come
from the measured sweep in ``results/`` (``benchmarks/bench_collectives.py``)
and can be overridden by environment variables.

A kernel that waits past the op timeout records the stuck peer in a
host-mapped status block; :meth:`check` turns that into
:class:`~mini_nccl_b200.errors.CollectiveTimeoutError`.
"""

from __future__ import annotations

import os

import torch

from . import collectives as _hostc
from .errors import CollectiveTimeoutError, DeviceCommError
from .utils import nvtx as _nvtx

#: Up to this many bytes ``auto`` uses the one-shot all-reduce (when NVLS is
#: not chosen).  Measured cut-over against the two-shot kernel on a
#: non-symmetric buffer: one-shot is ahead through 8 MiB and behind from
#: 16 MiB on, at W = 2 (results/collectives_w2.csv) and at W = 8
#: (results/collectives_w8_bf16.csv).
ONE_SHOT_MAX_BYTES = int(os.environ.get("MINI_NCCL_ONE_SHOT_MAX_BYTES", 8 << 20))
#: Initial staging buffer per rank (grows on demand, collectively).
STAGING_BYTES = int(os.environ.get("MINI_NCCL_STAGING_BYTES", 64 << 20))
#: CTAs a collective may use (the device meaning of "channels").  Bandwidth
#: grows with CTAs up to about one per SM; fewer leave SMs to overlapped compute.
MAX_BLOCKS = int(os.environ.get("MINI_NCCL_DEVICE_BLOCKS", 255))
#: CTAs (128 threads each) of an all-reduce run beside compute: one per SM.
BESIDE_BLOCKS = int(os.environ.get("MINI_NCCL_BESIDE_BLOCKS", 148))
#: NVLS collectives on (where the hardware and driver support them).
NVLS_ENABLED = os.environ.get("MINI_NCCL_NVLS", "1") != "0"
#: From this many bytes on ``auto`` sends all-reduces through the switch ...
#: (W = 8 sweep, bf16: one-shot ahead at 1 MiB, 30.8 vs 26.6 GB/s busbw; NVLS
#: ahead at 4 MiB, 99.8 vs 80.0)
NVLS_MIN_BYTES = int(os.environ.get("MINI_NCCL_NVLS_MIN_BYTES", 2 << 20))
#: ... on communicators of at least this many ranks.  With W ranks an NVLS
#: all-reduce moves about (1 + 1/W) x the message per GPU each way against
#: 2 (W-1)/W for two-shot: at W = 2 that is 1.5 vs 1 and the measured sweep
#: has two-shot ahead at every size; from W = 4 on the switch moves less.
NVLS_MIN_WORLD = int(os.environ.get("MINI_NCCL_NVLS_MIN_WORLD", 4))
#: CTAs an NVLS collective may use (each multimem access is one 16-byte request
#: the switch serves, so far fewer CTAs than the peer kernels need).
NVLS_BLOCKS = int(os.environ.get("MINI_NCCL_NVLS_BLOCKS", 64))
#: CTAs (128 threads) of an NVLS all-reduce that runs beside compute.
NVLS_BESIDE_BLOCKS = int(os.environ.get("MINI_NCCL_NVLS_BESIDE_BLOCKS", 64))
#: Initial NVLS staging buffer per rank (grows on demand, collectively).
NVLS_STAGING_BYTES = int(os.environ.get("MINI_NCCL_NVLS_STAGING_BYTES", 64 << 20))
#: Seconds the multicast set-up waits for a peer (socket hand-off).
NVLS_SETUP_TIMEOUT = float(os.environ.get("MINI_NCCL_NVLS_SETUP_TIMEOUT", 60.0))
_NVLS_DTYPES = (torch.float32, torch.bfloat16, torch.float16)

_OPS = {"sum": 0, "prod": 1, "max": 2, "min": 3}
OPNAMES = ["all_reduce", "reduce_scatter", "all_gather", "broadcast", "all_to_all", "barrier", "all_reduce_stepped",
           "gemm_reduce_scatter", "all_gather_gemm", "reduce_scatter_adamw", "gather_weight_gemm",
           "all_reduce_adamw"]


def _ext():
    from ._build import cuda_ext

    return cuda_ext()


def all_gather_blobs(comm, blob: bytes) -> list[bytes]:
    """Every rank's byte string, in rank order, over the host communicator.

    Blobs may differ in length (socket names, error messages) and may be
    empty: the lengths are gathered first, then every blob padded to the
    longest one, and each is cut back to its own length.
    """
    sizes = _hostc.all_gather(comm, torch.tensor([len(blob)], dtype=torch.int64))
    lengths = [int(s.item()) for s in sizes]
    longest = max(lengths)
    if longest == 0:
        return [b"" for _ in lengths]
    padded = torch.zeros(longest, dtype=torch.uint8)
    if blob:
        padded[: len(blob)] = torch.frombuffer(bytearray(blob), dtype=torch.uint8)
    parts = _hostc.all_gather(comm, padded)
    return [bytes(part[:n].numpy().tobytes()) for part, n in zip(parts, lengths, strict=True)]


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
        #: Whether NVLS collectives are available; :attr:`nvls_reason` says why not.
        self.nvls = False
        self.nvls_reason = "disabled (MINI_NCCL_NVLS=0)" if not NVLS_ENABLED else "single rank"
        self._nvls_objects: list[int] = []
        self._nvls_staging = -1
        if self.world_size > 1 and NVLS_ENABLED:
            self._init_nvls()
        self._schedules: dict[tuple, torch.Tensor] = {}
        self._last_issued: torch.cuda.Event | None = None
        self._nvtx_open: list[bool] = []
        recorder = getattr(comm, "recorder", None)
        if recorder is not None:
            recorder.attach_device_log(self.device_events)
        self._closed = False

    # ---- bootstrap ------------------------------------------------------------------

    def _all_gather_bytes(self, blob: bytes) -> list[bytes]:
        return all_gather_blobs(self.comm, blob)

    def _open(self, seg: int) -> None:
        handles = self._all_gather_bytes(bytes(self.impl.segment_handle(seg)))
        self.impl.open_segment(seg, handles)

    def _new_segment(self, nbytes: int) -> int:
        seg = self.impl.add_segment(int(nbytes))
        if self.world_size > 1:
            self._open(seg)
        return seg

    def symmetric_zeros(self, numel: int, dtype: torch.dtype, nvls: bool = False) -> torch.Tensor:
        """A zeroed tensor every peer has mapped (collective: same size on all ranks).

        ``nvls=True`` puts it in memory bound to an NVLS multicast object
        (when NVLS is available), so sum all-reduces on it run in place
        through the switch; otherwise peers map it through CUDA IPC.  The
        memory belongs to this communicator and stays valid until :meth:`close`.
        """
        nbytes = max(16, numel * torch.empty(0, dtype=dtype).element_size())
        if nvls and self.nvls:
            oid = self._nvls_new((nbytes + 255) // 256 * 256)
            return self.impl.nvls_tensor(oid, numel, dtype)
        seg = self._new_segment((nbytes + 255) // 256 * 256)
        return self.impl.segment_tensor(seg, numel, dtype)

    # ---- NVLS multicast objects -------------------------------------------------------

    def _agree(self, ok: bool) -> bool:
        """True when every rank passes True (a host collective, so also a barrier)."""
        return all(f == b"\x01" for f in self._all_gather_bytes(b"\x01" if ok else b"\x00"))

    def _nvls_new(self, nbytes: int) -> int:
        """Build one multicast object over every rank (collective).

        Each step ends with every rank agreeing that it worked, so a failure
        on one rank leaves every rank releasing its part and raising."""
        oid, err = None, ""
        try:
            oid = self.impl.nvls_create(int(nbytes))
        except RuntimeError as exc:
            err = str(exc)
        steps = (
            lambda: self.impl.nvls_exchange(oid, [bytes(n).decode() for n in self._all_gather_bytes(
                bytes(self.impl.nvls_socket_name(oid)) if oid is not None else b"")], NVLS_SETUP_TIMEOUT),
            lambda: self.impl.nvls_bind(oid),
        )
        if self._agree(oid is not None):
            for step in steps:
                ok = True
                try:
                    step()
                except RuntimeError as exc:
                    ok, err = False, str(exc)
                if not self._agree(ok):
                    break
            else:
                self._nvls_objects.append(oid)
                return oid
        if oid is not None:
            self.impl.nvls_release(oid)
        raise DeviceCommError(f"rank {self.rank}: NVLS set-up failed: {err or 'a peer failed'}")

    def _init_nvls(self) -> None:
        reasons = [bytes(r).decode() for r in self._all_gather_bytes(self.impl.nvls_reason().encode())]
        bad = [f"rank {r}: {why}" for r, why in enumerate(reasons) if why]
        if bad:
            self.nvls_reason = "; ".join(bad)
            return
        try:
            self._nvls_staging = self._nvls_new(2 * NVLS_STAGING_BYTES)
        except DeviceCommError as exc:
            self.nvls_reason = str(exc)
            return
        self.impl.set_nvls_staging(self._nvls_staging)
        self.nvls = True
        self.nvls_reason = ""

    def _ensure_nvls_staging(self, nbytes: int) -> None:
        """Grow the NVLS staging buffer (collectively: every rank makes the same call)."""
        if nbytes <= self.impl.nvls_staging_half():
            return
        size = 2 * max(nbytes, 2 * self.impl.nvls_staging_half())
        torch.cuda.synchronize(self.device)
        self._agree(True)  # nobody still runs a kernel on the old buffer
        old = self._nvls_staging
        self._nvls_staging = self._nvls_new(size)
        self.impl.set_nvls_staging(self._nvls_staging)
        self.impl.nvls_release(old)
        self._nvls_objects.remove(old)

    def _nvls_sum_ok(self, tensor: torch.Tensor, op: str) -> bool:
        return self.nvls and op == "sum" and tensor.dtype in _NVLS_DTYPES

    def scratch_zeros(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zeroed tensor inside the staging buffer's tail is not safe to hand out
        (collectives reuse it), so scratch is ordinary device memory."""
        return torch.zeros(numel, dtype=dtype, device=self.device)

    def _ensure_staging(self, nbytes: int) -> None:
        """Grow the staging buffer (collectively: every rank makes the same call)."""
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
        self._order_after_previous()
        self._nvtx_open.append(_nvtx.push(_nvtx.label(name, algorithm, nbytes)))
        rec = getattr(self.comm, "recorder", None)
        return rec.start(name, algorithm, channel=-1, nbytes=nbytes, device=True, **detail) if rec is not None else None

    def _finish(self, ev) -> None:
        self._mark_issued()
        rec = getattr(self.comm, "recorder", None)
        if rec is not None:
            rec.finish(ev)
        _nvtx.pop(self._nvtx_open.pop() if self._nvtx_open else False)

    # Every kernel of this communicator runs in host issue order, whichever
    # stream it is launched on: the kernels of different ranks wait for one
    # another, so two of them reordered by the streams on one rank but not on
    # another would each wait for a peer that is running the other one.
    def _order_after_previous(self) -> None:
        last = self._last_issued
        if last is not None:
            torch.cuda.current_stream(self.device).wait_event(last)

    def _mark_issued(self) -> None:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._last_issued = ev

    def all_reduce(
        self,
        tensor: torch.Tensor,
        op: str = "sum",
        algorithm: str = "auto",
        wire_dtype: torch.dtype | None = None,
        scale: float = 1.0,
        blocks: int | None = None,
        beside_compute: bool = False,
    ) -> torch.Tensor:
        """All-reduce ``tensor`` in place across the communicator.

        ``beside_compute=True`` (two-shot sums of bf16 / fp32) launches small
        CTAs that fit on an SM next to one CTA of the persistent GEMM and
        attention kernels, for all-reduces that overlap compute (DDP's
        buckets); every rank must pass the same value.
        """
        if op not in _OPS:
            raise ValueError(f"unknown op {op!r}; expected one of {sorted(_OPS)}")
        if not tensor.is_contiguous():
            raise ValueError("collectives require contiguous tensors")
        if self.world_size == 1:
            if scale != 1.0:
                tensor.mul_(scale)
            return tensor
        nbytes = tensor.numel() * tensor.element_size()
        wire_bf16 = 0
        if wire_dtype is not None:
            if wire_dtype.itemsize > tensor.element_size():
                raise ValueError(f"wire_dtype {wire_dtype} is wider than the tensor's {tensor.dtype}")
            if wire_dtype not in (torch.bfloat16, tensor.dtype):
                raise ValueError("the device wire type must be bfloat16")
            wire_bf16 = int(wire_dtype == torch.bfloat16)
        # the switch reads the tensor's own type: a narrower wire needs the peer kernels
        nvls_ok = self._nvls_sum_ok(tensor, op) and not (wire_bf16 and tensor.dtype != torch.bfloat16)
        if algorithm == "auto":
            algorithm = auto_all_reduce_algorithm(nbytes, self.world_size, nvls_ok,
                                                  nvls_ok and self.impl.is_nvls(tensor))
        if algorithm == "nvls" and not nvls_ok:
            raise ValueError(f"nvls all-reduce needs NVLS ({self.nvls_reason or 'available'}), op='sum', "
                             f"an fp32 / bf16 / fp16 tensor and no narrower wire type")
        if algorithm == "halving" and (self.world_size & (self.world_size - 1)):
            algorithm = "ring"
        ev = self._record("all_reduce", algorithm, nbytes, op=op,
                          wire=str(wire_dtype) if wire_dtype else "native")
        try:
            if algorithm == "nvls":
                if not self.impl.is_nvls(tensor):
                    self._ensure_nvls_staging((nbytes + 15) // 16 * 16)
                nb = blocks or (NVLS_BESIDE_BLOCKS if beside_compute else NVLS_BLOCKS)
                self.impl.nvls_all_reduce(tensor, tensor, float(scale), -nb if beside_compute else nb)
            elif algorithm in ("one_shot", "two_shot"):
                wire_bf16 = wire_bf16 if tensor.dtype == torch.float32 else 0
                wsz = 2 if wire_bf16 else tensor.element_size()
                kind = 1 if algorithm == "two_shot" else 0
                self._ensure_staging(self.impl.staging_need(kind, tensor.numel(), wsz))
                nb = blocks or (BESIDE_BLOCKS if beside_compute else MAX_BLOCKS)
                self.impl.all_reduce(tensor, tensor, _OPS[op], kind, wire_bf16, float(scale),
                                     -nb if beside_compute else nb)
            elif algorithm in ("ring", "tree", "halving", "naive"):
                narrow = tensor.dtype in (torch.bfloat16, torch.float16) and wire_bf16
                self._ensure_staging(self.impl.staging_need(5, tensor.numel(), 4 if narrow else tensor.element_size()))
                steps = self._schedule(algorithm, tensor.numel())
                self.impl.stepped_all_reduce(tensor, tensor, steps, _OPS[op], wire_bf16, float(scale))
            else:
                raise ValueError(f"unknown algorithm {algorithm!r}")
        finally:
            self._finish(ev)
        return tensor

    def reduce_scatter(self, flat: torch.Tensor, op: str = "sum", scale: float = 1.0,
                       blocks: int | None = None, algorithm: str = "auto") -> torch.Tensor:
        """This rank's chunk of the sum (op) over ranks; ``algorithm``: ``auto``,
        ``nvls`` (through the switch) or ``direct`` (peer stores)."""
        W = self.world_size
        if flat.numel() % W:
            raise ValueError(f"numel {flat.numel()} not divisible by world_size {W}")
        out = torch.empty(flat.numel() // W, dtype=flat.dtype, device=flat.device)
        if W == 1:
            out.copy_(flat)
            return out.mul_(scale) if scale != 1.0 else out
        nbytes = flat.numel() * flat.element_size()
        # auto: the switch only for an input already in multicast memory; on
        # other tensors the staging copy makes the direct kernel faster (W = 8
        # sweep: 488 vs 439 GB/s busbw at 1 GiB, ahead at every size)
        nvls = _pick(algorithm, self._nvls_sum_ok(flat, op) and (out.numel() * out.element_size()) % 16 == 0,
                     self.impl.is_nvls(flat), "reduce_scatter")
        if nvls:
            if not self.impl.is_nvls(flat):
                self._ensure_nvls_staging(nbytes)
        else:
            self._ensure_staging(self.impl.staging_need(2, flat.numel(), flat.element_size()))
        ev = self._record("reduce_scatter", "nvls" if nvls else "direct", nbytes, op=op)
        try:
            if nvls:
                self.impl.nvls_reduce_scatter(flat, out, float(scale), blocks or NVLS_BLOCKS)
            else:
                self.impl.reduce_scatter(flat, out, _OPS[op], float(scale), blocks or MAX_BLOCKS)
        finally:
            self._finish(ev)
        return out

    def reduce_scatter_adamw(self, flat_grad: torch.Tensor, param_shard: torch.Tensor, state: dict,
                             *, lr: float, betas: tuple[float, float], eps: float, weight_decay: float,
                             step: int, scale: float = 1.0, blocks: int | None = None) -> None:
        """Reduce-scatter ``flat_grad`` and apply AdamW to this rank's shard, in one kernel.

        ``state`` holds fp32 ``m``, ``v`` and (for bf16 parameters) ``master``
        tensors of the shard's length; ``step`` is the 1-based step count of
        this shard's moments.  Same update as :class:`ops.kernels.FusedAdamW`
        (decoupled weight decay, bias-corrected moments), applied to
        ``sum over ranks of flat_grad`` times ``scale`` (1/W for an average).
        """
        W = self.world_size
        if flat_grad.numel() % W:
            raise ValueError(f"gradient length {flat_grad.numel()} not divisible by world_size {W}")
        b1, b2 = betas
        nbytes = flat_grad.numel() * flat_grad.element_size()
        # overlapped with backward: the switch path wins at every world size here
        # (it leaves the SMs and most of the HBM bandwidth to the compute)
        nvls = (self._nvls_sum_ok(flat_grad, "sum") and flat_grad.dtype != torch.float16
                and (nbytes // W) % 16 == 0 and (nbytes >= NVLS_MIN_BYTES or self.impl.is_nvls(flat_grad)))
        if nvls:
            if not self.impl.is_nvls(flat_grad):
                self._ensure_nvls_staging(nbytes)
        else:
            self._ensure_staging(self.impl.staging_need(2, flat_grad.numel(), flat_grad.element_size()))
        ev = self._record("reduce_scatter_adamw", "nvls" if nvls else "fused", nbytes)
        args = (flat_grad, param_shard, state.get("master"), state["m"], state["v"], float(lr), float(b1), float(b2),
                float(eps), float(weight_decay), 1.0 - b1 ** step, 1.0 - b2 ** step, float(scale))
        try:
            if nvls:
                self.impl.nvls_rs_adamw(*args, blocks or NVLS_BLOCKS)
            else:
                self.impl.reduce_scatter_adamw(*args, blocks or MAX_BLOCKS)
        finally:
            self._finish(ev)

    def all_reduce_adamw(self, grad_bucket: torch.Tensor, param_bucket: torch.Tensor, state: dict, *, lr: float,
                         betas: tuple[float, float], eps: float, weight_decay: float, step: int, scale: float = 1.0,
                         beside_compute: bool = False, blocks: int | None = None) -> None:
        """One DDP bucket's gradient average and AdamW step as one kernel (ZeRO-1 layout).

        Rank r reduces the gradients of its 1/W slice of the bucket, applies
        AdamW to that slice (``state``: fp32 ``master``, ``m``, ``v`` of the
        slice's length) and writes the new parameters into every rank's
        ``param_bucket``: a reduce-scatter of gradients and an all-gather of
        parameters, the bytes of the all-reduce it replaces.  Both buckets are
        symmetric tensors of this communicator (NVLS ones reduce in the
        switch and store by multicast).  ``step`` is the 1-based update count.
        """
        b1, b2 = betas
        nbytes = grad_bucket.numel() * grad_bucket.element_size()
        nvls = self.impl.is_nvls(grad_bucket) and self.impl.is_nvls(param_bucket)
        if not nvls:
            self._ensure_staging(2 * nbytes)
        ev = self._record("all_reduce_adamw", "nvls" if nvls else "two_shot", nbytes)
        try:
            # the optimizer's state traffic and arithmetic ride along: one small CTA per SM
            nb = blocks or (BESIDE_BLOCKS if beside_compute else MAX_BLOCKS)
            self.impl.all_reduce_adamw(grad_bucket, param_bucket, state["master"], state["m"], state["v"], float(lr),
                                       float(b1), float(b2), float(eps), float(weight_decay), 1.0 - b1 ** step,
                                       1.0 - b2 ** step, float(scale), -nb if beside_compute else nb)
        finally:
            self._finish(ev)

    def all_gather(self, shard: torch.Tensor, out: torch.Tensor | None = None,
                   blocks: int | None = None, algorithm: str = "auto") -> torch.Tensor:
        W = self.world_size
        if out is None:
            out = torch.empty((W, shard.numel()), dtype=shard.dtype, device=shard.device)
        if W == 1:
            out.view(-1).copy_(shard.reshape(-1))
            return out
        nbytes = shard.numel() * shard.element_size()
        # auto: direct (W = 8 sweep: ahead of the switch path at every size)
        nvls = _pick(algorithm, self.nvls and nbytes % 16 == 0, False, "all_gather")
        if nvls:
            self._ensure_nvls_staging(nbytes * W)
        else:
            self._ensure_staging(self.impl.staging_need(3, nbytes, 1))
        ev = self._record("all_gather", "nvls" if nvls else "direct", nbytes)
        try:
            if nvls:
                self.impl.nvls_move(shard.contiguous(), out, 0, 0, blocks or NVLS_BLOCKS)
            else:
                self.impl.move(shard.contiguous(), out, 0, 0, blocks or MAX_BLOCKS)
        finally:
            self._finish(ev)
        return out

    def broadcast(self, tensor: torch.Tensor, src: int = 0, algorithm: str = "auto") -> torch.Tensor:
        if self.world_size == 1:
            return tensor
        nbytes = tensor.numel() * tensor.element_size()
        # auto: direct (W = 8 sweep: ahead of the switch path at every size)
        nvls = _pick(algorithm, self.nvls and nbytes % 16 == 0, False, "broadcast")
        if nvls:
            self._ensure_nvls_staging(nbytes)
        else:
            self._ensure_staging(self.impl.staging_need(4, nbytes, 1))
        ev = self._record("broadcast", "nvls" if nvls else "direct", nbytes, root=src)
        try:
            if nvls:
                self.impl.nvls_move(tensor, tensor, 1, int(src), NVLS_BLOCKS)
            else:
                self.impl.move(tensor, tensor, 1, int(src), MAX_BLOCKS)
        finally:
            self._finish(ev)
        return tensor

    def all_to_all(self, flat: torch.Tensor) -> torch.Tensor:
        W = self.world_size
        out = torch.empty_like(flat)
        if W == 1:
            return out.copy_(flat)
        nbytes = flat.numel() * flat.element_size()
        self._ensure_staging(self.impl.staging_need(3, nbytes // W, 1))
        ev = self._record("all_to_all", "direct", nbytes)
        try:
            self.impl.move(flat, out, 2, 0, MAX_BLOCKS)
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

    # ---- GEMMs fused with a collective (tensor parallelism, sequence-parallel layout) ---

    def gemm_reduce_scatter(self, x: torch.Tensor, w: torch.Tensor, *, w_mn: bool = False,
                            bias: torch.Tensor | None = None, resid: torch.Tensor | None = None,
                            force_kernel: bool = False, stamps: torch.Tensor | None = None) -> torch.Tensor:
        """``reduce_scatter_rows(x @ w^T) + bias + resid`` as one kernel.

        ``x`` [M, K] holds this rank's partial-sum input for all M rows (the
        row-parallel layer's local K slice); ``w`` is [N, K] (or [K, N] with
        ``w_mn``).  Returns this rank's [M / W, N] rows of the sum over ranks,
        with ``bias`` [N] and ``resid`` [M / W, N] added once.  The GEMM's
        epilogue stores each finished tile into its owner's memory, so the
        transfer overlaps the remaining MMAs (replaces the reference's
        forward all-reduce in ``tensor_parallel.py:74-91`` with the
        sequence-parallel reduce-scatter).  On one rank the plain GEMM runs
        unless ``force_kernel`` (profiling the fused kernel on one GPU).
        ``stamps`` (int64 [4], zeroed) receives ``%globaltimer`` phase times:
        kernel start, last CTA's tiles done, last CTA saw every rank's tiles,
        last CTA finished its reduction.
        """
        from .ops import kernels as K

        W = self.world_size
        M = x.shape[0]
        N = w.shape[1] if w_mn else w.shape[0]
        if M % W:
            raise ValueError(f"rows {M} not divisible by world_size {W}")
        if W == 1 and not force_kernel:
            return K.gemm(x, w, b_mn=w_mn, bias=bias, resid=resid)
        self._ensure_staging(2 * M * N * 2)
        out = torch.empty(M // W, N, dtype=torch.bfloat16, device=x.device)
        ev = self._record("gemm_reduce_scatter", "fused", M * N * 2)
        try:
            self.impl.gemm_rs(x.contiguous(), w, out, w_mn, bias, resid, K.status_word(x.device), stamps)
        finally:
            self._finish(ev)
        return out

    def all_gather_gemm(self, x_shard: torch.Tensor, w: torch.Tensor, *, w_mn: bool = False,
                        bias: torch.Tensor | None = None, gelu_out_aux: torch.Tensor | None = None,
                        gelu_grad_aux: torch.Tensor | None = None, resid: torch.Tensor | None = None,
                        gathered: torch.Tensor | None = None,
                        force_kernel: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
        """``epi(all_gather_rows(x_shard) @ w^T)`` as one kernel; returns (out, gathered).

        ``x_shard`` [M / W, K] is this rank's rows.  Two warps inside every
        CTA of the GEMM push this rank's shard into every peer's staging
        (each row crosses NVLink once) while the tiles of the local shard
        compute; a peer's tiles start as soon as that peer's pushes have all
        arrived.  The gathered [M, K] input is copied into ``gathered`` for
        reuse (the weight gradient needs it).  With ``gelu_out_aux`` the epilogue is
        ``out = gelu(acc + bias)``, ``aux = acc + bias``; with
        ``gelu_grad_aux`` it is ``out = acc * gelu'(aux)`` (an MLP backward).
        """
        from .ops import kernels as K

        W = self.world_size
        rows, Kd = x_shard.shape
        N = w.shape[1] if w_mn else w.shape[0]
        if W == 1 and not force_kernel:
            out = K.gemm(x_shard, w, b_mn=w_mn, bias=bias, gelu_out_aux=gelu_out_aux, gelu_grad_aux=gelu_grad_aux,
                         resid=resid)
            return out, x_shard
        if gathered is None:
            gathered = torch.empty(rows * W, Kd, dtype=torch.bfloat16, device=x_shard.device)
        self._ensure_staging(2 * W * rows * Kd * 2)
        out = torch.empty(rows * W, N, dtype=torch.bfloat16, device=x_shard.device)
        if gelu_out_aux is not None and gelu_grad_aux is not None:
            raise ValueError("gelu_out_aux and gelu_grad_aux are exclusive")
        epi, aux = (2, gelu_out_aux) if gelu_out_aux is not None else ((8, gelu_grad_aux) if gelu_grad_aux is not None
                                                                      else (0, None))
        ev = self._record("all_gather_gemm", "fused", rows * Kd * 2)
        try:
            self.impl.ag_gemm(x_shard.contiguous(), w, out, gathered, w_mn, bias, aux, resid, epi,
                              K.status_word(x_shard.device))
        finally:
            self._finish(ev)
        return out, gathered

    def gather_weight_gemm(self, x: torch.Tensor, shard: torch.Tensor, flat: torch.Tensor, w_off: int, n_rows: int,
                           bias: torch.Tensor | None = None) -> torch.Tensor:
        """FSDP's first GEMM fused with the all-gather of its parameters, as one kernel.

        ``shard`` is this rank's shard (a :meth:`symmetric_zeros` tensor) of a
        flattened parameter buffer of ``world * shard.numel()`` elements;
        ``flat`` (local, that many elements) receives the whole gathered
        buffer.  Returns ``x @ W^T (+ bias)`` for the ``[n_rows, K]`` weight at
        element offset ``w_off`` of the buffer.  Inside the kernel two warps
        per CTA copy the buffer in from every rank's shard -- this weight's
        chunks first -- and each output tile starts as soon as the chunks
        holding its weight rows have arrived, so the gather runs under the
        MMAs (the reference materialises the buffer with ``torch.cat`` before
        the unit runs: mini_nccl/fsdp.py:113-127).
        """
        from .ops import kernels as K

        x2 = x.reshape(-1, x.shape[-1])
        out = torch.empty(x2.shape[0], n_rows, dtype=torch.bfloat16, device=x.device)
        ev = self._record("gather_weight_gemm", "fused", shard.numel() * shard.element_size() * self.world_size)
        try:
            self.impl.gemm_agw(x2.contiguous(), shard, flat, int(w_off), int(n_rows), bias, out,
                               K.status_word(x.device))
        finally:
            self._finish(ev)
        return out

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
        """Free the communicator's memory (collective when NVLS objects exist).

        A rank that unbinds its memory from a multicast object while a peer's
        kernel still reads through the switch faults that peer, so with NVLS
        every rank first finishes its work and the ranks meet on the host."""
        if not self._closed:
            self._closed = True
            if self._nvls_objects:
                torch.cuda.synchronize(self.device)
                try:
                    self._agree(True)
                except Exception:  # the host communicator is gone: release anyway
                    pass
            self.impl.close()


def auto_all_reduce_algorithm(nbytes: int, world: int, nvls_ok: bool, in_multicast_memory: bool) -> str:
    """What ``all_reduce(algorithm="auto")`` runs for a message of ``nbytes``.

    The switch (``nvls``) for a sum it can do on a tensor already bound to the
    multicast object, or from :data:`NVLS_MIN_BYTES` on at
    :data:`NVLS_MIN_WORLD` ranks or more; otherwise one round of peer stores
    up to :data:`ONE_SHOT_MAX_BYTES` and the two-shot kernel above it.
    """
    if nvls_ok and (in_multicast_memory or (world >= NVLS_MIN_WORLD and nbytes >= NVLS_MIN_BYTES)):
        return "nvls"
    return "one_shot" if nbytes <= ONE_SHOT_MAX_BYTES else "two_shot"


def _pick(algorithm: str, eligible: bool, preferred: bool, op: str) -> bool:
    """Whether a collective goes through the switch: ``auto`` when it can and
    the size favours it; ``nvls`` / ``direct`` force one path."""
    if algorithm == "auto":
        return eligible and preferred
    if algorithm == "direct":
        return False
    if algorithm == "nvls":
        if not eligible:
            raise ValueError(f"{op}: the NVLS path needs NVLS, a 16-byte-multiple message (and for reductions "
                             f"op='sum' on fp32 / bf16 / fp16)")
        return True
    raise ValueError(f"unknown {op} algorithm {algorithm!r}; expected auto, nvls or direct")


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


# ====================================================================================
# Host-staged path: GPU tensors between ranks that share no peer memory
# ====================================================================================
#
# The entry points the reference offers for device tensors (mini_nccl/device.py:
# 57-320: is_accelerated, Staging, all_reduce_staged, all_reduce_pipelined,
# device_report).  On one NVSwitch box the peer-memory kernels above replace
# them; across hosts (MINI_NCCL_HOSTS naming several machines) a GPU tensor
# still has to cross a socket, and these functions move it through pinned host
# memory with the copies overlapped against the wire.

#: Bytes per staged chunk.
DEFAULT_CHUNK_BYTES = 4 << 20


def is_accelerated(tensor: torch.Tensor) -> bool:
    """True for tensors on a CUDA device."""
    return tensor.device.type == "cuda"


class _Window:
    """One pinned host window: an outbound and an inbound buffer and their events."""

    __slots__ = ("out", "inp", "down", "up", "uploading")

    def __init__(self, numel: int, dtype: torch.dtype, pinned: bool) -> None:
        self.out = torch.empty(numel, dtype=dtype, pin_memory=pinned)
        self.inp = torch.empty(numel, dtype=dtype, pin_memory=pinned)
        self.down = torch.cuda.Event() if pinned else None
        self.up = torch.cuda.Event() if pinned else None
        self.uploading = False


class Staging:
    """Pinned host windows plus a copy stream, reused by every step of a collective.

    A payload of ``numel`` elements is cut into ``n_chunks`` chunks of at most
    ``chunk_bytes``; ``n_slots`` windows let the download of chunk k+1 run on
    the copy engine while chunk k is on the wire.  On CPU tensors the windows
    are ordinary memory and every copy is synchronous, so the same chunking
    logic runs (and is tested) without a GPU.
    """

    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device,
                 chunk_bytes: int = DEFAULT_CHUNK_BYTES, n_slots: int = 2) -> None:
        self.device = torch.device(device)
        self.accelerated = self.device.type == "cuda"
        itemsize = torch.empty(0, dtype=dtype).element_size()
        self.chunk_numel = max(1, min(max(1, numel), chunk_bytes // itemsize))
        self.n_chunks = max(1, -(-numel // self.chunk_numel))
        self.stream = torch.cuda.Stream(self.device) if self.accelerated else None
        self.slots = [_Window(self.chunk_numel, dtype, self.accelerated)
                      for _ in range(max(1, min(n_slots, self.n_chunks)))]
        #: How many times the copy stream was ordered behind the compute stream
        #: (one per exchange; tests read it to check the dependency is expressed).
        self.orderings = 0

    def ranges(self, numel: int) -> list[tuple[int, int]]:
        return [(lo, min(numel, lo + self.chunk_numel)) for lo in range(0, numel, self.chunk_numel)]

    def order_after_compute(self) -> None:
        """Copy stream waits for everything already queued on the compute stream.

        Each exchange reads a block that the compute stream produced (the
        caller's data or the previous ring step's reduction); without this
        wait the download can read it before the reduction lands.
        """
        self.orderings += 1
        if self.accelerated:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))

    def download(self, w: _Window, src: torch.Tensor) -> None:
        dst = w.out[: src.numel()]
        if not self.accelerated:
            dst.copy_(src)
            return
        with torch.cuda.stream(self.stream):
            dst.copy_(src, non_blocking=True)
        w.down.record(self.stream)

    def wait_download(self, w: _Window) -> None:
        if self.accelerated:
            w.down.synchronize()

    def upload(self, w: _Window, dst: torch.Tensor) -> None:
        src = w.inp[: dst.numel()]
        if not self.accelerated:
            dst.copy_(src)
            return
        with torch.cuda.stream(self.stream):
            dst.copy_(src, non_blocking=True)
        w.up.record(self.stream)
        w.uploading = True

    def wait_upload(self, w: _Window) -> None:
        if self.accelerated and w.uploading:
            w.up.synchronize()
            w.uploading = False

    def order_compute_after_uploads(self) -> None:
        """Compute stream waits for the uploads in flight (the CPU does not block)."""
        if self.accelerated:
            cur = torch.cuda.current_stream(self.device)
            for w in self.slots:
                if w.uploading:
                    cur.wait_event(w.up)


def staged_exchange(pg, send: torch.Tensor, recv: torch.Tensor, dst: int, src: int, staging: Staging) -> None:
    """Send ``send`` to ``dst`` while receiving ``recv`` from ``src``, chunk by chunk.

    Downloads run ``len(staging.slots) - 1`` chunks ahead of the wire, so the
    copy engine and the socket work at the same time.  Chunk k uses window
    ``k % n_slots``; a window's inbound half is reused only after its upload
    finished.
    """
    spans = staging.ranges(send.numel())
    wins = staging.slots
    depth = len(wins)
    staging.order_after_compute()
    for k in range(min(depth, len(spans))):
        lo, hi = spans[k]
        staging.download(wins[k], send[lo:hi])
    for k, (lo, hi) in enumerate(spans):
        w = wins[k % depth]
        staging.wait_download(w)
        staging.wait_upload(w)
        n = hi - lo
        # send_recv returns once w.out is on the wire and w.inp is full, so
        # w.out can take the next download right after it.
        pg.send_recv(w.out[:n], dst, w.inp[:n], src)
        staging.upload(w, recv[lo:hi])
        nxt = k + depth
        if nxt < len(spans):
            nlo, nhi = spans[nxt]
            staging.download(w, send[nlo:nhi])
    staging.order_compute_after_uploads()


_PINNED: dict[tuple, torch.Tensor] = {}


def _pinned(numel: int, dtype: torch.dtype) -> torch.Tensor:
    """A cached pinned host buffer (page-locking is slow; reuse it across calls)."""
    key = (numel, dtype)
    buf = _PINNED.get(key)
    if buf is None:
        if len(_PINNED) > 8:
            _PINNED.clear()
        buf = _PINNED[key] = torch.empty(numel, dtype=dtype, pin_memory=True)
    return buf


def all_reduce_staged(pg, tensor: torch.Tensor, op: str = "sum", algorithm: str = "auto",
                      wire_dtype: torch.dtype | None = None) -> torch.Tensor:
    """All-reduce a GPU tensor through pinned host memory and the host collectives.

    The whole tensor goes down, the CPU algorithm (``algorithm``, channels,
    narrow wire) runs on the host copy, and the result goes back up.  CPU
    tensors go straight to the host collectives.
    """
    if not is_accelerated(tensor):
        return _hostc.all_reduce(pg, tensor, op=op, algorithm=algorithm, wire_dtype=wire_dtype)
    if not tensor.is_contiguous():
        raise ValueError("all_reduce_staged requires a contiguous tensor")
    flat = tensor.view(-1)
    host = _pinned(flat.numel(), flat.dtype)
    host.copy_(flat, non_blocking=True)
    torch.cuda.current_stream(tensor.device).synchronize()
    _hostc.all_reduce(pg, host, op=op, algorithm=algorithm, wire_dtype=wire_dtype)
    flat.copy_(host, non_blocking=True)
    torch.cuda.current_stream(tensor.device).synchronize()  # the host buffer is reused by the next call
    return tensor


def all_reduce_pipelined(pg, tensor: torch.Tensor, op: str = "sum",
                         chunk_bytes: int = DEFAULT_CHUNK_BYTES) -> torch.Tensor:
    """Ring all-reduce whose arithmetic stays on the device; only transfers are staged.

    2(W-1) ring steps; each moves one block through :func:`staged_exchange`
    and (in the reduce-scatter half) folds the received block into ours on
    the tensor's own device.
    """
    _hostc._check_op(op)
    if not tensor.is_contiguous():
        raise ValueError("all_reduce_pipelined requires a contiguous tensor")
    W, r = pg.world_size, pg.rank
    if W == 1:
        return tensor
    flat = tensor.view(-1)
    padded, blocks = _hostc._padded_blocks(flat, W)
    chunk = blocks.shape[1]
    staging = Staging(chunk, flat.dtype, flat.device, chunk_bytes=chunk_bytes)
    inbox = torch.empty(chunk, dtype=flat.dtype, device=flat.device)
    fold = _hostc._OPS[op]
    right, left = (r + 1) % W, (r - 1) % W
    rec = getattr(pg, "recorder", None)
    ev = rec.start("all_reduce_pipelined", "ring", channel=-1, nbytes=flat.numel() * flat.element_size(),
                   op=op, chunks=staging.n_chunks) if rec is not None else None
    try:
        for s in range(W - 1):  # reduce-scatter: block (r-s-1) accumulates
            staged_exchange(pg, blocks[(r - s) % W], inbox, right, left, staging)
            fold(blocks[(r - s - 1) % W], inbox)
        for s in range(W - 1):  # all-gather: finished blocks travel around
            staged_exchange(pg, blocks[(r + 1 - s) % W], blocks[(r - s) % W], right, left, staging)
        if padded.data_ptr() != flat.data_ptr():
            flat.copy_(padded[: flat.numel()])
        if staging.accelerated:
            torch.cuda.current_stream(flat.device).synchronize()
    finally:
        if rec is not None:
            rec.finish(ev)
    return tensor


def device_report() -> dict[str, object]:
    """What this machine can run: torch/CUDA versions, devices, peer access, our extension."""
    rep: dict[str, object] = {"torch": torch.__version__, "cuda_built": torch.version.cuda,
                              "cuda_available": torch.cuda.is_available()}
    try:
        from ._build import cuda_lib_path

        rep["extension_built"] = cuda_lib_path().exists()
    except Exception:  # noqa: BLE001 - a report never raises
        rep["extension_built"] = False
    if not torch.cuda.is_available():
        return rep
    n = torch.cuda.device_count()
    props = torch.cuda.get_device_properties(0)
    rep.update(device_name=props.name, device_count=n, compute_capability=f"{props.major}.{props.minor}",
               sm_count=props.multi_processor_count, total_memory_gib=round(props.total_memory / 2**30, 2),
               sm100a=(props.major, props.minor) == (10, 0))
    rep["peer_access"] = [[i == j or torch.cuda.can_device_access_peer(i, j) for j in range(n)] for i in range(n)]
    return rep
