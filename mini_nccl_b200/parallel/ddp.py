"""Data parallelism: bucketed, overlapped gradient averaging.

Semantics of the reference DDP (mini_nccl/ddp.py:113-247): rank 0's weights
are broadcast at construction; parameters are bucketed in *reverse*
registration order up to ``bucket_cap_mb`` (a dtype change starts a new
bucket); each ``param.grad`` is a view into its bucket's flat buffer so
autograd accumulates straight into the communication buffer; a
post-accumulate-grad hook marks readiness; buckets are always reduced in
index order so every rank issues the same collective sequence; ``no_sync()``
suppresses communication for gradient accumulation; ``sync()`` waits.

Two engines:

* **CUDA parameters.**  Bucket buffers are allocated in the group's
  *symmetric* device memory -- bound to an NVLS multicast object where the
  GPUs support it, so the switch sums the ranks' buckets in place
  (``multimem.ld_reduce`` / ``multimem.st``), else mapped by every peer, so
  the two-shot kernel stores into them over NVLink -- with no copy-in.  There is no communication thread: the
  hook that completes bucket ``i`` records a CUDA event on the compute stream,
  the communication stream waits on it and the fused all-reduce kernel (sum in
  fp32, ``1/W`` scale, bf16 or fp32 in and out) is launched there, while
  backward keeps running on the compute stream.  ``sync()`` only makes the
  compute stream wait on the communication stream; the host never blocks.
* **CPU parameters.**  A one-thread executor runs the host collectives while
  autograd continues, exactly as the reference does.

``optimizer_in_backward=dict(lr=..., betas=..., eps=..., weight_decay=...)``
(CUDA, world size > 1) moves the AdamW step into each bucket's reduction:
the parameters are re-homed into symmetric parameter buckets next to the
gradient buckets, and one kernel per bucket reduces this rank's 1/W slice of
the gradients, updates that slice (fp32 master weights and moments held for
the slice only: ZeRO-1) and writes the new parameters into every rank's
bucket.  The optimizer then runs during backward, on 1/W of the parameters
per rank, and its state shrinks W-fold; ``sync()`` leaves the parameters
updated, so no separate ``optimizer.step()`` is needed for bucketed
parameters.  Gradient clipping by global norm is not available in this mode
(each slice is updated as soon as its gradients are reduced).
"""

from __future__ import annotations

import os
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from contextlib import contextmanager

import torch
from torch import nn

from .. import collectives
from ..communicator import Communicator

#: CTAs a bucket all-reduce may use while backward runs beside it (0: the
#: device communicator's default).
DDP_COMM_BLOCKS = int(os.environ.get("MINI_NCCL_DDP_BLOCKS", "0"))
#: Bucket all-reduces run as small CTAs that share SMs with the backward
#: pass's persistent kernels instead of taking whole SMs from them.
DDP_BESIDE_COMPUTE = os.environ.get("MINI_NCCL_DDP_BESIDE", "1") != "0"
#: Buckets live in NVLS multicast memory where available (in-place switch reduction).
DDP_NVLS = os.environ.get("MINI_NCCL_DDP_NVLS", "1") != "0"


def average_gradients(pg: Communicator, params, algorithm: str = "ring") -> int:
    """Average ``params``' gradients over ``pg``; returns the bytes reduced.

    The explicit form of DDP's reduction, for pipelines (once after the
    schedule drains, not per microbatch) and for reducing along one mesh
    dimension only (mini_nccl/ddp.py:53-79).  CUDA gradients are reduced by
    one fused multi-tensor kernel per dtype: the kernel gathers the gradient
    pointers itself, so there is no flatten/unflatten copy, and the ``1/W``
    scale is applied in its epilogue.
    """
    if pg.world_size == 1:
        return 0
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return 0
    total = 0
    if grads[0].is_cuda and hasattr(pg, "device_comm"):
        dc = pg.device_comm()
        by_dtype: dict[torch.dtype, list[torch.Tensor]] = {}
        for g in grads:
            by_dtype.setdefault(g.dtype, []).append(g)
        for group in by_dtype.values():
            total += dc.all_reduce_multi(group, scale=1.0 / pg.world_size)
        return total
    flat = torch.cat([g.reshape(-1) for g in grads])
    collectives.all_reduce(pg, flat, algorithm=algorithm)
    flat.div_(pg.world_size)
    offset = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[offset : offset + n].view_as(g))
        offset += n
    return flat.numel() * flat.element_size()


class _Bucket:
    """A flat gradient buffer shared by a run of parameters."""

    def __init__(self, index: int, params: list[nn.Parameter], buffer: torch.Tensor) -> None:
        self.index = index
        self.params = params
        self.buffer = buffer
        self.views: list[torch.Tensor] = []
        offset = 0
        for p in params:
            n = p.numel()
            self.views.append(buffer[offset : offset + n].view(p.shape))
            offset += n
        self.pending = len(params)
        self.ready = threading.Event()
        self.lock = threading.Lock()
        self.launched = False

    def attach_grads(self) -> None:
        for p, v in zip(self.params, self.views, strict=True):
            p.grad = v

    def home_parameters(self, store: torch.Tensor, rank: int, world: int) -> None:
        """Move the parameters into ``store`` (views) and create this rank's slice of
        optimizer state: fp32 master weights, first and second moments."""
        self.param_buffer = store
        offset = 0
        with torch.no_grad():
            for p in self.params:
                n = p.numel()
                view = store[offset : offset + n].view(p.shape)
                view.copy_(p.data)
                p.data = view
                offset += n
        slice_n = store.numel() // world
        mine = store[rank * slice_n : (rank + 1) * slice_n]
        self.opt_state = {"master": mine.float().clone(), "m": torch.zeros(slice_n, device=store.device),
                          "v": torch.zeros(slice_n, device=store.device)}

    def mark_ready(self) -> bool:
        """Count one parameter in; True when the bucket just became complete."""
        with self.lock:
            self.pending -= 1
            done = self.pending == 0
        if done:
            self.ready.set()
        return done

    def reset(self) -> None:
        with self.lock:
            self.pending = len(self.params)
            self.ready.clear()
            self.launched = False

    @property
    def nbytes(self) -> int:
        return self.buffer.numel() * self.buffer.element_size()


class DistributedDataParallel(nn.Module):
    """Bucketed data parallelism over ``pg`` (see module docstring)."""

    def __init__(
        self,
        module: nn.Module,
        pg: Communicator,
        bucket_cap_mb: float = 1.0,
        overlap: bool = True,
        algorithm: str = "ring",
        broadcast_buffers: bool = True,
        optimizer_in_backward: dict | None = None,
    ) -> None:
        super().__init__()
        self.module = module
        self.pg = pg
        #: AdamW hyper-parameters of the fused optimizer (read at every step), or None.
        self.optimizer_hp = None
        self._opt_step = 0
        self.algorithm = algorithm
        self._overlap = overlap and pg.world_size > 1
        self._buckets: list[_Bucket] = []
        self._accumulating = False
        self._future: Future | None = None
        #: ``perf_counter_ns`` at which this iteration's first reduction was
        #: dispatched (None until then) -- lets tests check overlap mechanically.
        self.reduce_submitted_ns: int | None = None
        #: Per-step timeline (CUDA): when an int64 CUDA tensor is set here, each
        #: bucket's launch stamps ``%globaltimer`` into ``timeline[bucket.index]``
        #: on the compute stream (the moment its last gradient is written) and
        #: appends the device collective sequence number of its all-reduce to
        #: ``timeline_seqs``; the device event ring holds that all-reduce's
        #: start and end on the same clock (benchmarks/ddp_timeline.py).
        self.timeline: torch.Tensor | None = None
        self.timeline_seqs: list[int] = []
        params = [p for p in module.parameters()]
        self._cuda = bool(params) and params[0].is_cuda
        if optimizer_in_backward is not None:
            if not self._cuda or pg.world_size < 2:
                raise ValueError("optimizer_in_backward needs CUDA parameters and world_size > 1")
            hp = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
            hp.update(optimizer_in_backward)
            hp["betas"] = tuple(hp["betas"])
            self.optimizer_hp = hp

        if pg.world_size > 1:
            with torch.no_grad():
                for p in module.parameters():
                    collectives.broadcast(pg, p.data if p.data.is_contiguous() else p.data.contiguous(), src=0)
                if broadcast_buffers:
                    for b in module.buffers():
                        if b.is_contiguous():
                            collectives.broadcast(pg, b.data, src=0)
            self._build_buckets(bucket_cap_mb)
            for bucket in self._buckets:
                bucket.attach_grads()
                for p in bucket.params:
                    p.register_post_accumulate_grad_hook(self._make_hook(bucket))
            if self._cuda:
                self._dc = pg.device_comm()
                self._comm_stream = torch.cuda.Stream(device=params[0].device)
                self._next_launch = 0
                self._last_done: torch.cuda.Event | None = None
            else:
                self._comm = ThreadPoolExecutor(max_workers=1, thread_name_prefix="mnb-ddp")

    # ---- buckets --------------------------------------------------------------

    def _build_buckets(self, cap_mb: float) -> None:
        cap = int(cap_mb * 1024 * 1024)
        groups: list[list[nn.Parameter]] = []
        run: list[nn.Parameter] = []
        run_bytes = 0
        for p in reversed(list(self.module.parameters())):
            if not p.requires_grad:
                continue
            nb = p.numel() * p.element_size()
            if run and (run_bytes + nb > cap or p.dtype != run[0].dtype):
                groups.append(run)
                run, run_bytes = [], 0
            run.append(p)
            run_bytes += nb
        if run:
            groups.append(run)
        for i, ps in enumerate(groups):
            numel = sum(p.numel() for p in ps)
            if self._cuda:
                dc = self.pg.device_comm()
                if self.optimizer_hp is not None:  # W equal slices of whole 16-byte units
                    quantum = self.pg.world_size * (16 // ps[0].element_size())
                    numel = -(-numel // quantum) * quantum
                # NVLS memory when the GPUs have it: the bucket all-reduce then
                # runs in place through the switch
                buf = dc.symmetric_zeros(numel, ps[0].dtype, nvls=DDP_NVLS)
            else:
                buf = torch.zeros(numel, dtype=ps[0].dtype, device=ps[0].device)
            bucket = _Bucket(i, ps, buf)
            if self.optimizer_hp is not None:
                bucket.home_parameters(dc.symmetric_zeros(numel, ps[0].dtype, nvls=DDP_NVLS),
                                       self.pg.rank, self.pg.world_size)
            self._buckets.append(bucket)

    def _make_hook(self, bucket: _Bucket):
        def hook(_param: nn.Parameter) -> None:
            if self._accumulating:
                return  # inside no_sync(): keep summing into the buckets, no traffic
            complete = bucket.mark_ready()
            if not self._overlap:
                return
            if self._cuda:
                if complete:
                    self._launch_ready_prefix()
            elif self._future is None:
                self.reduce_submitted_ns = time.perf_counter_ns()
                self._future = self._comm.submit(self._reduce_all_host)

        return hook

    # ---- CUDA engine ------------------------------------------------------------

    def _launch(self, bucket: _Bucket) -> None:
        if self.reduce_submitted_ns is None:
            self.reduce_submitted_ns = time.perf_counter_ns()
        produced = torch.cuda.Event()
        if self.timeline is not None:
            from ..ops.kernels import ext

            ext().stamp(self.timeline, bucket.index)
            self.timeline_seqs.append(int(self._dc.impl.seq()))
        produced.record(torch.cuda.current_stream(bucket.buffer.device))
        ev = self.pg.recorder.start(
            f"ddp_bucket{bucket.index}", self.algorithm, channel=-1,
            nbytes=bucket.nbytes, params=len(bucket.params),
        )
        try:
            with torch.cuda.stream(self._comm_stream):
                self._comm_stream.wait_event(produced)
                if self.optimizer_hp is not None:
                    hp = self.optimizer_hp
                    self._dc.all_reduce_adamw(
                        bucket.buffer, bucket.param_buffer, bucket.opt_state, lr=hp["lr"], betas=hp["betas"],
                        eps=hp["eps"], weight_decay=hp["weight_decay"], step=self._opt_step + 1,
                        scale=1.0 / self.pg.world_size, blocks=DDP_COMM_BLOCKS or None,
                        beside_compute=DDP_BESIDE_COMPUTE)
                else:
                    self._dc.all_reduce(
                        bucket.buffer, op="sum", algorithm="auto", scale=1.0 / self.pg.world_size,
                        blocks=DDP_COMM_BLOCKS or None, beside_compute=DDP_BESIDE_COMPUTE,
                    )
                done = torch.cuda.Event()
                done.record(self._comm_stream)
                self._last_done = done
        finally:
            self.pg.recorder.finish(ev)
        bucket.launched = True

    def _launch_ready_prefix(self) -> None:
        """Launch, in index order, every bucket whose predecessors are launched."""
        while self._next_launch < len(self._buckets):
            b = self._buckets[self._next_launch]
            if not b.ready.is_set():
                return
            self._launch(b)
            self._next_launch += 1

    def _sync_cuda(self) -> None:
        while self._next_launch < len(self._buckets):
            self._launch(self._buckets[self._next_launch])  # unused params: reduce anyway
            self._next_launch += 1
        if self._last_done is not None:
            torch.cuda.current_stream(self._buckets[0].buffer.device).wait_event(self._last_done)
        self._next_launch = 0
        self._last_done = None

    # ---- host engine -------------------------------------------------------------

    def _reduce_all_host(self) -> None:
        for bucket in self._buckets:
            bucket.ready.wait()
            ev = self.pg.recorder.start(
                f"ddp_bucket{bucket.index}", self.algorithm, channel=-1,
                nbytes=bucket.nbytes, params=len(bucket.params),
            )
            try:
                collectives.all_reduce(self.pg, bucket.buffer, algorithm=self.algorithm)
                bucket.buffer.div_(self.pg.world_size)
            finally:
                self.pg.recorder.finish(ev)

    # ---- public ---------------------------------------------------------------------

    @contextmanager
    def no_sync(self):
        """Accumulate into the buckets without communicating (don't zero_grad inside)."""
        before = self._accumulating
        self._accumulating = True
        try:
            yield
        finally:
            self._accumulating = before

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def sync(self) -> None:
        """Finish gradient averaging; call after ``backward()``."""
        if self.pg.world_size == 1:
            return
        if self._cuda:
            if not self._overlap:
                for b in self._buckets:
                    b.ready.set()
            self._sync_cuda()
            if self.optimizer_hp is not None:
                self._opt_step += 1
        elif self._overlap:
            if self._future is not None:
                self._future.result()
                self._future = None
        else:
            for b in self._buckets:
                b.ready.set()
            self._reduce_all_host()
        for b in self._buckets:
            b.reset()
        self.reduce_submitted_ns = None

    def zero_grad(self, set_to_none: bool = False) -> None:
        """Zero the buckets in place (grads must stay views, so never ``None``)."""
        if self.pg.world_size == 1:
            # Nothing to bucket: dropping the grads lets autograd hand each
            # parameter its freshly computed gradient instead of a fill + add.
            self.module.zero_grad(set_to_none=True)
            return
        for b in self._buckets:
            b.buffer.zero_()
            b.attach_grads()

    def grad_buffers(self) -> list[torch.Tensor]:
        """The flat bucket buffers, in bucket order (for fused optimizers)."""
        return [b.buffer for b in self._buckets]

    def unbucketed_parameters(self) -> list[nn.Parameter]:
        """Parameters outside every bucket (frozen ones): what a separate optimizer
        still has to step when ``optimizer_in_backward`` is on."""
        bucketed = {id(p) for b in self._buckets for p in b.params}
        return [p for p in self.module.parameters() if id(p) not in bucketed and p.requires_grad]

    def optimizer_state_dict(self) -> dict:
        """This rank's slice of the fused optimizer's state (one file per rank)."""
        if self.optimizer_hp is None:
            raise ValueError("no fused optimizer (optimizer_in_backward is off)")
        return {"hp": dict(self.optimizer_hp), "step": self._opt_step, "rank": self.pg.rank,
                "world_size": self.pg.world_size,
                "buckets": [{k: t.detach().clone() for k, t in b.opt_state.items()} for b in self._buckets]}

    def load_optimizer_state_dict(self, sd: dict) -> None:
        if self.optimizer_hp is None:
            raise ValueError("no fused optimizer (optimizer_in_backward is off)")
        if sd["rank"] != self.pg.rank or sd["world_size"] != self.pg.world_size:
            raise ValueError("optimizer state was written by a different rank layout")
        self.optimizer_hp = dict(sd["hp"])
        self.optimizer_hp["betas"] = tuple(self.optimizer_hp["betas"])
        self._opt_step = int(sd["step"])
        with torch.no_grad():
            for b, st in zip(self._buckets, sd["buckets"], strict=True):
                for k, t in st.items():
                    b.opt_state[k].copy_(t)
