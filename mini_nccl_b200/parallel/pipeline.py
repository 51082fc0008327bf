"""Pipeline parallelism: GPipe and 1F1B schedules.

Semantics of the reference pipeline (mini_nccl/pipeline.py:61-323): a fixed
``activation_shape``/dtype for both sides of every boundary; forward and
backward events recorded on ``PIPELINE_CHANNEL = -2`` so stage-dependent
warm-up never looks like a desync; gradients are matched FIFO to the *oldest*
microbatch in flight; the last stage scales its loss by ``1/M``; every
argument is validated before any traffic; 1F1B warms up with ``W-1-s``
forwards, then alternates a forward with a backward using one fused
send-activation/receive-gradient exchange (no neighbour deadlock), then
drains.  ``in_flight_peak`` records the measured depth (``<= W - s``).

On CUDA the stage boundaries are NCCL point-to-point transfers issued on a
dedicated stream when the group has a NCCL group attached
(``init_process_group(nccl_p2p=True)``), so sends and receives overlap the
neighbour's compute; activation buffers are allocated on the stage's device.
"""

from __future__ import annotations

from collections import deque

import torch
from torch import nn

from ..communicator import Communicator
from ..utils import nvtx as _nvtx

SCHEDULES = ("1f1b", "gpipe")

#: Pipeline events get their own recorder channel (see module docstring).
PIPELINE_CHANNEL = -2


class PipelineParallel:
    """Drive one pipeline stage through a GPipe or 1F1B schedule."""

    def __init__(
        self,
        stage: nn.Module,
        pg: Communicator,
        activation_shape: tuple[int, ...],
        loss_fn=None,
        schedule: str = "1f1b",
        dtype: torch.dtype = torch.float32,
        device: torch.device | str | None = None,
    ) -> None:
        if schedule not in SCHEDULES:
            raise ValueError(f"unknown schedule {schedule!r}; expected one of {SCHEDULES}")
        if loss_fn is None and pg.rank == pg.world_size - 1:
            raise ValueError("the last stage needs loss_fn to start the backward pass")
        self.stage = stage
        self.pg = pg
        self.schedule = schedule
        self.activation_shape = tuple(activation_shape)
        self.loss_fn = loss_fn
        self.dtype = dtype
        if device is None:
            first = next(iter(stage.parameters()), None)
            device = first.device if first is not None else torch.device("cpu")
        self.device = torch.device(device)
        self._gpu = self.device.type == "cuda"
        self.rank = pg.rank
        self.n_stages = pg.world_size
        self.is_first = self.rank == 0
        self.is_last = self.rank == self.n_stages - 1
        self.prev, self.next = self.rank - 1, self.rank + 1
        numel = 1
        for d in self.activation_shape:
            numel *= d
        self._activation_bytes = numel * torch.empty(0, dtype=dtype).element_size()
        self._queue: deque[tuple[torch.Tensor | None, torch.Tensor]] = deque()
        self.in_flight_peak = 0

    # ---- boundary traffic -----------------------------------------------------------

    def _buffer(self) -> torch.Tensor:
        return torch.empty(self.activation_shape, dtype=self.dtype, device=self.device)

    def _recv_activation(self) -> torch.Tensor:
        buf = self._buffer()
        self.pg.recv(buf, self.prev)
        return buf.requires_grad_(True)  # its .grad is what the previous stage needs

    def _send_activation(self, act: torch.Tensor) -> None:
        self.pg.send(act.detach().to(self.dtype).contiguous(), self.next)

    def _recv_gradient(self) -> torch.Tensor:
        buf = self._buffer()
        self.pg.recv(buf, self.next)
        return buf

    def _send_gradient(self, grad: torch.Tensor) -> None:
        self.pg.send(grad.contiguous(), self.prev)

    def _send_activation_recv_gradient(self, act: torch.Tensor) -> torch.Tensor:
        """Push the newest activation while pulling the oldest gradient (one exchange)."""
        buf = self._buffer()
        self.pg.send_recv(act.detach().to(self.dtype).contiguous(), self.next, buf, self.next)
        return buf

    # ---- one microbatch ---------------------------------------------------------------

    def _forward(self, micro_input, micro_target, n_micro: int):
        ev = self.pg.recorder.start(
            "pp_forward", self.schedule, channel=PIPELINE_CHANNEL,
            nbytes=self._activation_bytes, stage=self.rank, depth=len(self._queue),
        )
        opened = _nvtx.push(_nvtx.label("pp_forward", self.schedule, self._activation_bytes)) if self._gpu else False
        try:
            x = None if self.is_first else self._recv_activation()
            out = self.stage(micro_input if self.is_first else x)
            if self.is_last:
                out = self.loss_fn(out, micro_target) / n_micro
            self._queue.append((x, out))
            self.in_flight_peak = max(self.in_flight_peak, len(self._queue))
            return out
        finally:
            self.pg.recorder.finish(ev)
            _nvtx.pop(opened)

    def _backward(self, grad: torch.Tensor | None) -> None:
        """Backward of the *oldest* queued microbatch (FIFO: the next stage lags)."""
        ev = self.pg.recorder.start(
            "pp_backward", self.schedule, channel=PIPELINE_CHANNEL,
            nbytes=self._activation_bytes, stage=self.rank, depth=len(self._queue),
        )
        opened = _nvtx.push(_nvtx.label("pp_backward", self.schedule, self._activation_bytes)) if self._gpu else False
        try:
            x, out = self._queue.popleft()
            if self.is_last:
                out.backward()
            else:
                out.backward(grad)
            if not self.is_first:
                assert x is not None and x.grad is not None
                self._send_gradient(x.grad)
        finally:
            self.pg.recorder.finish(ev)
            _nvtx.pop(opened)

    # ---- schedules ----------------------------------------------------------------------

    def step(
        self,
        inputs: torch.Tensor | None = None,
        targets: torch.Tensor | None = None,
        n_microbatches: int = 1,
    ) -> float:
        """One optimizer step's microbatches; grads accumulate.  Returns the loss
        (summed over microbatches) on the last stage, 0.0 elsewhere."""
        if n_microbatches < 1:
            raise ValueError("n_microbatches must be at least 1")
        if self.is_first and inputs is None:
            raise ValueError("the first stage needs inputs")
        if self.is_last and targets is None:
            raise ValueError("the last stage needs targets")
        for label, t in (("inputs", inputs), ("targets", targets)):
            if t is not None and t.shape[0] % n_microbatches:
                raise ValueError(
                    f"{label} batch of {t.shape[0]} is not divisible by n_microbatches={n_microbatches}"
                )
        m_in = list(torch.chunk(inputs, n_microbatches)) if (self.is_first and inputs is not None) else [None] * n_microbatches
        m_tg = list(torch.chunk(targets, n_microbatches)) if (self.is_last and targets is not None) else [None] * n_microbatches
        self._queue.clear()
        self.in_flight_peak = 0
        losses: list[torch.Tensor] = []

        if self.n_stages == 1:
            for i in range(n_microbatches):
                out = self._forward(m_in[i], m_tg[i], n_microbatches)
                losses.append(out.detach())
                self._backward(None)
        elif self.schedule == "gpipe":
            self._gpipe(m_in, m_tg, n_microbatches, losses)
        else:
            self._one_f_one_b(m_in, m_tg, n_microbatches, losses)
        if not losses:
            return 0.0
        return float(torch.stack([l.float() for l in losses]).sum())

    def _keep(self, out: torch.Tensor, losses: list[torch.Tensor]) -> None:
        if self.is_last:
            losses.append(out.detach())

    def _gpipe(self, m_in, m_tg, n: int, losses) -> None:
        for i in range(n):
            out = self._forward(m_in[i], m_tg[i], n)
            self._keep(out, losses)
            if not self.is_last:
                self._send_activation(out)
        for _ in range(n):
            self._backward(None if self.is_last else self._recv_gradient())

    def _one_f_one_b(self, m_in, m_tg, n: int, losses) -> None:
        warm = min(self.n_stages - 1 - self.rank, n)
        i = 0
        for _ in range(warm):
            out = self._forward(m_in[i], m_tg[i], n)
            self._keep(out, losses)
            if not self.is_last:
                self._send_activation(out)
            i += 1
        for _ in range(n - warm):
            out = self._forward(m_in[i], m_tg[i], n)
            self._keep(out, losses)
            i += 1
            if self.is_last:
                self._backward(None)
            else:
                self._backward(self._send_activation_recv_gradient(out))
        for _ in range(warm):
            self._backward(None if self.is_last else self._recv_gradient())
