"""The cross-stream waits that keep the GPU strategies race-free, asserted as a mechanism.

The bug class is a kernel on a side stream reading a buffer before the
compute stream has finished writing it (the reference shipped one in its
staging path and fixed it with an explicit stream wait).  Timing cannot show
such a race reliably, so these tests count the waits themselves: every
``wait_event`` / ``wait_stream`` call is recorded through a spy on
``torch.cuda.Stream`` while one training step runs on two GPUs, and the
tests demand

* DDP: one wait of the communication stream per gradient bucket, on an event
  recorded on the compute stream when that bucket's last gradient was
  written, and ``sync()`` making the compute stream wait for the last
  bucket's all-reduce;
* FSDP (prefetch on, activations kept): the side stream waits for the
  compute stream before every prefetched gather, the compute stream waits for
  every prefetched gather before using it, and the communication stream waits
  for the compute stream before every gradient reduce-scatter.

``tests/mutation_check.py`` removes each of these waits in turn and these
tests must fail.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F
from torch import nn

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

from mini_nccl_b200.launcher import run  # noqa: E402

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs at least 2 GPUs")


class Spy:
    """Record every Stream.wait_event / wait_stream call (stream, argument), and the
    stream each event was recorded on, so a wait can be traced to its producer."""

    def __init__(self) -> None:
        self.calls: list[tuple[str, int, object]] = []
        self.recorded_on: dict[int, int] = {}
        self._orig = (torch.cuda.Stream.wait_event, torch.cuda.Stream.wait_stream, torch.cuda.Event.record)

    def __enter__(self):
        spy = self
        orig_event, orig_stream, orig_record = self._orig

        def wait_event(stream, event):
            spy.calls.append(("event", stream.cuda_stream, event))
            return orig_event(stream, event)

        def wait_stream(stream, other):
            spy.calls.append(("stream", stream.cuda_stream, other.cuda_stream))
            return orig_stream(stream, other)

        def record(event, stream=None):
            s = stream if stream is not None else torch.cuda.current_stream()
            spy.recorded_on[id(event)] = s.cuda_stream
            return orig_record(event, stream)

        torch.cuda.Stream.wait_event = wait_event
        torch.cuda.Stream.wait_stream = wait_stream
        torch.cuda.Event.record = record
        return self

    def __exit__(self, *exc):
        torch.cuda.Stream.wait_event, torch.cuda.Stream.wait_stream, torch.cuda.Event.record = self._orig

    def waits_on_events_from(self, stream, producer) -> int:
        """How often ``stream`` waited on an event recorded on ``producer``."""
        return sum(1 for kind, s, ev in self.calls if kind == "event" and s == stream.cuda_stream
                   and self.recorded_on.get(id(ev)) == producer.cuda_stream)

    def on(self, kind: str, stream) -> list:
        return [c for c in self.calls if c[0] == kind and c[1] == stream.cuda_stream]


def _mlp(width: int = 256, depth: int = 6) -> nn.Module:
    torch.manual_seed(3)
    layers: list[nn.Module] = []
    for _ in range(depth):
        layers += [nn.Linear(width, width), nn.GELU()]
    return nn.Sequential(*layers)


def _ddp_waits(pg) -> dict:
    from mini_nccl_b200.ddp import DistributedDataParallel

    dev = torch.device("cuda", torch.cuda.current_device())
    ddp = DistributedDataParallel(_mlp().to(dev), pg, bucket_cap_mb=0.3)
    x = torch.randn(64, 256, device=dev)
    ddp.zero_grad()
    F.mse_loss(ddp(x), x).backward()
    ddp.sync()  # first step outside the spy: streams and buffers exist now
    compute = torch.cuda.current_stream(dev)
    with Spy() as spy:
        ddp.zero_grad()
        F.mse_loss(ddp(x), x).backward()
        ddp.sync()
    torch.cuda.synchronize(dev)
    # the comm stream also waits on the device communicator's own issue-order
    # events (recorded on itself); the waits that matter are on compute events
    return {"buckets": len(ddp._buckets),
            "comm_waits": spy.waits_on_events_from(ddp._comm_stream, compute),
            "compute_waits": len(spy.on("event", compute)),
            "last_done_awaited": spy.waits_on_events_from(compute, ddp._comm_stream) >= 1}


@needs2
def test_ddp_comm_stream_waits_for_every_bucket():
    for rep in run(_ddp_waits, 2, devices="cuda", timeout=300.0, op_timeout=60.0):
        assert rep["buckets"] > 1, rep
        assert rep["comm_waits"] == rep["buckets"], rep  # one compute-stream producer event per bucket
        assert rep["compute_waits"] >= 1 and rep["last_done_awaited"], rep  # sync() joins the comm stream


class Unit(nn.Module):
    def __init__(self, width: int = 256) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(width)
        self.fc = nn.Linear(width, width)

    def forward(self, x):
        return x + self.fc(self.norm(x))


class Stack(nn.Module):
    def __init__(self, n: int = 4) -> None:
        super().__init__()
        self.units = nn.ModuleList(Unit() for _ in range(n))
        self.head = nn.Linear(256, 1)

    def forward(self, x):
        for u in self.units:
            x = u(x)
        return self.head(x)


def _fsdp_waits(pg) -> dict:
    from mini_nccl_b200.fsdp import FullyShardedDataParallel

    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(4)
    fsdp = FullyShardedDataParallel(Stack().to(dev), pg, unit_cls=Unit, prefetch=True, recompute=False)
    x = torch.randn(32, 256, device=dev)

    def step():
        fsdp.zero_grad()
        fsdp(x).square().mean().backward()
        fsdp.sync()

    step()
    compute = torch.cuda.current_stream(dev)
    with Spy() as spy:
        step()
    torch.cuda.synchronize(dev)
    side, comm = fsdp._side, fsdp._comm_stream
    return {
        "units": len(fsdp.units),
        "side_waits_compute": sum(1 for c in spy.on("stream", side) if c[2] == compute.cuda_stream),
        "compute_waits_prefetch": len(spy.on("event", compute)),
        "comm_waits_compute": sum(1 for c in spy.on("stream", comm) if c[2] == compute.cuda_stream),
        "compute_joins_comm": sum(1 for c in spy.on("stream", compute) if c[2] == comm.cuda_stream),
    }


@needs2
def test_fsdp_side_and_comm_streams_wait_for_their_producers():
    for rep in run(_fsdp_waits, 2, devices="cuda", timeout=300.0, op_timeout=60.0):
        n = rep["units"]
        # forward prefetches units 1..n-1, backward re-gathers units n-2..0 ahead of use
        assert rep["side_waits_compute"] >= 2 * (n - 1), rep
        assert rep["compute_waits_prefetch"] >= 2 * (n - 1), rep
        assert rep["comm_waits_compute"] == n, rep  # one per unit's gradient reduce-scatter
        assert rep["compute_joins_comm"] >= 1, rep  # sync() joins the comm stream back
