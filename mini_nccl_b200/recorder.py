"""Flight recorder: a bounded, per-rank log of every collective.

Behaviour follows the reference recorder (mini_nccl/recorder.py:1-245):

* every collective is stamped with a monotonically increasing sequence number
  *per channel* (channel -1 is the collective issue order, -2 the pipeline
  schedule), so two ranks can be aligned by sequence number even after their
  logs have wrapped;
* the log is a fixed-capacity ring (``MINI_NCCL_TRACE_CAPACITY``, default
  32768) that counts what it dropped;
* recording is off unless ``MINI_NCCL_TRACE=1`` or ``trace=True``; a disabled
  recorder's ``start`` returns ``None`` and costs one attribute test;
* ``dump`` writes ``rank<N>.json`` for :mod:`mini_nccl_b200.diagnose`, and
  ``chrome_trace_events`` emits Trace Event Format for Perfetto.

What is new for the GPU path: a device collective writes its kernel-level
sequence number and ``%globaltimer`` start/end stamps into a small host-mapped
ring owned by the device communicator.  :meth:`attach_device_log` registers a
reader for that ring; its records are merged into ``state()`` under
``device_events`` so ``diagnose`` can compare what each GPU actually executed
with what each host issued.
"""

from __future__ import annotations

import json
import os
import threading
import time
from collections import deque
from collections.abc import Callable
from dataclasses import dataclass, field
from pathlib import Path

DEFAULT_CAPACITY = int(os.environ.get("MINI_NCCL_TRACE_CAPACITY", "32768"))

_TRUTHY = {"1", "true", "yes", "on"}


def trace_enabled_by_env() -> bool:
    return os.environ.get("MINI_NCCL_TRACE", "").strip().lower() in _TRUTHY


@dataclass
class Event:
    """One recorded operation.  ``end_ns`` stays ``None`` while it is in flight."""

    op: str
    algorithm: str
    channel: int
    seq: int
    nbytes: int
    start_ns: int
    end_ns: int | None = None
    detail: dict = field(default_factory=dict)

    @property
    def duration_us(self) -> float:
        stop = time.perf_counter_ns() if self.end_ns is None else self.end_ns
        return (stop - self.start_ns) / 1e3

    def describe(self) -> str:
        status = "PENDING" if self.end_ns is None else "completed"
        return (
            f"{self.op}[{self.algorithm}] seq={self.seq} channel={self.channel} "
            f"bytes={self.nbytes} {status} after {self.duration_us / 1e3:.1f}ms"
        )


class Recorder:
    """Thread-safe bounded event log for one rank."""

    def __init__(
        self,
        rank: int,
        world_size: int,
        enabled: bool = False,
        capacity: int = DEFAULT_CAPACITY,
    ) -> None:
        self.rank = rank
        self.world_size = world_size
        self.enabled = enabled
        self.capacity = capacity
        self._events: deque[Event] = deque(maxlen=capacity)
        self._dropped = 0
        self._seq: dict[int, int] = {}
        self._lock = threading.Lock()
        self._t0_ns = time.perf_counter_ns()
        self._t0_wall = time.time()
        self._device_logs: list[Callable[[], list[dict]]] = []

    # ---- sequence numbers ---------------------------------------------------

    def next_seq(self, channel: int) -> int:
        with self._lock:
            value = self._seq.get(channel, 0)
            self._seq[channel] = value + 1
        return value

    def peek_seq(self, channel: int) -> int:
        with self._lock:
            return self._seq.get(channel, 0)

    # ---- recording ----------------------------------------------------------

    def start(
        self,
        name: str,
        algorithm: str = "",
        channel: int = 0,
        nbytes: int = 0,
        **detail,
    ) -> Event | None:
        """Open an event (``None`` when disabled).

        ``name`` is the operation; keyword extras become trace annotations
        (``op="sum"`` is a legitimate annotation, hence not ``op=`` here).
        """
        if not self.enabled:
            return None
        ev = Event(
            op=name,
            algorithm=algorithm,
            channel=channel,
            seq=self.next_seq(channel),
            nbytes=nbytes,
            start_ns=time.perf_counter_ns(),
            detail=detail,
        )
        with self._lock:
            if self._events.maxlen is not None and len(self._events) >= self._events.maxlen:
                self._dropped += 1
            self._events.append(ev)
        return ev

    def finish(self, ev: Event | None) -> None:
        if ev is not None:
            ev.end_ns = time.perf_counter_ns()

    def attach_device_log(self, reader: Callable[[], list[dict]]) -> None:
        """Register a callable returning kernel-level records for ``state()``."""
        self._device_logs.append(reader)

    # ---- queries --------------------------------------------------------------

    def pending(self) -> list[Event]:
        with self._lock:
            return [ev for ev in self._events if ev.end_ns is None]

    def last_completed(self) -> Event | None:
        with self._lock:
            for ev in reversed(self._events):
                if ev.end_ns is not None:
                    return ev
        return None

    def context(self) -> str:
        """One line of local state, embedded in timeout errors."""
        if not self.enabled:
            return "flight recorder disabled (set MINI_NCCL_TRACE=1 for details)"
        pending = self.pending()
        last = self.last_completed()
        with self._lock:
            seqs = dict(sorted(self._seq.items()))
        inflight = "; ".join(ev.describe() for ev in pending) if pending else "nothing"
        done = last.describe() if last is not None else "none"
        return (
            f"rank {self.rank} | in flight: {inflight} | last completed: {done} | "
            f"next seq per channel: {seqs}"
        )

    # ---- output -----------------------------------------------------------------

    def _as_dict(self, ev: Event) -> dict:
        rel_us = (ev.start_ns - self._t0_ns) / 1e3
        return {
            "op": ev.op,
            "algorithm": ev.algorithm,
            "channel": ev.channel,
            "seq": ev.seq,
            "nbytes": ev.nbytes,
            "start_us": rel_us,
            "dur_us": None if ev.end_ns is None else ev.duration_us,
            "wall_start": self._t0_wall + rel_us / 1e6,
            "detail": ev.detail,
        }

    def device_events(self) -> list[dict]:
        out: list[dict] = []
        for reader in self._device_logs:
            try:
                out.extend(reader())
            except Exception as exc:  # a diagnostic must never mask the real error
                out.append({"error": f"device log unreadable: {exc}"})
        return out

    def state(self) -> dict:
        with self._lock:
            events = list(self._events)
            seqs = dict(self._seq)
            dropped = self._dropped
        return {
            "rank": self.rank,
            "world_size": self.world_size,
            "wall_start": self._t0_wall,
            "capacity": self.capacity,
            "dropped": dropped,
            "next_seq": seqs,
            "pending": [self._as_dict(ev) for ev in events if ev.end_ns is None],
            "events": [self._as_dict(ev) for ev in events],
            "device_events": self.device_events(),
        }

    def dump(self, directory: str | Path) -> Path:
        """Write ``<directory>/rank<N>.json``."""
        path = Path(directory)
        path.mkdir(parents=True, exist_ok=True)
        target = path / f"rank{self.rank}.json"
        target.write_text(json.dumps(self.state(), indent=1), encoding="utf-8")
        return target

    def chrome_trace_events(self, wall_zero: float | None = None) -> list[dict]:
        """Trace Event Format: pid = rank, tid = channel."""
        zero = self._t0_wall if wall_zero is None else wall_zero
        records: list[dict] = [
            {"name": "process_name", "ph": "M", "pid": self.rank, "args": {"name": f"rank {self.rank}"}}
        ]
        named: set[int] = set()
        with self._lock:
            events = list(self._events)
        for ev in events:
            if ev.channel not in named:
                named.add(ev.channel)
                label = "collective" if ev.channel < 0 else f"channel {ev.channel}"
                records.append(
                    {"name": "thread_name", "ph": "M", "pid": self.rank, "tid": ev.channel,
                     "args": {"name": label}}
                )
            wall = self._t0_wall + (ev.start_ns - self._t0_ns) / 1e9
            records.append(
                {
                    "name": f"{ev.op}:{ev.algorithm}" if ev.algorithm else ev.op,
                    "cat": "collective",
                    "ph": "X",
                    "ts": (wall - zero) * 1e6,
                    "dur": ev.duration_us,
                    "pid": self.rank,
                    "tid": ev.channel,
                    "args": {"seq": ev.seq, "bytes": ev.nbytes, **ev.detail},
                }
            )
        return records

    def dump_chrome_trace(self, path: str | Path) -> Path:
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        target.write_text(json.dumps(self.chrome_trace_events()), encoding="utf-8")
        return target
