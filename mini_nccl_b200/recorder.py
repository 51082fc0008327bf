"""Flight recorder: what each rank issued, kept in a bounded per-rank log.

The file format and the numbering rule are interfaces shared with the
reference (``mini_nccl/recorder.py:1-245``) so that its ``diagnose`` tooling
and tests apply unchanged: a ``rank<N>.json`` dump with ``events`` /
``pending`` / ``next_seq`` / ``dropped``, a Trace Event Format export with
pid = rank and tid = channel, and one sequence counter *per channel*
(channel -1 is the collective issue order, -2 the pipeline schedule).  The
machinery is this library's own:

* **Slot ring.**  Records go into a preallocated list of ``capacity`` slots
  at ``written % capacity``; nothing is ever shifted or reallocated, and the
  number of records the ring has overwritten is ``written - capacity``
  (derived, not counted).
* **Open-operation index.**  An operation stays in a dict keyed by its record
  number from ``start`` to ``finish``, so "what is in flight" is answered
  without scanning the ring, and an operation still in flight stays visible
  even after the ring has wrapped past its slot.
* **Device stream.**  A device communicator registers a reader of its
  host-mapped kernel event ring (kernel-level sequence numbers and
  ``%globaltimer`` stamps, written by the GPU).  Dumps carry those records
  as ``device_events``, and :meth:`Recorder.context` -- the line a timeout
  error embeds -- reports the last kernel each GPU finished next to what the
  host issued, which is what tells a stuck kernel from a host that never
  launched one.

Recording is off unless ``MINI_NCCL_TRACE=1`` or ``trace=True``; a disabled
recorder's ``start`` returns ``None`` after one attribute test.
"""

from __future__ import annotations

import json
import os
import threading
import time
from collections.abc import Callable
from pathlib import Path

DEFAULT_CAPACITY = int(os.environ.get("MINI_NCCL_TRACE_CAPACITY", "32768"))


def trace_enabled_by_env() -> bool:
    return os.environ.get("MINI_NCCL_TRACE", "").strip().lower() in ("1", "true", "yes", "on")


class Event:
    """One recorded operation; ``end_ns`` is ``None`` while it is in flight.

    Field names are part of the dump format.  ``start_ns`` / ``end_ns`` are
    ``time.perf_counter_ns`` readings.
    """

    __slots__ = ("op", "algorithm", "channel", "seq", "nbytes", "start_ns", "end_ns", "detail", "_rid")

    def __init__(self, op: str, algorithm: str, channel: int, seq: int, nbytes: int, start_ns: int,
                 end_ns: int | None = None, detail: dict | None = None) -> None:
        self.op = op
        self.algorithm = algorithm
        self.channel = channel
        self.seq = seq
        self.nbytes = nbytes
        self.start_ns = start_ns
        self.end_ns = end_ns
        self.detail = {} if detail is None else detail
        self._rid = -1

    @property
    def done(self) -> bool:
        return self.end_ns is not None

    @property
    def duration_us(self) -> float:
        until = self.end_ns if self.end_ns is not None else time.perf_counter_ns()
        return (until - self.start_ns) / 1e3

    def describe(self) -> str:
        what = f"{self.op}[{self.algorithm}]" if self.algorithm else self.op
        state = "done" if self.done else "IN FLIGHT"
        return (f"{what} #{self.seq} on channel {self.channel}, {self.nbytes} B, {state} "
                f"({self.duration_us / 1e3:.1f} ms)")

    def __repr__(self) -> str:
        return f"Event({self.describe()})"


class Recorder:
    """Bounded event log of one rank; safe to use from several threads."""

    def __init__(self, rank: int, world_size: int, enabled: bool = False,
                 capacity: int = DEFAULT_CAPACITY) -> None:
        self.rank = rank
        self.world_size = world_size
        self.enabled = enabled
        self._mutex = threading.Lock()
        self._slots: list[Event | None] = []
        self._written = 0
        self._open: dict[int, Event] = {}
        self._next_seq: dict[int, int] = {}
        self._device_readers: list[Callable[[], list[dict]]] = []
        # One instant read on both clocks: perf_counter stamps become wall time.
        self._perf_anchor = time.perf_counter_ns()
        self._wall_anchor = time.time()
        self.resize(capacity)

    # ---- configuration ---------------------------------------------------------

    @property
    def capacity(self) -> int:
        return len(self._slots)

    def resize(self, capacity: int) -> None:
        """Keep at most ``capacity`` records from now on (the newest survive)."""
        if capacity < 1:
            raise ValueError("capacity must be at least 1")
        with self._mutex:
            kept = self._ordered()[-capacity:]
            self._slots = [None] * capacity
            base = self._written - len(kept)
            for i, ev in enumerate(kept):
                self._slots[(base + i) % capacity] = ev

    def attach_device_log(self, reader: Callable[[], list[dict]]) -> None:
        """Register a callable that returns the GPU's kernel-level records."""
        self._device_readers.append(reader)

    # ---- numbering and recording ----------------------------------------------

    def _take_seq(self, channel: int) -> int:
        """Next sequence number of ``channel`` (caller holds the mutex)."""
        seq = self._next_seq.get(channel, 0)
        self._next_seq[channel] = seq + 1
        return seq

    def next_seq(self, channel: int) -> int:
        """Take the next sequence number of ``channel``."""
        with self._mutex:
            return self._take_seq(channel)

    def peek_seq(self, channel: int) -> int:
        with self._mutex:
            return self._next_seq.get(channel, 0)

    def start(self, name: str, algorithm: str = "", channel: int = 0, nbytes: int = 0, **detail) -> Event | None:
        """Open a record of operation ``name``; ``None`` when recording is off.

        Keyword extras are annotations (``op="sum"`` among them, which is why
        the operation itself is called ``name`` here).
        """
        if not self.enabled:
            return None
        now = time.perf_counter_ns()
        with self._mutex:
            ev = Event(name, algorithm, channel, self._take_seq(channel), nbytes, now, None, detail)
            ev._rid = self._written
            self._slots[self._written % len(self._slots)] = ev
            self._written += 1
            self._open[ev._rid] = ev
        return ev

    def finish(self, ev: Event | None) -> None:
        if ev is None:
            return
        ev.end_ns = time.perf_counter_ns()
        with self._mutex:
            self._open.pop(ev._rid, None)

    # ---- queries ------------------------------------------------------------------

    @property
    def dropped(self) -> int:
        """Records overwritten because the ring was full."""
        return max(0, self._written - len(self._slots))

    def _ordered(self) -> list[Event]:
        """Records still in the ring, oldest first (caller holds the mutex)."""
        n = len(self._slots)
        if n == 0:
            return []
        first = max(0, self._written - n)
        return [ev for i in range(first, self._written) if (ev := self._slots[i % n]) is not None]

    def events(self) -> list[Event]:
        with self._mutex:
            return self._ordered()

    def pending(self) -> list[Event]:
        """Operations started and not finished, in issue order."""
        with self._mutex:
            return [self._open[k] for k in sorted(self._open)]

    def last_completed(self) -> Event | None:
        with self._mutex:
            n = len(self._slots)
            for i in range(self._written - 1, max(-1, self._written - n - 1), -1):
                ev = self._slots[i % n]
                if ev is not None and ev.done:
                    return ev
        return None

    def device_events(self) -> list[dict]:
        records: list[dict] = []
        for reader in self._device_readers:
            try:
                records.extend(reader())
            except Exception as exc:  # diagnostics must not hide the error being reported
                records.append({"error": f"device log unreadable: {exc}"})
        return records

    def context(self) -> str:
        """The local state in one line, for timeout and desync errors."""
        if not self.enabled:
            return "flight recorder disabled (set MINI_NCCL_TRACE=1 for details)"
        open_ops = self.pending()
        last = self.last_completed()
        with self._mutex:
            counters = ", ".join(f"ch{c}:{n}" for c, n in sorted(self._next_seq.items()))
        pieces = [f"rank {self.rank}"]
        pieces.append(f"{len(open_ops)} in flight" + (": " + "; ".join(e.describe() for e in open_ops)
                                                     if open_ops else ""))
        pieces.append("last done: " + (last.describe() if last is not None else "none"))
        kernels = [d for d in self.device_events() if "seq" in d]
        if kernels:
            finished = [d for d in kernels if d.get("end_ns")]
            tail = max(finished, key=lambda d: d["seq"]) if finished else None
            pieces.append("GPU last finished kernel: " + (
                f"{tail.get('op')} #{tail['seq']}" if tail is not None else "none")
                + f" ({len(kernels) - len(finished)} started, not finished)")
        pieces.append(f"issued per channel: {counters or 'nothing'}")
        return " | ".join(pieces)

    # ---- output -------------------------------------------------------------------

    def _wall(self, perf_ns: int) -> float:
        return self._wall_anchor + (perf_ns - self._perf_anchor) / 1e9

    def _record(self, ev: Event) -> dict:
        return {
            "op": ev.op,
            "algorithm": ev.algorithm,
            "channel": ev.channel,
            "seq": ev.seq,
            "nbytes": ev.nbytes,
            "start_us": (ev.start_ns - self._perf_anchor) / 1e3,
            "dur_us": ev.duration_us if ev.done else None,
            "wall_start": self._wall(ev.start_ns),
            "detail": ev.detail,
        }

    def state(self) -> dict:
        """The ``rank<N>.json`` document."""
        with self._mutex:
            ring = self._ordered()
            open_ops = [self._open[k] for k in sorted(self._open)]
            counters = dict(self._next_seq)
            dropped = self.dropped
            capacity = len(self._slots)
        return {
            "rank": self.rank,
            "world_size": self.world_size,
            "wall_start": self._wall_anchor,
            "capacity": capacity,
            "dropped": dropped,
            "next_seq": counters,
            "pending": [self._record(ev) for ev in open_ops],
            "events": [self._record(ev) for ev in ring],
            "device_events": self.device_events(),
        }

    def dump(self, directory: str | Path) -> Path:
        """Write ``<directory>/rank<N>.json`` and return its path."""
        folder = Path(directory)
        folder.mkdir(parents=True, exist_ok=True)
        path = folder / f"rank{self.rank}.json"
        path.write_text(json.dumps(self.state(), indent=1), encoding="utf-8")
        return path

    def chrome_trace_events(self, wall_zero: float | None = None) -> list[dict]:
        """Trace Event Format records (pid = rank, tid = channel)."""
        origin = self._wall_anchor if wall_zero is None else wall_zero
        out: list[dict] = [{"name": "process_name", "ph": "M", "pid": self.rank,
                            "args": {"name": f"rank {self.rank}"}}]
        tracks: set[int] = set()
        for ev in self.events():
            if ev.channel not in tracks:
                tracks.add(ev.channel)
                label = {-1: "collective", -2: "pipeline"}.get(ev.channel, f"channel {ev.channel}")
                out.append({"name": "thread_name", "ph": "M", "pid": self.rank, "tid": ev.channel,
                            "args": {"name": label}})
            out.append({
                "name": f"{ev.op}:{ev.algorithm}" if ev.algorithm else ev.op,
                "cat": "collective",
                "ph": "X",
                "ts": (self._wall(ev.start_ns) - origin) * 1e6,
                "dur": ev.duration_us,
                "pid": self.rank,
                "tid": ev.channel,
                "args": {"seq": ev.seq, "bytes": ev.nbytes, **ev.detail},
            })
        return out

    def dump_chrome_trace(self, path: str | Path) -> Path:
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        target.write_text(json.dumps(self.chrome_trace_events()), encoding="utf-8")
        return target
