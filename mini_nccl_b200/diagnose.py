"""Read flight-recorder dumps and point at the rank that broke the job.

    python -m mini_nccl_b200.diagnose <trace_dir> [--trace merged.json]

Input: the ``rank*.json`` files :meth:`Recorder.dump` writes (the format the
reference's ``mini_nccl/diagnose.py:1-262`` reads).  Each rank's dump becomes a
:class:`RankTrace`; independent analyses each return a list of
:class:`Finding`; the report prints them and exits 1 if any is an error.

Analyses:

* **coverage** -- ranks without a dump (they died before writing it).
* **desync** -- collectives are matched across ranks by their per-channel
  sequence number (never by list position, so logs that wrapped by
  different amounts still line up).  The first number at which the ranks'
  ``(op, nbytes)`` signatures disagree is reported as
  ``DESYNC at collective #N`` with one ``rank R: op`` line per rank; the
  ranks that differ from the majority are named.  With no disagreement,
  ranks whose streams end before the others' are named instead.
* **arrival order** (advisory) -- for every collective that all ranks
  recorded, the rank that spent the least time inside it is the one the
  others waited for: it arrived last.  A rank that arrives last, by a clear
  margin, in most collectives is reported as ``STRAGGLER``.
* **unfinished** -- operations that started and never returned.
* **device streams** -- the kernel-level records each GPU wrote (sequence
  number, op, status): the last kernel each GPU finished, the first kernel
  number at which GPUs ran different collectives, and kernels that ended
  with an error status (a bounded wait that gave up on a peer).

``--trace`` also writes every rank's events into one Trace Event Format file
(one process per rank, one track per channel) for Perfetto.
"""

from __future__ import annotations

import argparse
import json
import statistics
from collections import Counter
from dataclasses import dataclass, field
from pathlib import Path

COLLECTIVE_CHANNEL = -1
TRACK_NAMES = {-1: "collective order", -2: "pipeline"}


@dataclass
class Finding:
    kind: str
    error: bool
    lines: list[str] = field(default_factory=list)


class RankTrace:
    """One rank's dump, indexed for cross-rank comparison."""

    def __init__(self, state: dict) -> None:
        self.state = state
        self.rank = int(state["rank"])
        self.world = int(state["world_size"])
        self.collectives = {e["seq"]: e for e in state["events"] if e["channel"] == COLLECTIVE_CHANNEL}
        self.kernels = {d["seq"]: d for d in state.get("device_events", []) if "seq" in d}

    def signature(self, seq: int) -> tuple[str, int] | None:
        e = self.collectives.get(seq)
        return None if e is None else (e["op"], e["nbytes"])

    def duration(self, seq: int) -> float | None:
        e = self.collectives.get(seq)
        return None if e is None else e["dur_us"]

    @property
    def last_seq(self) -> int:
        return max(self.collectives, default=-1)

    def issued(self) -> dict[str, int]:
        return {TRACK_NAMES.get(int(c), f"channel {c}"): n
                for c, n in sorted(self.state["next_seq"].items(), key=lambda kv: int(kv[0]))}


def load(directory: Path) -> list[dict]:
    paths = sorted(Path(directory).glob("rank*.json"))
    if not paths:
        raise SystemExit(f"no rank*.json dumps found in {directory}")
    return sorted((json.loads(p.read_text(encoding="utf-8")) for p in paths), key=lambda s: s["rank"])


# ---- analyses ------------------------------------------------------------------------


def check_coverage(traces: list[RankTrace]) -> list[Finding]:
    absent = sorted(set(range(traces[0].world)) - {t.rank for t in traces})
    if not absent:
        return []
    return [Finding("coverage", True, [f"  MISSING DUMPS from ranks {absent}: these processes ended without "
                                       f"writing their log (a crash or a kill), so look at them first."])]


def check_desync(traces: list[RankTrace]) -> list[Finding]:
    if len(traces) < 2:
        return []
    numbers = sorted(set().union(*(t.collectives for t in traces)))
    for seq in numbers:
        sigs = {t.rank: s for t in traces if (s := t.signature(seq)) is not None}
        if len(sigs) < 2 or len(set(sigs.values())) == 1:
            continue
        majority, _ = Counter(sigs.values()).most_common(1)[0]
        odd = sorted(r for r, s in sigs.items() if s != majority)
        lines = [f"DESYNC at collective #{seq}: the ranks disagree on which collective this is."]
        lines += [f"    rank {r}: {op} ({nbytes} bytes)" for r, (op, nbytes) in sorted(sigs.items())]
        lines.append(f"  Most ranks ran {majority[0]} ({majority[1]} bytes); rank(s) {odd} ran something else. "
                     f"Their code took a different path before collective #{seq}: check what they executed "
                     f"between #{seq - 1} and #{seq} (a branch on rank or data, a skipped step, an extra batch).")
        return [Finding("desync", True, lines)]
    ends = {t.rank: t.last_seq for t in traces}
    furthest = max(ends.values())
    short = sorted(r for r, e in ends.items() if e < furthest)
    if not short:
        return []
    return [Finding("desync", True, [
        f"DESYNC: ranks {short} stopped early, at collectives #{[ends[r] for r in short]}, "
        f"while the others reached #{furthest}.",
        "  Every collective before that matched, so the ranks that stopped are the cause (an exception, a hang "
        "outside communication, an early exit); the others are only waiting for them."])]


def check_arrival_order(traces: list[RankTrace], margin: float = 1.5, min_votes: int = 3) -> list[Finding]:
    """Name a rank that is usually the last to reach a collective (advisory)."""
    if len(traces) < 3:
        return []
    shared = set.intersection(*(set(t.collectives) for t in traces))
    votes: Counter[int] = Counter()
    judged = 0
    for seq in sorted(shared):
        times = {t.rank: t.duration(seq) for t in traces}
        if any(v is None for v in times.values()):
            continue
        judged += 1
        quickest = min(times, key=lambda r: times[r])
        rest = [v for r, v in times.items() if r != quickest]
        if times[quickest] * margin < statistics.median(rest):
            votes[quickest] += 1
    if judged < min_votes or not votes:
        return []
    rank, n = votes.most_common(1)[0]
    if n * 2 <= judged:
        return []
    return [Finding("arrival", False, [
        f"STRAGGLER: rank {rank} arrived last at {n} of {judged} collectives that every rank completed.",
        f"  It spends the least time inside each collective because the others are already waiting when it "
        f"arrives, so the delay is in rank {rank}'s work between collectives (its data, its host, its GPU), "
        f"not in the communication the other ranks report as slow."])]


def check_unfinished(traces: list[RankTrace]) -> list[Finding]:
    out = []
    for t in traces:
        for e in t.state["pending"]:
            out.append(Finding("unfinished", True, [
                f"UNFINISHED on rank {t.rank}: {e['op']}[{e['algorithm']}] seq={e['seq']} "
                f"channel={e['channel']} bytes={e['nbytes']} never completed."]))
    return out


def check_device_streams(traces: list[RankTrace]) -> list[Finding]:
    with_kernels = [t for t in traces if t.kernels]
    if not with_kernels:
        return []
    progress = ["device progress (last kernel-level collective completed):"]
    for t in with_kernels:
        finished = [s for s, rec in t.kernels.items() if rec.get("end_ns")]
        progress.append(f"  rank {t.rank}: seq {max(finished) if finished else None} of {len(t.kernels)} recorded")
    out = [Finding("device", False, progress)]
    if len(with_kernels) > 1:
        common = set.intersection(*(set(t.kernels) for t in with_kernels))
        for seq in sorted(common):
            sigs = {t.rank: (t.kernels[seq].get("op"), t.kernels[seq].get("nbytes")) for t in with_kernels}
            if len(set(sigs.values())) > 1:
                out.append(Finding("device", True, [f"DEVICE DESYNC at kernel seq #{seq}: " + ", ".join(
                    f"rank {r}: {op} ({nb} bytes)" for r, (op, nb) in sorted(sigs.items()))]))
                break
    for t in with_kernels:
        for seq, rec in sorted(t.kernels.items()):
            if rec.get("status", 0) not in (0, None):
                out.append(Finding("device", True, [
                    f"DEVICE ERROR on rank {t.rank}: kernel seq {seq} ({rec.get('op')}) ended with status "
                    f"{rec['status']}: one of its waits on a peer ran out of time."]))
    return out


ANALYSES = (check_coverage, check_desync, check_arrival_order, check_device_streams, check_unfinished)


def report(states: list[dict]) -> int:
    """Print the diagnosis; return the exit code (0 clean, 1 something is wrong)."""
    traces = [RankTrace(s) for s in states]
    print(f"ranks reporting: {len(traces)}/{traces[0].world}")
    print("\nper-rank progress (collectives issued, by channel):")
    for t in traces:
        wrapped = t.state.get("dropped")
        print(f"  rank {t.rank}: {t.issued()}" + (f"  [ring buffer dropped {wrapped} older events]" if wrapped else ""))
    findings = [f for analysis in ANALYSES for f in analysis(traces)]
    for f in findings:
        print("\n" + "\n".join(f.lines))
    errors = sum(f.error for f in findings)
    if not errors:
        print("\nno desync or unfinished collectives found; all ranks agree.")
    return 1 if errors else 0


def merge_trace(states: list[dict], out_path: Path) -> None:
    """Write every rank's events into one Trace Event Format file."""
    origin = min(s["wall_start"] for s in states)
    out: list[dict] = []
    for s in states:
        pid = s["rank"]
        out.append({"name": "process_name", "ph": "M", "pid": pid, "args": {"name": f"rank {pid}"}})
        tracks = sorted({e["channel"] for e in s["events"]})
        out += [{"name": "thread_name", "ph": "M", "pid": pid, "tid": ch,
                 "args": {"name": TRACK_NAMES.get(ch, f"channel {ch}")}} for ch in tracks]
        for e in s["events"]:
            out.append({
                "name": f"{e['op']}:{e['algorithm']}" if e["algorithm"] else e["op"],
                "cat": "collective",
                "ph": "X",
                "ts": (e["wall_start"] - origin) * 1e6,
                "dur": e["dur_us"] or 0.0,
                "pid": pid,
                "tid": e["channel"],
                "args": {"seq": e["seq"], "bytes": e["nbytes"], "completed": e["dur_us"] is not None,
                         **e.get("detail", {})},
            })
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_text(json.dumps(out), encoding="utf-8")
    print(f"\nwrote merged trace {out_path} ({len(out)} records); open it in https://ui.perfetto.dev")


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("directory", type=Path, help="directory of rank*.json dumps")
    ap.add_argument("--trace", type=Path, help="also write a merged Trace Event Format file here")
    args = ap.parse_args(argv)
    states = load(args.directory)
    code = report(states)
    if args.trace:
        merge_trace(states, args.trace)
    raise SystemExit(code)


if __name__ == "__main__":
    main()
