"""Read flight-recorder dumps and name the rank that is the problem.

    python -m mini_nccl_b200.diagnose <trace_dir> [--trace merged.json]

Reads every ``rank*.json`` written by :meth:`Recorder.dump` and reports, in
the reference's terms (mini_nccl/diagnose.py:1-262):

* per-rank progress per channel (and how many old events a ring dropped);
* **DESYNC**: the first collective sequence number at which ranks recorded
  different operations, or, failing that, ranks that stopped early.  Streams
  are aligned by sequence number, never by list position, so logs that wrapped
  by different amounts still line up;
* **STRAGGLER**: the rank whose collectives are consistently the *fastest*.
  Arriving last, it finds everyone waiting and returns at once, while the
  others spend the wait inside the collective;
* **UNFINISHED** operations that never returned;
* device-side progress: the last kernel-level sequence number each GPU
  completed, from the device event ring, and any rank whose kernel stream
  disagrees with the others.

Exit status 0 when clean, 1 when something is wrong.  ``--trace`` merges all
ranks into one Trace Event Format file (one process per rank, one track per
channel).
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

CHANNEL_LABEL = {-1: "collective order", -2: "pipeline"}


def load(directory: Path) -> list[dict]:
    states = [json.loads(p.read_text(encoding="utf-8")) for p in sorted(Path(directory).glob("rank*.json"))]
    if not states:
        raise SystemExit(f"no rank*.json dumps found in {directory}")
    return sorted(states, key=lambda s: s["rank"])


def _collective_streams(states: list[dict]) -> dict[int, dict[int, dict]]:
    """rank -> {seq: event} for the collective-order channel."""
    return {s["rank"]: {e["seq"]: e for e in s["events"] if e["channel"] == -1} for s in states}


def _find_divergence(streams: dict[int, dict[int, dict]]) -> int:
    if len(streams) < 2:
        return 0
    every_seq = sorted(set().union(*(d.keys() for d in streams.values())))
    for seq in every_seq:
        holders = {rank: d[seq] for rank, d in streams.items() if seq in d}
        if len(holders) < 2:
            continue
        sig = {rank: (e["op"], e["nbytes"]) for rank, e in holders.items()}
        if len(set(sig.values())) == 1:
            continue
        print(f"\nDESYNC at collective #{seq}: ranks issued *different* collectives.")
        for rank in sorted(sig):
            op, nbytes = sig[rank]
            print(f"    rank {rank}: {op} ({nbytes} bytes)")
        print(
            "  Ranks must issue identical collective sequences. Look at what the odd "
            "rank out did just before this point (a conditional, an early return, an "
            "unequal number of batches)."
        )
        return 1
    last = {rank: (max(d) if d else -1) for rank, d in streams.items()}
    if len(set(last.values())) > 1:
        top = max(last.values())
        behind = sorted(r for r, v in last.items() if v < top)
        print(
            f"\nDESYNC: ranks {behind} stopped early, reaching collective "
            f"#{[last[r] for r in behind]} while others reached #{top}.\n"
            f"  The lagging ranks are the cause; the rest are blocked waiting on them."
        )
        return 1
    return 0


def _straggler_report(states: list[dict], factor: float = 1.5, min_samples: int = 3) -> None:
    """Name a rank whose collective durations are consistently short (see module doc)."""
    if len(states) < 3:
        return
    durations: dict[int, dict[str, list[float]]] = {}
    for s in states:
        per_op: dict[str, list[float]] = {}
        for e in s["events"]:
            if e["channel"] == -1 and e["dur_us"] is not None:
                per_op.setdefault(e["op"], []).append(e["dur_us"])
        durations[s["rank"]] = per_op
    ops = sorted({op for per_op in durations.values() for op in per_op})
    quick = dict.fromkeys(durations, 0)
    judged = 0
    for op in ops:
        med = {
            rank: statistics.median(per_op[op])
            for rank, per_op in durations.items()
            if len(per_op.get(op, ())) >= min_samples
        }
        if len(med) < 3:
            continue
        judged += 1
        typical = statistics.median(med.values())
        if typical <= 0:
            continue
        for rank, m in med.items():
            if m * factor < typical:
                quick[rank] += 1
    if not judged:
        return
    for rank, n in sorted(quick.items()):
        if n > judged / 2:
            print(
                f"\nSTRAGGLER: rank {rank} spent less than 1/{factor:g} of the median "
                f"time inside {n} of {judged} collectives.\n"
                f"  It arrives last, finds its peers already waiting and returns at "
                f"once. Look for a slower host, an unbalanced shard or contention on "
                f"that rank, not at the ranks reporting long waits."
            )


def _device_report(states: list[dict]) -> int:
    """Compare kernel-level collective streams written by the GPUs themselves."""
    streams = {}
    for s in states:
        recs = [d for d in s.get("device_events", []) if "seq" in d]
        if recs:
            streams[s["rank"]] = {d["seq"]: d for d in recs}
    if not streams:
        return 0
    print("\ndevice progress (last kernel-level collective completed):")
    for rank, d in sorted(streams.items()):
        done = [q for q, rec in d.items() if rec.get("end_ns")]
        print(f"  rank {rank}: seq {max(done) if done else None} of {len(d)} recorded")
    findings = 0
    common = set.intersection(*(set(d) for d in streams.values())) if len(streams) > 1 else set()
    for seq in sorted(common):
        sig = {rank: (d[seq].get("op"), d[seq].get("nbytes")) for rank, d in streams.items()}
        if len(set(sig.values())) > 1:
            print(f"\nDEVICE DESYNC at kernel seq #{seq}: " + ", ".join(
                f"rank {r}: {op} ({nb} bytes)" for r, (op, nb) in sorted(sig.items())))
            findings += 1
            break
    for rank, d in sorted(streams.items()):
        for seq, rec in sorted(d.items()):
            if rec.get("status", 0) not in (0, None):
                print(f"\nDEVICE ERROR on rank {rank}: kernel seq {seq} ({rec.get('op')}) "
                      f"ended with status {rec['status']} (timeout waiting on a peer)")
                findings += 1
    return findings


def report(states: list[dict]) -> int:
    """Print a diagnosis; return the exit code (0 clean, 1 suspicious)."""
    world = states[0]["world_size"]
    print(f"ranks reporting: {len(states)}/{world}")
    findings = 0
    missing = sorted(set(range(world)) - {s["rank"] for s in states})
    if missing:
        print(f"  MISSING DUMPS from ranks {missing} (crashed before writing?)")
        findings += 1
    print("\nper-rank progress (collectives issued, by channel):")
    for s in states:
        counts = {CHANNEL_LABEL.get(int(c), f"ch{c}"): n for c, n in sorted(s["next_seq"].items(), key=lambda kv: int(kv[0]))}
        note = f"  [ring buffer dropped {s['dropped']} older events]" if s.get("dropped") else ""
        print(f"  rank {s['rank']}: {counts}{note}")
    findings += _find_divergence(_collective_streams(states))
    _straggler_report(states)
    findings += _device_report(states)
    for s in states:
        for e in s["pending"]:
            print(
                f"\nUNFINISHED on rank {s['rank']}: {e['op']}[{e['algorithm']}] "
                f"seq={e['seq']} channel={e['channel']} bytes={e['nbytes']} never completed."
            )
            findings += 1
    if not findings:
        print("\nno desync or unfinished collectives found; all ranks agree.")
    return 1 if findings else 0


def merge_trace(states: list[dict], out_path: Path) -> None:
    """One Trace Event Format file for every rank."""
    zero = min(s["wall_start"] for s in states)
    records: list[dict] = []
    for s in states:
        rank = s["rank"]
        records.append({"name": "process_name", "ph": "M", "pid": rank, "args": {"name": f"rank {rank}"}})
        named: set[int] = set()
        for e in s["events"]:
            ch = e["channel"]
            if ch not in named:
                named.add(ch)
                records.append({"name": "thread_name", "ph": "M", "pid": rank, "tid": ch,
                                "args": {"name": CHANNEL_LABEL.get(ch, f"channel {ch}")}})
            records.append({
                "name": f"{e['op']}:{e['algorithm']}" if e["algorithm"] else e["op"],
                "cat": "collective",
                "ph": "X",
                "ts": (e["wall_start"] - zero) * 1e6,
                "dur": e["dur_us"] if e["dur_us"] is not None else 0.0,
                "pid": rank,
                "tid": ch,
                "args": {"seq": e["seq"], "bytes": e["nbytes"], "completed": e["dur_us"] is not None,
                         **e.get("detail", {})},
            })
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_text(json.dumps(records), encoding="utf-8")
    print(f"\nwrote merged trace {out_path} ({len(records)} records)")
    print("open it in https://ui.perfetto.dev or chrome://tracing")


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("directory", type=Path, help="directory of rank*.json dumps")
    ap.add_argument("--trace", type=Path, help="also write a merged Chrome trace here")
    args = ap.parse_args(argv)
    states = load(args.directory)
    code = report(states)
    if args.trace:
        merge_trace(states, args.trace)
    raise SystemExit(code)


if __name__ == "__main__":
    main()
