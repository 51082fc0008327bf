"""Local multi-process launcher.

``run(fn, world_size, *args)`` spawns one process per rank, builds a
:class:`ProcessGroup` in each, calls ``fn(pg, *args)`` and returns the
per-rank results (reference API: mini_nccl/launcher.py:72-154).

Differences from the reference that matter on a GPU box:

* ``devices="cuda"`` pins rank ``r`` to ``cuda:r`` (``cuda:r % n_gpus``)
  before anything touches CUDA, so each worker owns one GPU;
* the parent supervises through ``multiprocessing.connection.wait`` on the
  result pipe *and* every child's sentinel, so a rank that dies without
  reporting (``os._exit``, a segfault, the OOM killer) is noticed the moment
  it exits rather than at the next poll tick;
* a flight-recorder dump is written even when ``fn`` raises, since failures
  are when it matters.
"""

from __future__ import annotations

import contextlib
import multiprocessing as mp
import os
import socket
import time
import traceback
from multiprocessing.connection import wait
from pathlib import Path

from .process_group import DEFAULT_N_CHANNELS, ProcessGroup
from .transport import DEFAULT_OP_TIMEOUT


def _free_ports(count: int) -> list[int]:
    """``count`` distinct ports the OS considers free right now."""
    holders, ports = [], []
    for _ in range(count):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        holders.append(s)
        ports.append(s.getsockname()[1])
    for s in holders:
        s.close()
    return ports


def _worker(fn, rank, world_size, addrs, args, conn, options) -> None:
    trace_dir = options.get("trace_dir")
    device = options.get("device")
    pg = None
    try:
        if device == "cuda":
            import torch

            n = torch.cuda.device_count()
            dev = torch.device("cuda", rank % max(1, n))
            torch.cuda.set_device(dev)
            os.environ.setdefault("LOCAL_RANK", str(dev.index))
        else:
            dev = None
        pg = ProcessGroup(
            rank,
            world_size,
            addrs,
            n_channels=options.get("n_channels", DEFAULT_N_CHANNELS),
            op_timeout=options.get("op_timeout", DEFAULT_OP_TIMEOUT),
            trace=True if trace_dir else None,
            device=dev,
        )
        try:
            result = fn(pg, *args)
        finally:
            if trace_dir:
                pg.recorder.dump(trace_dir)
            pg.close()
        conn.send((rank, "ok", result))
    except BaseException:
        if pg is not None and trace_dir:
            with contextlib.suppress(Exception):
                pg.recorder.dump(trace_dir)
        with contextlib.suppress(Exception):
            conn.send((rank, "err", traceback.format_exc()))
        raise SystemExit(1) from None
    finally:
        with contextlib.suppress(Exception):
            conn.close()


def run(
    fn,
    world_size: int,
    *args,
    timeout: float = 300.0,
    n_channels: int = DEFAULT_N_CHANNELS,
    op_timeout: float = DEFAULT_OP_TIMEOUT,
    trace_dir: str | Path | None = None,
    devices: str | None = None,
) -> list:
    """Run ``fn(pg, *args)`` on ``world_size`` local processes.

    ``fn`` must be picklable (module level) because workers are spawned.
    Returns results indexed by rank; any failure raises one ``RuntimeError``
    listing every rank's traceback (and the diagnose command when tracing).
    """
    ctx = mp.get_context("spawn")
    addrs = [("127.0.0.1", p) for p in _free_ports(world_size)]
    options = {
        "n_channels": n_channels,
        "op_timeout": op_timeout,
        "trace_dir": str(trace_dir) if trace_dir else None,
        "device": devices,
    }
    pipes = []
    procs = []
    for r in range(world_size):
        parent_end, child_end = ctx.Pipe(duplex=False)
        p = ctx.Process(
            target=_worker,
            args=(fn, r, world_size, addrs, args, child_end, options),
            daemon=True,
        )
        p.start()
        child_end.close()
        pipes.append(parent_end)
        procs.append(p)

    results: dict[int, object] = {}
    errors: dict[int | str, str] = {}
    open_pipes = {id(c): (r, c) for r, c in enumerate(pipes)}
    sentinels = {p.sentinel: r for r, p in enumerate(procs)}
    reported: set[int] = set()
    deadline = time.monotonic() + timeout

    while len(reported) < world_size:
        left = deadline - time.monotonic()
        if left <= 0:
            errors["timeout"] = (
                f"timed out after {timeout}s waiting for ranks "
                f"{sorted(set(range(world_size)) - reported)}; "
                f"exitcodes={[p.exitcode for p in procs]}"
            )
            break
        ready = wait([c for _, c in open_pipes.values()] + list(sentinels), timeout=min(left, 1.0))
        for obj in ready:
            if obj in sentinels:
                continue
            r, conn = open_pipes[id(obj)]
            try:
                rank, status, payload = conn.recv()
            except (EOFError, OSError):
                del open_pipes[id(obj)]
                continue
            del open_pipes[id(obj)]
            reported.add(rank)
            if status == "ok":
                results[rank] = payload
            else:
                errors[rank] = payload
        # A rank that exited without reporting is a hard death.  Give its pipe
        # one last look first (a result may be in flight), then name it.
        for sent, r in list(sentinels.items()):
            if procs[r].exitcode is None:
                continue
            del sentinels[sent]
            if r in reported:
                continue
            conn = pipes[r]
            with contextlib.suppress(Exception):
                if conn.poll(0.2):
                    rank, status, payload = conn.recv()
                    reported.add(rank)
                    (results if status == "ok" else errors)[rank] = payload
                    open_pipes.pop(id(conn), None)
                    continue
            open_pipes.pop(id(conn), None)
            reported.add(r)
            errors[r] = (
                f"rank {r} exited with code {procs[r].exitcode} without reporting "
                f"(killed or crashed hard)"
            )

    for p in procs:
        p.join(5.0)
    for p in procs:
        if p.is_alive():
            p.terminate()
            p.join(2.0)

    if errors:
        detail = "\n\n".join(f"[{key}]\n{tb}" for key, tb in errors.items())
        hint = f"\n\nFlight recorder logs: python -m mini_nccl_b200.diagnose {trace_dir}" if trace_dir else ""
        raise RuntimeError(f"{len(errors)} worker failure(s):\n\n{detail}{hint}")
    return [results[r] for r in range(world_size)]
