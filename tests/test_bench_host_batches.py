"""The end-to-end phase's batch source in bench.py, checked without a GPU.

``HostBatches`` hands each step a pinned (x, y) pair and draws the next pair
while the step runs; two buffers per input alternate, so the pair being drawn
is never the one whose host-to-device copy the current step enqueued.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_host_batches_alternate_buffers_and_draw_fresh_pairs(monkeypatch) -> None:
    # pinning needs a CUDA driver; the buffer logic does not
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    bench = _bench_module()
    src = bench.HostBatches(torch, rows=3, seq=5, vocab=1000, seed=7)
    seen = []
    for _ in range(4):
        x, y = src.current()
        assert x.shape == (3, 5) and y.shape == (3, 5) and x.dtype == torch.int64
        assert int(x.max()) < 1000 and int(x.min()) >= 0
        seen.append((x.data_ptr(), x.clone(), y.clone()))
        src.advance()
    # buffers alternate: step i and step i+2 share storage, i and i+1 do not
    assert seen[0][0] == seen[2][0] != seen[1][0] == seen[3][0]
    # every step sees a newly drawn pair
    for (_, xa, ya), (_, xb, yb) in zip(seen, seen[1:]):
        assert not torch.equal(xa, xb) and not torch.equal(ya, yb)


def test_host_batches_are_reproducible_from_the_seed(monkeypatch) -> None:
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    bench = _bench_module()
    a = bench.HostBatches(torch, rows=2, seq=4, vocab=50, seed=3)
    b = bench.HostBatches(torch, rows=2, seq=4, vocab=50, seed=3)
    for _ in range(3):
        assert all(torch.equal(u, v) for u, v in zip(a.current(), b.current()))
        a.advance()
        b.advance()
