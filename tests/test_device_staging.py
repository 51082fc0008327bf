"""The host-staged device API: chunking, the pipelined ring, the staged path.

These entry points move a GPU tensor through pinned host memory (the path for
ranks that share no peer memory); on CPU tensors the same chunking and
window logic runs with ordinary copies, which is what these tests exercise.
The CUDA path is covered in tests/test_device_comm_gpu.py.
(Reference behaviour: tests/test_device.py:44-122.)
"""

from __future__ import annotations

import pytest
import torch

from mini_nccl_b200 import device as D
from mini_nccl_b200.launcher import run


@pytest.mark.parametrize("numel,chunk_bytes", [(1, 4), (10, 8), (1000, 64), (1 << 16, 1 << 12), (12345, 400)])
def test_staging_ranges_cover_the_payload_exactly(numel, chunk_bytes):
    st = D.Staging(numel, torch.float32, torch.device("cpu"), chunk_bytes=chunk_bytes)
    spans = st.ranges(numel)
    assert spans[0][0] == 0 and spans[-1][1] == numel
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert all(0 < hi - lo <= st.chunk_numel for lo, hi in spans)
    assert len(spans) == st.n_chunks
    assert 1 <= len(st.slots) <= 2


def test_staging_payload_smaller_than_a_chunk():
    st = D.Staging(3, torch.float32, torch.device("cpu"), chunk_bytes=1 << 20)
    assert st.chunk_numel == 3 and st.n_chunks == 1 and len(st.slots) == 1
    assert st.ranges(3) == [(0, 3)]


def _pipelined(pg, numel, chunk_bytes):
    # integer-valued payloads: every summation order gives the same bits
    g = torch.Generator().manual_seed(50 + pg.rank)
    t = torch.randint(-100, 100, (numel,), generator=g).float()
    D.all_reduce_pipelined(pg, t, chunk_bytes=chunk_bytes)
    want = sum(torch.randint(-100, 100, (numel,), generator=torch.Generator().manual_seed(50 + r)).float()
               for r in range(pg.world_size))
    assert torch.equal(t, want), (numel, chunk_bytes)
    return True


@pytest.mark.parametrize("chunk_bytes", [64, 1024, 1 << 20])
def test_pipelined_matches_expected_for_any_chunk_size(chunk_bytes):
    run(_pipelined, 3, 10_001, chunk_bytes, timeout=120.0)


def _vs_ring(pg):
    g = torch.Generator().manual_seed(7 + pg.rank)
    x = torch.randint(-9, 9, (4099,), generator=g).float()
    a, b = x.clone(), x.clone()
    D.all_reduce_pipelined(pg, a, chunk_bytes=512)
    from mini_nccl_b200 import collectives as C

    C.all_reduce(pg, b, algorithm="ring")
    assert torch.equal(a, b)
    return True


def test_pipelined_agrees_with_the_plain_ring():
    run(_vs_ring, 2, timeout=120.0)


def _staged(pg):
    t = torch.full((777,), float(pg.rank + 1))
    D.all_reduce_staged(pg, t, op="max", algorithm="tree")
    assert torch.equal(t, torch.full((777,), float(pg.world_size)))
    return True


def test_staged_on_cpu_tensors():
    run(_staged, 3, timeout=120.0)


def _order_count(pg):
    calls = []
    orig = D.Staging.order_after_compute

    def spy(self):
        calls.append(1)
        orig(self)

    D.Staging.order_after_compute = spy
    try:
        D.all_reduce_pipelined(pg, torch.ones(4096), chunk_bytes=1024)
    finally:
        D.Staging.order_after_compute = orig
    return len(calls)


def test_every_exchange_orders_the_copy_stream_behind_compute():
    """Mechanism check: each of the 2(W-1) ring exchanges expresses the dependency."""
    counts = run(_order_count, 3, timeout=120.0)
    assert counts == [2 * (3 - 1)] * 3


def test_pipelined_rejects_non_contiguous():
    class Solo:
        rank, world_size = 0, 2

    with pytest.raises(ValueError, match="contiguous"):
        D.all_reduce_pipelined(Solo(), torch.ones(4, 4).t())


def test_device_report_is_honest():
    rep = D.device_report()
    assert rep["torch"] == torch.__version__
    assert rep["cuda_available"] == torch.cuda.is_available()
    if not torch.cuda.is_available():
        assert "device_name" not in rep
    else:
        assert rep["device_count"] == torch.cuda.device_count()
        assert len(rep["peer_access"]) == rep["device_count"]
    assert D.is_accelerated(torch.ones(1)) is False
