"""DDP must train exactly like one process on the whole batch."""

from __future__ import annotations

import copy

import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200.ddp import DistributedDataParallel, average_gradients
from mini_nccl_b200.launcher import run


def net() -> nn.Module:
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(16, 48), nn.Tanh(), nn.Linear(48, 24), nn.Tanh(), nn.Linear(24, 1))


def _parity(pg, overlap: bool, cap_mb: float, steps: int = 6) -> None:
    W, per = pg.world_size, 8
    model = net()
    ref = copy.deepcopy(model)
    ddp = DistributedDataParallel(model, pg, bucket_cap_mb=cap_mb, overlap=overlap)
    if cap_mb < 0.01:
        assert len(ddp._buckets) > 1
    opt = torch.optim.SGD(model.parameters(), lr=0.1, momentum=0.9)
    ref_opt = torch.optim.SGD(ref.parameters(), lr=0.1, momentum=0.9)
    gen = torch.Generator().manual_seed(42)
    for _ in range(steps):
        x = torch.randn(W * per, 16, generator=gen)
        y = torch.randn(W * per, 1, generator=gen)
        mine = slice(pg.rank * per, (pg.rank + 1) * per)
        ddp.zero_grad()
        F.mse_loss(ddp(x[mine]), y[mine]).backward()
        ddp.sync()
        opt.step()
        ref_opt.zero_grad()
        F.mse_loss(ref(x), y).backward()
        ref_opt.step()
    for p, q in zip(model.parameters(), ref.parameters(), strict=True):
        torch.testing.assert_close(p, q, rtol=1e-4, atol=1e-5)


def _battery(pg) -> None:
    _parity(pg, overlap=True, cap_mb=1.0)
    _parity(pg, overlap=False, cap_mb=1.0)
    _parity(pg, overlap=True, cap_mb=0.001)


def test_ddp_matches_single_process() -> None:
    run(_battery, 2)


def test_ddp_matches_single_process_world3() -> None:
    run(_battery, 3)


def _no_sync(pg, steps: int = 4) -> None:
    W, micro = pg.world_size, 6
    model = net()
    ref = copy.deepcopy(model)
    ddp = DistributedDataParallel(model, pg)
    opt = torch.optim.SGD(model.parameters(), lr=0.05)
    ref_opt = torch.optim.SGD(ref.parameters(), lr=0.05)
    gen = torch.Generator().manual_seed(7)
    for _ in range(steps):
        x = torch.randn(W * 2 * micro, 16, generator=gen)
        y = torch.randn(W * 2 * micro, 1, generator=gen)
        a = slice(pg.rank * 2 * micro, pg.rank * 2 * micro + micro)
        b = slice(a.stop, a.stop + micro)
        ddp.zero_grad()
        with ddp.no_sync():
            (F.mse_loss(ddp(x[a]), y[a]) / 2).backward()
        (F.mse_loss(ddp(x[b]), y[b]) / 2).backward()
        ddp.sync()
        opt.step()
        ref_opt.zero_grad()
        F.mse_loss(ref(x), y).backward()
        ref_opt.step()
    for p, q in zip(model.parameters(), ref.parameters(), strict=True):
        torch.testing.assert_close(p, q, rtol=1e-4, atol=1e-5)


def test_no_sync_accumulates_without_communicating() -> None:
    run(_no_sync, 2)


def _broadcast_init(pg) -> None:
    torch.manual_seed(100 + pg.rank)
    m = nn.Linear(8, 8)
    DistributedDataParallel(m, pg)
    torch.manual_seed(100)
    want = nn.Linear(8, 8)
    torch.testing.assert_close(m.weight, want.weight)
    torch.testing.assert_close(m.bias, want.bias)


def test_ddp_broadcasts_initial_weights() -> None:
    run(_broadcast_init, 2)


def _grads_are_bucket_views(pg) -> None:
    model = net()
    ddp = DistributedDataParallel(model, pg, bucket_cap_mb=0.001)
    F.mse_loss(ddp(torch.randn(4, 16)), torch.randn(4, 1)).backward()
    ddp.sync()
    storages = {b.buffer.untyped_storage().data_ptr() for b in ddp._buckets}
    for p in model.parameters():
        assert p.grad.untyped_storage().data_ptr() in storages
    # buckets hold parameters in reverse registration order
    assert ddp._buckets[0].params[0] is list(model.parameters())[-1]


def test_gradients_live_in_the_buckets() -> None:
    run(_grads_are_bucket_views, 2)


def _avg(pg) -> None:
    ps = [nn.Parameter(torch.zeros(3)), nn.Parameter(torch.zeros(2, 2))]
    for p in ps:
        p.grad = torch.full(p.shape, float(pg.rank + 1))
    n = average_gradients(pg, ps)
    assert n == 7 * 4
    for p in ps:
        torch.testing.assert_close(p.grad, torch.full(p.shape, 1.5))


def test_average_gradients() -> None:
    run(_avg, 2)
