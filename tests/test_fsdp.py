"""FSDP: same training as one process, less memory, correct recompute."""

from __future__ import annotations

import copy

import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200.fsdp import FullyShardedDataParallel
from mini_nccl_b200.launcher import run


class Block(nn.Module):
    def __init__(self, width: int) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(width)
        self.fc1 = nn.Linear(width, 2 * width)
        self.fc2 = nn.Linear(2 * width, width)

    def forward(self, x):
        return x + self.fc2(torch.tanh(self.fc1(self.norm(x))))


class Model(nn.Module):
    def __init__(self, width: int = 12, depth: int = 3) -> None:
        super().__init__()
        self.embed = nn.Linear(8, width)
        self.blocks = nn.ModuleList(Block(width) for _ in range(depth))
        self.head = nn.Linear(width, 1)

    def forward(self, x):
        h = self.embed(x)
        for b in self.blocks:
            h = b(h)
        return self.head(h)


def _parity(pg, steps: int = 5, recompute: bool = True, fuse_gather_gemm: bool = False) -> dict:
    W, per = pg.world_size, 6
    torch.manual_seed(0)
    model = Model()
    ref = copy.deepcopy(model)
    fsdp = FullyShardedDataParallel(model, pg, unit_cls=Block, recompute=recompute, fuse_gather_gemm=fuse_gather_gemm)
    assert len(fsdp.units) == 3
    if fuse_gather_gemm:  # 1-D parameters (LayerNorm, biases) stay whole; only matrices are sharded
        assert all(len(u.entries) == 2 and all(len(e[2]) == 2 for e in u.entries) for u in fsdp.units)
    assert all(u.shard.numel() < u.padded_numel or W == 1 for u in fsdp.units)
    opt = torch.optim.SGD(fsdp.parameters(), lr=0.05, momentum=0.9)
    ref_opt = torch.optim.SGD(ref.parameters(), lr=0.05, momentum=0.9)
    gen = torch.Generator().manual_seed(11)
    for _ in range(steps):
        x = torch.randn(W * per, 8, generator=gen)
        y = torch.randn(W * per, 1, generator=gen)
        mine = slice(pg.rank * per, (pg.rank + 1) * per)
        fsdp.zero_grad()
        F.mse_loss(fsdp(x[mine]), y[mine]).backward()
        fsdp.sync()
        opt.step()
        ref_opt.zero_grad()
        F.mse_loss(ref(x), y).backward()
        ref_opt.step()
    state = fsdp.full_state_dict()
    for name, p in ref.named_parameters():
        torch.testing.assert_close(state[name], p.detach(), rtol=1e-4, atol=1e-5, msg=lambda m, n=name: f"{n}: {m}")
    return fsdp.memory_report()


def test_fsdp_matches_single_process() -> None:
    reports = run(_parity, 2)
    assert reports[0] == reports[1]


def test_fsdp_without_recompute_matches_single_process() -> None:
    """Activations saved, parameters freed after forward and gathered again for backward."""
    reports = run(_parity, 2, 5, False)
    assert reports[0] == reports[1]
    run(_parity, 3, 3, False)


def test_fsdp_units_keeping_vectors_whole_match_single_process() -> None:
    """The layout fuse_gather_gemm uses (on CPU the gather itself is the plain one):
    vectors replicated and averaged in sync(), matrices sharded."""
    reports = run(_parity, 2, 4, False, True)
    assert reports[0] == reports[1]


def test_fuse_gather_gemm_needs_saved_activations() -> None:
    import pytest

    with pytest.raises(RuntimeError, match="fuse_gather_gemm needs recompute=False"):
        run(_fused_with_recompute, 1)  # the worker's ValueError comes back through the launcher


def _fused_with_recompute(pg) -> None:
    FullyShardedDataParallel(Model(), pg, unit_cls=Block, recompute=True, fuse_gather_gemm=True)


def test_fsdp_matches_single_process_world4() -> None:
    run(_parity, 4)


class DropBlock(nn.Module):
    def __init__(self, width: int = 16) -> None:
        super().__init__()
        self.fc = nn.Linear(width, width)
        self.drop = nn.Dropout(0.5)

    def forward(self, x):
        return x + self.drop(torch.tanh(self.fc(x)))


class DropModel(nn.Module):
    def __init__(self, width: int = 16) -> None:
        super().__init__()
        torch.manual_seed(0)
        self.blocks = nn.ModuleList(DropBlock(width) for _ in range(2))
        self.head = nn.Linear(width, 1)

    def forward(self, x):
        for b in self.blocks:
            x = b(x)
        return self.head(x)


def _dropout(pg, width: int = 16) -> None:
    """The recompute must replay the dropout mask; check the *sharded* grads.

    The head sits downstream of the recomputed units, so its gradient stays
    right even when the mask is wrong -- only the unit shards reveal the bug.
    """
    model = DropModel(width)
    ref = copy.deepcopy(model)
    fsdp = FullyShardedDataParallel(model, pg, unit_cls=DropBlock)
    model.train()
    ref.train()
    x = torch.randn(8, width, generator=torch.Generator().manual_seed(1))
    y = torch.randn(8, 1, generator=torch.Generator().manual_seed(2))
    torch.manual_seed(99)
    fsdp.zero_grad()
    F.mse_loss(fsdp(x), y).backward()
    fsdp.sync()
    torch.manual_seed(99)
    ref.zero_grad()
    F.mse_loss(ref(x), y).backward()
    for i, unit in enumerate(fsdp.units):
        blk = ref.blocks[i]
        want = torch.cat([blk.fc.weight.grad.reshape(-1), blk.fc.bias.grad.reshape(-1)])
        torch.testing.assert_close(unit.shard.grad[: want.numel()], want, rtol=1e-5, atol=1e-6)


def test_recompute_replays_randomness() -> None:
    run(_dropout, 1)


def _memory(pg) -> dict:
    model = Model(width=64, depth=4)
    fsdp = FullyShardedDataParallel(model, pg, unit_cls=Block)
    fsdp(torch.randn(4, 8)).sum().backward()
    fsdp.sync()
    return fsdp.memory_report()


def test_fsdp_reduces_parameter_memory() -> None:
    W = 4
    rep = run(_memory, W)[0]
    assert abs(rep["sharded_params_resident"] - rep["sharded_params_full"] // W) <= 4 * W
    assert rep["peak_transient"] <= (rep["sharded_params_full"] // 4) * 1.1, rep
    assert rep["fsdp_peak"] < rep["ddp_equivalent"], rep


def _opt_state(pg) -> int:
    model = Model(width=64, depth=4)
    fsdp = FullyShardedDataParallel(model, pg, unit_cls=Block)
    opt = torch.optim.Adam(fsdp.parameters(), lr=1e-3)
    fsdp.zero_grad()
    fsdp(torch.randn(4, 8)).sum().backward()
    fsdp.sync()
    opt.step()
    return sum(v.numel() for st in opt.state.values() for v in st.values() if isinstance(v, torch.Tensor))


def test_optimizer_state_is_sharded() -> None:
    sharded = run(_opt_state, 4)[0]
    single = run(_opt_state, 1)[0]
    assert sharded < single * 0.6, (sharded, single)


def _sharded_ckpt(pg, path) -> None:
    torch.manual_seed(0)
    fsdp = FullyShardedDataParallel(Model(), pg, unit_cls=Block)
    state = fsdp.sharded_state_dict()
    torch.save(state, f"{path}/shard{pg.rank}.pt")
    with torch.no_grad():
        for u in fsdp.units:
            u.shard.zero_()
    fsdp.load_sharded_state_dict(torch.load(f"{path}/shard{pg.rank}.pt"))
    for u, want in zip(fsdp.units, state["shards"].values(), strict=True):
        assert torch.equal(u.shard.detach(), want)


def test_sharded_checkpoint_round_trip(tmp_path) -> None:
    run(_sharded_ckpt, 2, str(tmp_path))


def _opt_in_backward(pg, steps: int = 4, recompute: bool = True) -> None:
    """AdamW fused into the gradient reduce-scatter == single-process AdamW."""
    W, per = pg.world_size, 6
    torch.manual_seed(0)
    model = Model()
    ref = copy.deepcopy(model)
    hp = dict(lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    fsdp = FullyShardedDataParallel(model, pg, unit_cls=Block, optimizer_in_backward=hp, recompute=recompute)
    rest = torch.optim.AdamW([p for p in fsdp.parameters() if all(p is not u.shard for u in fsdp.units)], **hp)
    ref_opt = torch.optim.AdamW(ref.parameters(), **hp)
    gen = torch.Generator().manual_seed(11)
    for _ in range(steps):
        x = torch.randn(W * per, 8, generator=gen)
        y = torch.randn(W * per, 1, generator=gen)
        mine = slice(pg.rank * per, (pg.rank + 1) * per)
        fsdp.zero_grad()
        F.mse_loss(fsdp(x[mine]), y[mine]).backward()
        assert all(u.shard.grad is None for u in fsdp.units)  # consumed inside the reduce-scatter
        fsdp.sync()
        rest.step()
        ref_opt.zero_grad()
        F.mse_loss(ref(x), y).backward()
        ref_opt.step()
    state = fsdp.full_state_dict()
    for name, p in ref.named_parameters():
        torch.testing.assert_close(state[name], p.detach(), rtol=1e-4, atol=1e-5, msg=lambda m, n=name: f"{n}: {m}")


def test_optimizer_in_backward_matches_single_process() -> None:
    run(_opt_in_backward, 2)


def test_optimizer_in_backward_without_recompute() -> None:
    run(_opt_in_backward, 2, 4, False)


def _train(fsdp, opt, pg, steps: int, first_step: int) -> None:
    W, per = pg.world_size, 5
    for k in range(first_step, first_step + steps):
        gen = torch.Generator().manual_seed(900 + k)  # batch k is the same however the run was split
        x = torch.randn(W * per, 8, generator=gen)
        y = torch.randn(W * per, 1, generator=gen)
        mine = slice(pg.rank * per, (pg.rank + 1) * per)
        fsdp.zero_grad()
        F.mse_loss(fsdp(x[mine]), y[mine]).backward()
        fsdp.sync()
        opt.step()


def _resume_bit_exact(pg, path, fused: bool) -> None:
    hp = dict(lr=3e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)

    def fresh():
        torch.manual_seed(3)
        fsdp = FullyShardedDataParallel(Model(), pg, unit_cls=Block,
                                        optimizer_in_backward=hp if fused else None)
        # With the shard optimizer fused into backward the user's optimizer only
        # sees the replicated parameters; otherwise it steps shards too.
        params = fsdp.replicated_parameters() if fused else list(fsdp.parameters())
        return fsdp, torch.optim.AdamW(params, **hp)

    straight, straight_opt = fresh()
    _train(straight, straight_opt, pg, 4, 0)

    first, first_opt = fresh()
    _train(first, first_opt, pg, 2, 0)
    ckpt = path / f"rank{pg.rank}.pt"
    torch.save(first.sharded_state_dict(optimizer=first_opt), ckpt)
    del first, first_opt

    resumed, resumed_opt = fresh()
    resumed.load_sharded_state_dict(torch.load(ckpt, weights_only=False), optimizer=resumed_opt)
    _train(resumed, resumed_opt, pg, 2, 2)

    for (name, a), b in zip(straight.full_state_dict().items(), resumed.full_state_dict().values(), strict=True):
        assert torch.equal(a, b), f"{name} differs after resuming"
    if fused:
        for name, st in straight.shard_optimizer.state.items():
            other = resumed.shard_optimizer.state[name]
            assert st["step"] == other["step"] == 4
            assert torch.equal(st["m"], other["m"]) and torch.equal(st["v"], other["v"])


def test_resume_from_sharded_checkpoint_is_bit_exact(tmp_path) -> None:
    """2 steps, save, load into a fresh model, 2 more steps == 4 uninterrupted steps."""
    run(_resume_bit_exact, 2, tmp_path, False)


def test_resume_with_fused_shard_optimizer_is_bit_exact(tmp_path) -> None:
    """The fused reduce-scatter + AdamW keeps its moments and step count across a resume."""
    run(_resume_bit_exact, 2, tmp_path, True)
