"""Tensor-parallel layers against unsharded references: outputs *and* grads."""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200 import collectives
from mini_nccl_b200.launcher import run
from mini_nccl_b200.tensor_parallel import (
    ColumnParallelLinear,
    ParallelMLP,
    ParallelSelfAttention,
    RowParallelLinear,
    _qkv_shard_rows,
)

WIDTH, BATCH = 16, 4


def _mlp(pg) -> None:
    torch.manual_seed(3)
    ref = nn.Sequential(nn.Linear(WIDTH, 4 * WIDTH), nn.GELU(), nn.Linear(4 * WIDTH, WIDTH))
    up, down = ref[0], ref[2]
    par = ParallelMLP(WIDTH, pg)
    par.up.load_full_weight(up.weight.detach(), up.bias.detach())
    par.down.load_full_weight(down.weight.detach(), down.bias.detach())
    if pg.world_size > 1:
        assert par.up.weight.numel() < up.weight.numel()
    g = torch.Generator().manual_seed(5)
    x = torch.randn(BATCH, WIDTH, generator=g)
    gy = torch.randn(BATCH, WIDTH, generator=g)
    xr = x.clone().requires_grad_(True)
    ref(xr).backward(gy)
    xp = x.clone().requires_grad_(True)
    yp = par(xp)
    yp.backward(gy.clone())
    torch.testing.assert_close(yp, ref(x), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(xp.grad, xr.grad, rtol=1e-5, atol=1e-6)
    a, b = par.up.shard_start, par.up.shard_start + par.up.shard_size
    torch.testing.assert_close(par.up.weight.grad, up.weight.grad[a:b], rtol=1e-5, atol=1e-6)
    a, b = par.down.shard_start, par.down.shard_start + par.down.shard_size
    torch.testing.assert_close(par.down.weight.grad, down.weight.grad[:, a:b], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(par.down.bias.grad, down.bias.grad, rtol=1e-5, atol=1e-6)


def test_parallel_mlp_matches_reference_world2() -> None:
    run(_mlp, 2)


def test_parallel_mlp_matches_reference_world4() -> None:
    run(_mlp, 4)


class RefAttention(nn.Module):
    def __init__(self, width: int, n_head: int) -> None:
        super().__init__()
        torch.manual_seed(7)
        self.n_head, self.hd = n_head, width // n_head
        self.qkv = nn.Linear(width, 3 * width)
        self.proj = nn.Linear(width, width)

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = (t.view(B, T, self.n_head, self.hd).transpose(1, 2) for t in self.qkv(x).split(C, -1))
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.proj(y.transpose(1, 2).reshape(B, T, C))


def _attention(pg, sequence_parallel: bool = False) -> None:
    n_head, T = 4, 8
    ref = RefAttention(WIDTH, n_head)
    par = ParallelSelfAttention(WIDTH, n_head, pg, sequence_parallel=sequence_parallel)
    par.qkv.load_full_weight(ref.qkv.weight.detach(), ref.qkv.bias.detach())
    par.proj.load_full_weight(ref.proj.weight.detach(), ref.proj.bias.detach())
    assert par.local_heads == n_head // pg.world_size
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, T, WIDTH, generator=g)
    gy = torch.randn(2, T, WIDTH, generator=g)
    xr = x.clone().requires_grad_(True)
    yr = ref(xr)
    yr.backward(gy)
    if sequence_parallel:
        # sequence-major layout, each rank holding a contiguous run of tokens
        W, r = pg.world_size, pg.rank
        per = T // W
        xs = x.transpose(0, 1)[r * per : (r + 1) * per].contiguous().requires_grad_(True)
        ys = par(xs)
        ys.backward(gy.transpose(0, 1)[r * per : (r + 1) * per].contiguous())
        torch.testing.assert_close(ys, yr.detach().transpose(0, 1)[r * per : (r + 1) * per], rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(xs.grad, xr.grad.transpose(0, 1)[r * per : (r + 1) * per], rtol=1e-4, atol=1e-5)
    else:
        xp = x.clone().requires_grad_(True)
        par(xp).backward(gy.clone())
        torch.testing.assert_close(xp.grad, xr.grad, rtol=1e-4, atol=1e-6)
    rows = _qkv_shard_rows(WIDTH, n_head, WIDTH // n_head, pg)
    torch.testing.assert_close(par.qkv.weight.grad, ref.qkv.weight.grad.index_select(0, rows), rtol=1e-4, atol=1e-5)


def test_parallel_attention_matches_reference() -> None:
    run(_attention, 2)
    run(_attention, 4)


def test_sequence_parallel_attention_matches_reference() -> None:
    run(_attention, 2, True)


def _gather_output(pg) -> None:
    torch.manual_seed(21)
    ref = nn.Linear(WIDTH, 3 * WIDTH)
    nn.init.normal_(ref.weight, std=0.05)
    layer = ColumnParallelLinear(WIDTH, 3 * WIDTH, pg, gather_output=True)
    layer.load_full_weight(ref.weight.detach(), ref.bias.detach())
    g = torch.Generator().manual_seed(13)
    x = torch.randn(BATCH, WIDTH, generator=g)
    gy = torch.randn(BATCH, 3 * WIDTH, generator=g)
    xr = x.clone().requires_grad_(True)
    ref(xr).backward(gy)
    xp = x.clone().requires_grad_(True)
    yp = layer(xp)
    yp.backward(gy.clone())
    torch.testing.assert_close(yp, ref(x), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(xp.grad, xr.grad, rtol=1e-5, atol=1e-6)


def test_column_parallel_gather_output() -> None:
    run(_gather_output, 4)


def _drift(pg, steps: int = 8) -> None:
    """Replicated params beside TP layers must stay *bitwise* identical."""
    torch.manual_seed(31)
    norm = nn.LayerNorm(WIDTH)
    mlp = ParallelMLP(WIDTH, pg)
    opt = torch.optim.SGD(list(norm.parameters()) + list(mlp.parameters()), lr=0.1)
    g = torch.Generator().manual_seed(37)
    for _ in range(steps):
        x = torch.randn(BATCH, WIDTH, generator=g)
        opt.zero_grad()
        mlp(norm(x)).square().mean().backward()
        opt.step()
    for name, p in norm.named_parameters():
        got = collectives.all_gather(pg, p.detach())
        for r, other in enumerate(got):
            assert torch.equal(other, got[0]), f"replicated {name} diverged on rank {r}"


def test_replicated_layers_stay_bitwise_identical() -> None:
    run(_drift, 4)


def _sp_drift(pg, steps: int = 6) -> None:
    """Sequence parallel: LayerNorm and row bias see only local tokens; after
    ``allreduce_sequence_parallel_grads`` they match the unsharded gradients and
    stay bitwise identical across ranks."""
    from mini_nccl_b200.tensor_parallel import (
        allreduce_sequence_parallel_grads, gather_from_sequence_parallel, mark_sequence_parallel,
        scatter_to_sequence_parallel)

    torch.manual_seed(41)
    norm = nn.LayerNorm(WIDTH)
    mlp = ParallelMLP(WIDTH, pg, sequence_parallel=True)
    mark_sequence_parallel(norm)
    params = list(norm.parameters()) + list(mlp.parameters())
    opt = torch.optim.SGD(params, lr=0.1)
    g = torch.Generator().manual_seed(43)
    T = 4 * pg.world_size
    for _ in range(steps):
        x = torch.randn(T, 2, WIDTH, generator=g)  # sequence-major, replicated
        opt.zero_grad()
        xs = scatter_to_sequence_parallel(pg, x)
        y = gather_from_sequence_parallel(pg, mlp(norm(xs), residual=xs))
        y.square().mean().backward()
        allreduce_sequence_parallel_grads(norm, pg)
        allreduce_sequence_parallel_grads(mlp, pg)
        opt.step()
    for name, p_ in list(norm.named_parameters()) + [("mlp.down.bias", mlp.down.bias)]:
        got = collectives.all_gather(pg, p_.detach())
        for r, other in enumerate(got):
            assert torch.equal(other, got[0]), f"replicated {name} diverged on rank {r}"


def test_sequence_parallel_replicated_params_stay_identical() -> None:
    run(_sp_drift, 2)


def _sp_grads_match(pg) -> None:
    """SP MLP block gradients (incl. the replicated bias and LN) equal a single process."""
    from mini_nccl_b200.tensor_parallel import (
        allreduce_sequence_parallel_grads, gather_from_sequence_parallel, mark_sequence_parallel,
        scatter_to_sequence_parallel)

    torch.manual_seed(51)
    ref_norm, ref_up, ref_down = nn.LayerNorm(WIDTH), nn.Linear(WIDTH, 4 * WIDTH), nn.Linear(4 * WIDTH, WIDTH)
    norm = nn.LayerNorm(WIDTH)
    norm.load_state_dict(ref_norm.state_dict())
    mlp = ParallelMLP(WIDTH, pg, sequence_parallel=True)
    mlp.up.load_full_weight(ref_up.weight.detach(), ref_up.bias.detach())
    mlp.down.load_full_weight(ref_down.weight.detach(), ref_down.bias.detach())
    mark_sequence_parallel(norm)
    T = 3 * pg.world_size
    x = torch.randn(T, 2, WIDTH, generator=torch.Generator().manual_seed(53))
    xr = x.clone().requires_grad_(True)
    h = ref_norm(xr)
    (xr + ref_down(F.gelu(ref_up(h)))).square().mean().backward()
    xp = x.clone().requires_grad_(True)
    xs = scatter_to_sequence_parallel(pg, xp)
    gather_from_sequence_parallel(pg, mlp(norm(xs), residual=xs)).square().mean().backward()
    allreduce_sequence_parallel_grads(norm, pg)
    allreduce_sequence_parallel_grads(mlp, pg)
    torch.testing.assert_close(xp.grad, xr.grad, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(norm.weight.grad, ref_norm.weight.grad, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(mlp.down.bias.grad, ref_down.bias.grad, rtol=1e-4, atol=1e-6)
    s0, n = mlp.up.shard_start, mlp.up.shard_size
    torch.testing.assert_close(mlp.up.weight.grad, ref_up.weight.grad[s0 : s0 + n], rtol=1e-4, atol=1e-6)


def test_sequence_parallel_grads_match_single_process() -> None:
    run(_sp_grads_match, 2)


def _unsharded_input(pg) -> None:
    torch.manual_seed(23)
    ref = nn.Linear(4 * WIDTH, WIDTH)
    layer = RowParallelLinear(4 * WIDTH, WIDTH, pg, input_is_sharded=False)
    layer.load_full_weight(ref.weight.detach(), ref.bias.detach())
    x = torch.randn(BATCH, 4 * WIDTH, generator=torch.Generator().manual_seed(17))
    torch.testing.assert_close(layer(x), ref(x), rtol=1e-5, atol=1e-6)


def test_row_parallel_unsharded_input() -> None:
    run(_unsharded_input, 2)


def test_qkv_rows_cover_each_third() -> None:
    class G:
        world_size, rank = 2, 1

    rows = _qkv_shard_rows(8, 4, 2, G())
    assert rows.tolist() == [4, 5, 6, 7, 12, 13, 14, 15, 20, 21, 22, 23]
