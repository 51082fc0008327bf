"""Data x pipeline x tensor parallelism at once, against one process.

Eight CPU ranks as a 2 (dp) x 2 (pp) x 2 (tp) mesh: each rank holds one
pipeline stage, one tensor-parallel shard of that stage's blocks, and belongs
to one of two data-parallel replicas.  The gradients of every parameter slice
must equal the single-process gradients of the whole model on the whole
batch.  Two rules this pins (reference behaviour: tests/test_three_dimensional.py:
120-249): gradients are averaged along dp only, and after the pipeline has
drained (``average_gradients``), never per microbatch.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200.ddp import average_gradients
from mini_nccl_b200.launcher import run
from mini_nccl_b200.mesh import ParallelMesh
from mini_nccl_b200.pipeline import PipelineParallel
from mini_nccl_b200.tensor_parallel import ColumnParallelLinear, RowParallelLinear

C = 8            # width
HID = 16         # MLP hidden width
PER_REPLICA = 4  # samples per data-parallel replica per step
MICRO = 2        # microbatches


class Block(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(C)
        self.up = nn.Linear(C, HID)
        self.down = nn.Linear(HID, C)

    def forward(self, x):
        return x + self.down(F.gelu(self.up(self.norm(x))))


class Whole(nn.Module):
    """in-projection -> block -> block -> out-projection."""

    def __init__(self) -> None:
        super().__init__()
        torch.manual_seed(77)
        self.inp = nn.Linear(C, C)
        self.b0 = Block()
        self.b1 = Block()
        self.out = nn.Linear(C, 1)

    def forward(self, x):
        return self.out(self.b1(self.b0(self.inp(x))))


class TPBlock(nn.Module):
    """``Block`` with the MLP split over the tp group (column up, row down)."""

    def __init__(self, ref: Block, tp) -> None:
        super().__init__()
        self.norm = nn.LayerNorm(C)
        self.norm.load_state_dict(ref.norm.state_dict())
        self.up = ColumnParallelLinear(C, HID, tp)
        self.down = RowParallelLinear(HID, C, tp)
        self.up.load_full_weight(ref.up.weight.detach(), ref.up.bias.detach())
        self.down.load_full_weight(ref.down.weight.detach(), ref.down.bias.detach())

    def forward(self, x):
        return x + self.down(F.gelu(self.up(self.norm(x))))


def _stage(ref: Whole, stage: int, tp) -> nn.Module:
    if stage == 0:
        inp = nn.Linear(C, C)
        inp.load_state_dict(ref.inp.state_dict())
        return nn.Sequential(inp, TPBlock(ref.b0, tp))
    out = nn.Linear(C, 1)
    out.load_state_dict(ref.out.state_dict())
    return nn.Sequential(TPBlock(ref.b1, tp), out)


def _data():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2 * PER_REPLICA, C, generator=g)
    y = torch.randn(2 * PER_REPLICA, 1, generator=g)
    return x, y


def _reference_grads() -> dict[str, torch.Tensor]:
    ref = Whole()
    x, y = _data()
    F.mse_loss(ref(x), y).backward()
    return {n: p.grad.clone() for n, p in ref.named_parameters()}


def _worker(pg):
    mesh = ParallelMesh(pg, dp=2, pp=2, tp=2)
    dp, pp, tp = mesh.group("dp"), mesh.group("pp"), mesh.group("tp")
    d, s, t = mesh.coordinate("dp"), mesh.coordinate("pp"), mesh.coordinate("tp")
    ref = Whole()
    stage = _stage(ref, s, tp)
    pipe = PipelineParallel(stage, pp, activation_shape=(PER_REPLICA // MICRO, C),
                            loss_fn=lambda out, tgt: F.mse_loss(out, tgt))
    x, y = _data()
    xs, ys = x[d * PER_REPLICA : (d + 1) * PER_REPLICA], y[d * PER_REPLICA : (d + 1) * PER_REPLICA]
    pipe.step(xs if s == 0 else None, ys if s == 1 else None, n_microbatches=MICRO)
    average_gradients(dp, list(stage.parameters()))
    want = _reference_grads()
    blk = "b0" if s == 0 else "b1"
    tpb = stage[1] if s == 0 else stage[0]
    a, n = tpb.up.shard_start, tpb.up.shard_size
    checks = {
        f"{blk}.up.weight": (tpb.up.weight.grad, want[f"{blk}.up.weight"][a : a + n]),
        f"{blk}.up.bias": (tpb.up.bias.grad, want[f"{blk}.up.bias"][a : a + n]),
        f"{blk}.down.weight": (tpb.down.weight.grad, want[f"{blk}.down.weight"][:, a : a + n]),
        f"{blk}.down.bias": (tpb.down.bias.grad, want[f"{blk}.down.bias"]),
        f"{blk}.norm.weight": (tpb.norm.weight.grad, want[f"{blk}.norm.weight"]),
    }
    if s == 0:
        checks["inp.weight"] = (stage[0].weight.grad, want["inp.weight"])
    else:
        checks["out.weight"] = (stage[1].weight.grad, want["out.weight"])
    for name, (got, exp) in checks.items():
        torch.testing.assert_close(got, exp, rtol=1e-4, atol=1e-6, msg=lambda m, name=name: f"{name}: {m}")
    return (d, s, t)


def test_three_dimensional_matches_single_process() -> None:
    coords = run(_worker, 8, timeout=300.0)
    assert sorted(coords) == [(d, s, t) for d in range(2) for s in range(2) for t in range(2)]


def _degenerate(pg):
    """dp=4 x pp=1 x tp=1 is plain data parallelism."""
    mesh = ParallelMesh(pg, dp=4, pp=1, tp=1)
    assert mesh.size("pp") == 1 and mesh.size("tp") == 1
    assert mesh.group("dp").world_size == 4
    torch.manual_seed(3)
    model = nn.Linear(C, 1)
    g = torch.Generator().manual_seed(9)
    x, y = torch.randn(8, C, generator=g), torch.randn(8, 1, generator=g)
    r = mesh.coordinate("dp")
    F.mse_loss(model(x[2 * r : 2 * r + 2]), y[2 * r : 2 * r + 2]).backward()
    average_gradients(mesh.group("dp"), list(model.parameters()))
    ref = nn.Linear(C, 1)
    ref.load_state_dict(model.state_dict())
    ref.zero_grad()
    F.mse_loss(ref(x), y).backward()
    torch.testing.assert_close(model.weight.grad, ref.weight.grad, rtol=1e-5, atol=1e-7)
    return True


def test_degenerate_dimensions_reduce_to_data_parallel() -> None:
    run(_degenerate, 4, timeout=120.0)


def _gpt_3d(pg):
    """GPTStage (TP + SP blocks, 1F1B pipeline, DP replicas) == one process, same weights."""
    import types

    from mini_nccl_b200.models.tp_gpt import GPTStage, sync_tensor_parallel_grads

    V, T, L, H, Cw = 37, 8, 2, 4, 16
    mesh = ParallelMesh(pg, dp=2, pp=2, tp=2)
    dp, pp, tp = mesh.group("dp"), mesh.group("pp"), mesh.group("tp")
    d, s = mesh.coordinate("dp"), mesh.coordinate("pp")
    torch.manual_seed(123)
    solo = types.SimpleNamespace(world_size=1, rank=0)
    ref = GPTStage(V, T, L, H, Cw, solo, 0, 1, sequence_parallel=False)
    stage = GPTStage(V, T, L, H, Cw, tp, s, 2, sequence_parallel=True)
    per = L // 2
    with torch.no_grad():
        if s == 0:
            stage.tok_emb.weight.copy_(ref.tok_emb.weight)
            stage.pos_emb.copy_(ref.pos_emb)
        else:
            stage.ln_f.load_state_dict(ref.ln_f.state_dict())
            stage.head.weight.copy_(ref.head.weight)
        for j, blk in enumerate(stage.blocks):
            rb = ref.blocks[s * per + j]
            blk.ln1.load_state_dict(rb.ln1.state_dict())
            blk.ln2.load_state_dict(rb.ln2.state_dict())
            blk.attn.qkv.load_full_weight(rb.attn.qkv.weight, rb.attn.qkv.bias)
            blk.attn.proj.load_full_weight(rb.attn.proj.weight, rb.attn.proj.bias)
            blk.mlp.up.load_full_weight(rb.mlp.up.weight, rb.mlp.up.bias)
            blk.mlp.down.load_full_weight(rb.mlp.down.weight, rb.mlp.down.bias)
    g = torch.Generator().manual_seed(7)
    idx = torch.randint(0, V, (8, T), generator=g)  # 2 replicas x 2 microbatches x 2 sequences
    tgt = torch.randint(0, V, (8, T), generator=g)
    # reference: the whole batch at once
    ref.loss(ref(idx), tgt).backward()
    # 3D: this replica's half, two microbatches through the pipeline
    pipe = PipelineParallel(stage, pp, activation_shape=(T // 2, 2, Cw), loss_fn=stage.loss if s == 1 else None)
    mine = slice(4 * d, 4 * d + 4)
    pipe.step(idx[mine] if s == 0 else None, tgt[mine] if s == 1 else None, n_microbatches=2)
    sync_tensor_parallel_grads(stage, tp)
    average_gradients(dp, list(stage.parameters()))
    close = dict(rtol=2e-4, atol=2e-6)
    if s == 0:
        torch.testing.assert_close(stage.tok_emb.weight.grad, ref.tok_emb.weight.grad, **close)
    else:
        torch.testing.assert_close(stage.head.weight.grad, ref.head.weight.grad, **close)
        torch.testing.assert_close(stage.ln_f.weight.grad, ref.ln_f.weight.grad, **close)
    for j, blk in enumerate(stage.blocks):
        rb = ref.blocks[s * per + j]
        torch.testing.assert_close(blk.ln1.weight.grad, rb.ln1.weight.grad, **close)
        torch.testing.assert_close(blk.attn.proj.bias.grad, rb.attn.proj.bias.grad, **close)
        a, n = blk.mlp.up.shard_start, blk.mlp.up.shard_size
        torch.testing.assert_close(blk.mlp.up.weight.grad, rb.mlp.up.weight.grad[a : a + n], **close)
        rows = blk.attn.qkv.shard_rows
        torch.testing.assert_close(blk.attn.qkv.weight.grad, rb.attn.qkv.weight.grad.index_select(0, rows), **close)
    return True


def test_gpt_stage_3d_matches_single_process() -> None:
    run(_gpt_3d, 8, timeout=300.0)
