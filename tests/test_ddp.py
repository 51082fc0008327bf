"""Data parallelism on CPU ranks: gradients and training equal one process.

Scenarios are this library's own:

* the char-level GPT of the CPU configuration (vocab 65, context 64, 4 layers,
  4 heads, width 128, pre-LayerNorm, tied head; 16 sequences per rank, AdamW
  lr 3e-4): for 100 steps the averaged gradients of two ranks equal the
  gradients one process computes on both ranks' data, to 1e-5;
* a small tied-embedding language model trained with Nesterov SGD and weight
  decay under several bucket layouts, overlap on and off, at 2 and 3 ranks;
* accumulation over three microbatches with ``no_sync``;
* buckets that split at a dtype change;
* rank 0's parameters and buffers reach every rank at construction.
"""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from mini_nccl_b200.ddp import DistributedDataParallel, average_gradients
from mini_nccl_b200.launcher import run
from mini_nccl_b200.models.gpt import GPT


def _char_gpt_gradients(pg, steps: int = 100) -> float:
    W, per_rank, T, V = pg.world_size, 16, 64, 65
    torch.manual_seed(0)
    model = GPT(vocab_size=V, block_size=T, n_layer=4, n_head=4, n_embd=128)
    whole = copy.deepcopy(model)
    ddp = DistributedDataParallel(model, pg, bucket_cap_mb=0.25)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    data = torch.Generator().manual_seed(0)
    worst = 0.0
    for _ in range(steps):
        tokens = torch.randint(0, V, (W * per_rank, T + 1), generator=data)
        x, y = tokens[:, :-1], tokens[:, 1:]
        mine = slice(pg.rank * per_rank, (pg.rank + 1) * per_rank)
        ddp.zero_grad()
        _, loss = ddp(x[mine], y[mine])
        loss.backward()
        ddp.sync()
        # One process, same parameters, every rank's sequences.
        with torch.no_grad():
            for p, q in zip(whole.parameters(), model.parameters(), strict=True):
                p.copy_(q)
        whole.zero_grad(set_to_none=True)
        whole(x, y)[1].backward()
        for (name, p), q in zip(model.named_parameters(), whole.parameters(), strict=True):
            diff = (p.grad - q.grad).abs().max().item()
            assert diff <= 1e-5, f"{name}: gradient differs by {diff:.3e}"
            worst = max(worst, diff)
        opt.step()
    return worst


def test_char_gpt_gradients_match_one_process_for_100_adamw_steps() -> None:
    worst = run(_char_gpt_gradients, 2, timeout=600.0)
    print(f"largest gradient difference over 100 steps: {max(worst):.2e}")


class TiedLM(nn.Module):
    """Embedding -> LayerNorm -> MLP -> LayerNorm -> head tied to the embedding."""

    def __init__(self, vocab: int = 37, width: int = 20) -> None:
        super().__init__()
        self.emb = nn.Embedding(vocab, width)
        self.ln1 = nn.LayerNorm(width)
        self.up = nn.Linear(width, 3 * width)
        self.down = nn.Linear(3 * width, width)
        self.ln2 = nn.LayerNorm(width)
        self.head = nn.Linear(width, vocab, bias=False)
        self.head.weight = self.emb.weight

    def forward(self, idx: torch.Tensor) -> torch.Tensor:
        h = self.emb(idx)
        h = h + self.down(F.gelu(self.up(self.ln1(h))))
        return self.head(self.ln2(h))


def _lm_loss(model, idx, tgt) -> torch.Tensor:
    logits = model(idx)
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1))


def _train_like_one_process(pg, overlap: bool, cap_mb: float, steps: int = 5) -> int:
    W, per_rank, T = pg.world_size, 3, 9
    torch.manual_seed(31)
    model = TiedLM()
    whole = copy.deepcopy(model)
    ddp = DistributedDataParallel(model, pg, bucket_cap_mb=cap_mb, overlap=overlap)
    sgd = dict(lr=0.05, momentum=0.8, nesterov=True, weight_decay=1e-2)
    opt = torch.optim.SGD(model.parameters(), **sgd)
    whole_opt = torch.optim.SGD(whole.parameters(), **sgd)
    data = torch.Generator().manual_seed(1234 + W)
    for _ in range(steps):
        idx = torch.randint(0, 37, (W * per_rank, T), generator=data)
        tgt = torch.randint(0, 37, (W * per_rank, T), generator=data)
        mine = slice(pg.rank * per_rank, (pg.rank + 1) * per_rank)
        ddp.zero_grad()
        _lm_loss(ddp, idx[mine], tgt[mine]).backward()
        ddp.sync()
        opt.step()
        whole_opt.zero_grad()
        _lm_loss(whole, idx, tgt).backward()
        whole_opt.step()
    for (name, p), q in zip(model.named_parameters(), whole.parameters(), strict=True):
        torch.testing.assert_close(p, q, rtol=2e-5, atol=2e-6, msg=lambda m, n=name: f"{n}: {m}")
    return len(ddp._buckets)


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("overlap,cap_mb", [(True, 4.0), (False, 4.0), (True, 0.002)])
def test_tied_lm_trains_like_one_process(world, overlap, cap_mb) -> None:
    buckets = run(_train_like_one_process, world, overlap, cap_mb)[0]
    assert (buckets == 1) if cap_mb > 1 else (buckets >= 4), buckets


def _accumulate_three_microbatches(pg) -> None:
    W, micro, T = pg.world_size, 2, 7
    torch.manual_seed(8)
    model = TiedLM(vocab=23, width=12)
    whole = copy.deepcopy(model)
    ddp = DistributedDataParallel(model, pg, bucket_cap_mb=0.001)
    pg.recorder.enabled = True
    data = torch.Generator().manual_seed(77)
    idx = torch.randint(0, 23, (W, 3, micro, T), generator=data)
    tgt = torch.randint(0, 23, (W, 3, micro, T), generator=data)
    sent_before = pg.recorder.peek_seq(-1)
    ddp.zero_grad()
    with ddp.no_sync():
        for k in range(2):
            (_lm_loss(ddp, idx[pg.rank, k], tgt[pg.rank, k]) / 3).backward()
    assert pg.recorder.peek_seq(-1) == sent_before, "no_sync must not communicate"
    (_lm_loss(ddp, idx[pg.rank, 2], tgt[pg.rank, 2]) / 3).backward()
    ddp.sync()
    _lm_loss(whole, idx.reshape(-1, T), tgt.reshape(-1, T)).backward()  # a mean over every token
    for p, q in zip(model.parameters(), whole.parameters(), strict=True):
        torch.testing.assert_close(p.grad, q.grad, rtol=1e-5, atol=1e-6)


def test_no_sync_accumulates_three_microbatches() -> None:
    run(_accumulate_three_microbatches, 2)


class MixedPrecisionHead(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.body = nn.Linear(6, 6)
        self.head = nn.Linear(6, 2).double()

    def forward(self, x):
        return self.head(torch.tanh(self.body(x)).double())


def _dtype_breaks_bucket(pg) -> list[str]:
    torch.manual_seed(2)
    ddp = DistributedDataParallel(MixedPrecisionHead(), pg, bucket_cap_mb=100.0)
    ddp.zero_grad()
    ddp(torch.randn(4, 6)).sum().backward()
    ddp.sync()
    for b in ddp._buckets:
        assert {p.dtype for p in b.params} == {b.buffer.dtype}
        for p in b.params:
            assert p.grad.untyped_storage().data_ptr() == b.buffer.untyped_storage().data_ptr()
    return [str(b.buffer.dtype) for b in ddp._buckets]


def test_a_dtype_change_starts_a_new_bucket() -> None:
    # reverse registration order: the float64 head first, then the float32 body
    assert run(_dtype_breaks_bucket, 2)[0] == ["torch.float64", "torch.float32"]


class WithBuffer(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.lin = nn.Linear(5, 3)
        self.norm = nn.BatchNorm1d(3)


def _rank0_state_everywhere(pg) -> None:
    torch.manual_seed(500 + 17 * pg.rank)
    m = WithBuffer()
    m.norm.running_mean.fill_(float(pg.rank + 1))
    DistributedDataParallel(m, pg)
    torch.manual_seed(500)
    want = WithBuffer()
    torch.testing.assert_close(m.lin.weight, want.lin.weight, rtol=0, atol=0)
    torch.testing.assert_close(m.lin.bias, want.lin.bias, rtol=0, atol=0)
    assert torch.all(m.norm.running_mean == 1.0)


def test_construction_copies_rank0_parameters_and_buffers() -> None:
    run(_rank0_state_everywhere, 3)


def _average_mixed_shapes(pg) -> int:
    ps = [nn.Parameter(torch.zeros(5)), nn.Parameter(torch.zeros(2, 3)), nn.Parameter(torch.zeros(1))]
    for i, p in enumerate(ps):
        p.grad = torch.arange(p.numel(), dtype=torch.float32).view(p.shape) * (pg.rank + 1) + i
    frozen = nn.Parameter(torch.zeros(4))  # no gradient: skipped, not an error
    n = average_gradients(pg, ps + [frozen])
    mean_factor = sum(r + 1 for r in range(pg.world_size)) / pg.world_size
    for i, p in enumerate(ps):
        want = torch.arange(p.numel(), dtype=torch.float32).view(p.shape) * mean_factor + i
        torch.testing.assert_close(p.grad, want)
    assert frozen.grad is None
    return n


def test_average_gradients_skips_missing_grads() -> None:
    assert run(_average_mixed_shapes, 3)[0] == 12 * 4
