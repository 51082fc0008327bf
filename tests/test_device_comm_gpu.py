"""Device (peer-memory) collectives across real GPUs, one process per GPU.

Every rank recomputes every rank's input from seeds and checks the exact
expected result, as the host battery does.  Needs >= 2 GPUs; on a 1-GPU box
these tests skip (kernels that wait on each other never share one GPU).
"""

from __future__ import annotations

import os

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

from mini_nccl_b200 import collectives as C  # noqa: E402
from mini_nccl_b200.launcher import run  # noqa: E402


def n_gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


needs2 = pytest.mark.skipif(n_gpus() < 2, reason="needs at least 2 GPUs")


def seeded(rank: int, numel: int, dtype: torch.dtype, dev) -> torch.Tensor:
    g = torch.Generator().manual_seed(9000 + rank)
    if dtype.is_floating_point:
        return torch.randn(numel, generator=g).to(dtype).to(dev)
    return torch.randint(-40, 40, (numel,), generator=g, dtype=dtype).to(dev)


def expected(world: int, numel: int, dtype, op: str, dev) -> torch.Tensor:
    parts = [seeded(r, numel, dtype, "cpu").double() if dtype.is_floating_point else seeded(r, numel, dtype, "cpu")
             for r in range(world)]
    out = parts[0].clone()
    for p in parts[1:]:
        out = {"sum": out + p, "prod": out * p, "max": torch.maximum(out, p), "min": torch.minimum(out, p)}[op]
    return out.to(dev)


def _battery(pg) -> None:
    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = pg.world_size, pg.rank
    tol = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.int64: 0}
    for algorithm in ("one_shot", "two_shot", "ring", "tree", "halving", "naive"):
        for dtype in (torch.float32, torch.bfloat16, torch.int64):
            for op in ("sum", "max", "min"):
                for numel in (1, 3, 1000, 262_147):
                    t = seeded(r, numel, dtype, dev)
                    C.all_reduce(pg, t, op=op, algorithm=algorithm)
                    want = expected(W, numel, dtype, op, dev)
                    if dtype == torch.int64:
                        assert torch.equal(t, want), (algorithm, op, numel)
                    else:
                        err = (t.double() - want).abs().max().item()
                        assert err <= tol[dtype] * (want.abs().max().item() + 1), (algorithm, dtype, op, numel, err)
    # identical bits on every rank (fixed reduction order)
    t = seeded(r, 4096, torch.float32, dev)
    C.all_reduce(pg, t, algorithm="two_shot")
    everyone = C.all_gather(pg, t)
    for other in everyone:
        assert torch.equal(other, everyone[0])
    # scale fused into the kernel (DDP averaging) and symmetric in-place path
    dc = pg.device_comm()
    sym = dc.symmetric_zeros(1 << 20, torch.bfloat16)
    sym.copy_(seeded(r, 1 << 20, torch.bfloat16, dev))
    dc.all_reduce(sym, algorithm="two_shot", scale=1.0 / W)
    want = expected(W, 1 << 20, torch.bfloat16, "sum", dev) / W
    assert (sym.double() - want).abs().max().item() < 3e-2
    # the small-CTA variant DDP runs beside the backward pass: same results
    sym.copy_(seeded(r, 1 << 20, torch.bfloat16, dev))
    dc.all_reduce(sym, algorithm="two_shot", scale=1.0 / W, beside_compute=True)
    assert (sym.double() - want).abs().max().item() < 3e-2
    for dtype, wire in ((torch.float32, None), (torch.float32, torch.bfloat16), (torch.bfloat16, None)):
        t = seeded(r, 300_017, dtype, dev)
        dc.all_reduce(t, algorithm="two_shot", wire_dtype=wire, beside_compute=True)
        assert (t.double() - expected(W, 300_017, dtype, "sum", dev)).abs().max().item() < 0.05
        everyone = C.all_gather(pg, t)
        assert all(torch.equal(o, everyone[0]) for o in everyone)
    # narrow wire: fp32 tensor, bf16 on the wire, fp32 accumulation
    t = seeded(r, 100_003, torch.float32, dev)
    C.all_reduce(pg, t, algorithm="two_shot", wire_dtype=torch.bfloat16)
    want = expected(W, 100_003, torch.float32, "sum", dev)
    assert (t.double() - want).abs().max().item() < 0.05
    # broadcast from every root (odd byte count and a 16-byte-multiple one)
    for src in range(W):
        t = seeded(r, 4097, torch.float32, dev)
        C.broadcast(pg, t, src=src)
        assert torch.equal(t, seeded(src, 4097, torch.float32, dev))
        t = seeded(r, (1 << 20) + 24, torch.bfloat16, dev)
        C.broadcast(pg, t, src=src)
        assert torch.equal(t, seeded(src, (1 << 20) + 24, torch.bfloat16, dev))
    # all_gather in rank order
    t = seeded(r, 6 * 13, torch.bfloat16, dev).view(6, 13)
    got = C.all_gather(pg, t)
    for i, g in enumerate(got):
        assert torch.equal(g, seeded(i, 6 * 13, torch.bfloat16, dev).view(6, 13))
    # reduce_scatter: my chunk of the sum, input untouched
    n = 1000 * W
    t = seeded(r, n, torch.float32, dev)
    before = t.clone()
    mine = C.reduce_scatter(pg, t)
    want = expected(W, n, torch.float32, "sum", dev).view(W, -1)[r]
    assert (mine.double() - want).abs().max().item() < 1e-4
    assert torch.equal(t, before)
    # all_to_all
    n = 9 * W
    out = C.all_to_all(pg, seeded(r, n, torch.float32, dev))
    for src in range(W):
        assert torch.equal(out.view(W, -1)[src], seeded(src, n, torch.float32, dev).view(W, -1)[r])
    # large message through a grown staging buffer
    big = seeded(r, 40 << 20, torch.bfloat16, dev)  # 80 MB > initial staging
    C.all_reduce(pg, big)
    C.barrier(pg)
    dc.synchronize()


@needs2
def test_device_collective_battery():
    run(_battery, 2, devices="cuda", timeout=600.0, op_timeout=60.0)


def _ddp_parity(pg) -> None:
    import copy

    import torch.nn.functional as F
    from torch import nn

    from mini_nccl_b200.ddp import DistributedDataParallel

    dev = torch.device("cuda", torch.cuda.current_device())
    W, per = pg.world_size, 8
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(16, 64), nn.Tanh(), nn.Linear(64, 1)).to(dev)
    ref = copy.deepcopy(model)
    ddp = DistributedDataParallel(model, pg, bucket_cap_mb=0.001)
    assert len(ddp._buckets) > 1
    opt = torch.optim.SGD(model.parameters(), lr=0.1, momentum=0.9)
    ropt = torch.optim.SGD(ref.parameters(), lr=0.1, momentum=0.9)
    gen = torch.Generator().manual_seed(42)
    for _ in range(5):
        x = torch.randn(W * per, 16, generator=gen).to(dev)
        y = torch.randn(W * per, 1, generator=gen).to(dev)
        mine = slice(pg.rank * per, (pg.rank + 1) * per)
        ddp.zero_grad()
        F.mse_loss(ddp(x[mine]), y[mine]).backward()
        ddp.sync()
        opt.step()
        ropt.zero_grad()
        F.mse_loss(ref(x), y).backward()
        ropt.step()
    for p, q in zip(model.parameters(), ref.parameters()):
        torch.testing.assert_close(p, q, rtol=1e-4, atol=1e-5)


@needs2
def test_ddp_on_gpus_matches_single_process():
    run(_ddp_parity, 2, devices="cuda", timeout=600.0, op_timeout=60.0)


def _timeout(pg) -> str:
    """Rank 1 never launches its half: rank 0's kernel must time out cleanly."""
    from mini_nccl_b200.errors import CollectiveTimeoutError

    dev = torch.device("cuda", torch.cuda.current_device())
    dc = pg.device_comm()
    dc.set_timeout(1.0)
    C.barrier(pg)  # host barrier: both communicators exist
    if pg.rank == 1:
        C.barrier(pg)  # wait (on the host) until rank 0 has seen its error
        return "withheld"
    t = torch.ones(1024, device=dev)
    dc.all_reduce(t, algorithm="one_shot")
    try:
        dc.synchronize()
    except CollectiveTimeoutError as exc:
        assert "timed out waiting for rank 1" in str(exc)
        outcome = "timeout"
    else:
        outcome = "no error"
    # the context must still work afterwards
    x = torch.arange(10.0, device=dev)
    assert float(x.sum()) == 45.0
    C.barrier(pg)
    return outcome


@needs2
def test_device_wait_times_out_without_hanging(monkeypatch):
    # No multicast objects in a failure test: a rank that leaves while its
    # memory is bound to one can fault the other GPUs.
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    monkeypatch.setenv("MINI_NCCL_NVLS", "0")
    results = run(_timeout, 2, devices="cuda", timeout=300.0, op_timeout=60.0)
    assert results[0] == "timeout", results


def _nvls_battery(pg) -> str:
    """Every NVLS collective against values each rank recomputes from seeds."""
    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = pg.world_size, pg.rank
    dc = pg.device_comm()
    if not dc.nvls:
        return "unavailable: " + dc.nvls_reason
    tol = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-3}
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        for numel in (1, 3, 1000, 262_147, (3 << 20) + 5):
            t = seeded(r, numel, dtype, dev)
            dc.all_reduce(t, algorithm="nvls")
            want = expected(W, numel, dtype, "sum", dev)
            err = (t.double() - want).abs().max().item()
            assert err <= tol[dtype] * (want.abs().max().item() + 1), (dtype, numel, err)
            everyone = C.all_gather(pg, t)  # one reduction per element: identical bits everywhere
            assert all(torch.equal(o, everyone[0]) for o in everyone), (dtype, numel)
    # in place on NVLS memory (DDP's buckets), with the 1/W scale, both CTA shapes
    n = (5 << 20) + 3
    sym = dc.symmetric_zeros(n, torch.bfloat16, nvls=True)
    assert dc.impl.is_nvls(sym)
    want = expected(W, n, torch.bfloat16, "sum", dev) / W
    for beside in (False, True):
        sym.copy_(seeded(r, n, torch.bfloat16, dev))
        dc.all_reduce(sym, scale=1.0 / W, beside_compute=beside)  # auto -> nvls
        assert (sym.double() - want).abs().max().item() < 3e-2, beside
    # reduce-scatter through the switch (input untouched, 1/W fused)
    n = (1 << 20) * W
    for dtype in (torch.float32, torch.bfloat16):
        t = seeded(r, n, dtype, dev)
        before = t.clone()
        mine = dc.reduce_scatter(t, scale=1.0 / W)
        want = expected(W, n, dtype, "sum", dev).view(W, -1)[r] / W
        assert (mine.double() - want).abs().max().item() < tol[dtype] * 10, dtype
        assert torch.equal(t, before)
    # all-gather and broadcast by multimem stores
    shard = seeded(r, 1 << 19, torch.bfloat16, dev)
    got = dc.all_gather(shard)
    for i in range(W):
        assert torch.equal(got[i], seeded(i, 1 << 19, torch.bfloat16, dev)), i
    for src in range(W):
        t = seeded(r, 1 << 20, torch.float32, dev)
        dc.broadcast(t, src=src)
        assert torch.equal(t, seeded(src, 1 << 20, torch.float32, dev)), src
    # reduce-scatter fused with AdamW, the summed gradient taken from the switch
    n = (1 << 19) * W
    grad = seeded(r, n, torch.bfloat16, dev)
    w0 = seeded(100 + r, n // W, torch.float32, dev)
    param = w0.to(torch.bfloat16)
    state = {"m": torch.zeros(n // W, device=dev), "v": torch.zeros(n // W, device=dev), "master": w0.clone()}
    lr, b1, b2, eps, wd = 1e-2, 0.9, 0.95, 1e-8, 0.1
    dc.reduce_scatter_adamw(grad, param, state, lr=lr, betas=(b1, b2), eps=eps, weight_decay=wd, step=1,
                            scale=1.0 / W)
    g = (expected(W, n, torch.bfloat16, "sum", dev).view(W, -1)[r] / W).float()
    m, v = (1 - b1) * g, (1 - b2) * g * g
    w = w0 * (1 - lr * wd) - lr * (m / (1 - b1)) / ((v / (1 - b2)).sqrt() + eps)
    assert (state["master"] - w).abs().max().item() < 1e-4
    # a message larger than the staging buffer grows it (collectively)
    big = seeded(r, 100 << 20, torch.bfloat16, dev)
    C.all_reduce(pg, big)
    want = expected(W, 100 << 20, torch.bfloat16, "sum", dev)
    assert (big.double() - want).abs().max().item() < 0.1
    dc.synchronize()
    return "ok"


@needs2
def test_nvls_collectives_two_ranks():
    out = run(_nvls_battery, 2, devices="cuda", timeout=600.0, op_timeout=60.0)
    if out[0].startswith("unavailable"):
        pytest.skip(out[0])
    assert out == ["ok", "ok"], out


def _gather_weight_gemm(pg) -> None:
    """FSDP's fused gather + first GEMM == a plain all-gather followed by the GEMM."""
    from mini_nccl_b200.ops import kernels as K

    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = pg.world_size, pg.rank
    dc = pg.device_comm()
    for shard_n, w_off, N, Kd, M in ((40_000, 8, 384, 64, 300), (262_144, 4096, 1536, 256, 1024)):
        shard = dc.symmetric_zeros(shard_n, torch.bfloat16)
        shard.copy_(seeded(r, shard_n, torch.bfloat16, dev))
        x = seeded(50 + r, M * Kd, torch.bfloat16, dev).view(M, Kd)
        bias = seeded(77, N, torch.bfloat16, dev)
        flat = torch.full((W * shard_n,), float("nan"), dtype=torch.bfloat16, device=dev)
        for _ in range(2):  # twice: the chunk counters are reset per launch
            out = dc.gather_weight_gemm(x, shard, flat, w_off, N, bias=bias)
        dc.synchronize()
        want_flat = torch.cat([seeded(i, shard_n, torch.bfloat16, dev) for i in range(W)])
        assert torch.equal(flat, want_flat)
        w = want_flat[w_off : w_off + N * Kd].view(N, Kd)
        ref = K.gemm(x, w, bias=bias)
        assert torch.equal(out, ref), (out.float() - ref.float()).abs().max().item()


@needs2
def test_fsdp_gather_weight_gemm_two_ranks():
    run(_gather_weight_gemm, 2, devices="cuda", timeout=300.0, op_timeout=60.0)


def _fsdp_fused_vs_plain(pg) -> None:
    from mini_nccl_b200.fsdp import FullyShardedDataParallel
    from mini_nccl_b200.models.gpt import GPT, Block

    dev = torch.device("cuda", torch.cuda.current_device())
    states = []
    for fused in (False, True):
        torch.manual_seed(0)
        model = GPT(vocab_size=512, block_size=256, n_layer=2, n_head=4, n_embd=256).to(dev, torch.bfloat16)
        fsdp = FullyShardedDataParallel(model, pg, unit_cls=Block, recompute=False, fuse_gather_gemm=fused)
        opt = torch.optim.SGD(fsdp.parameters(), lr=0.5)
        g = torch.Generator().manual_seed(5 + pg.rank)
        losses = []
        for _ in range(2):
            idx = torch.randint(0, 512, (4, 256), generator=g).to(dev)
            tgt = torch.randint(0, 512, (4, 256), generator=g).to(dev)
            fsdp.zero_grad()
            _, loss = fsdp(idx, tgt)
            loss.backward()
            fsdp.sync()
            opt.step()
            losses.append(float(loss))
        states.append((losses, {k: v.float() for k, v in fsdp.full_state_dict().items()}))
    (l0, s0), (l1, s1) = states
    assert abs(l0[0] - l1[0]) < 1e-3 and abs(l0[1] - l1[1]) < 2e-2, (l0, l1)
    for name, v in s0.items():
        err = (v - s1[name]).abs().max().item()
        assert err <= 2e-2 * (v.abs().max().item() + 1e-3), (name, err)


@needs2
def test_fsdp_fused_gather_trains_like_plain_gather():
    run(_fsdp_fused_vs_plain, 2, devices="cuda", timeout=600.0, op_timeout=60.0)


def _ddp_fused_optimizer(pg) -> str:
    """DDP with AdamW inside each bucket's reduction == DDP followed by FusedAdamW."""
    from mini_nccl_b200.ddp import DistributedDataParallel
    from mini_nccl_b200.models.gpt import GPT
    from mini_nccl_b200.ops.kernels import FusedAdamW

    dev = torch.device("cuda", torch.cuda.current_device())
    hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    finals, kinds = [], []
    for fused in (False, True):
        torch.manual_seed(0)
        model = GPT(vocab_size=512, block_size=128, n_layer=2, n_head=4, n_embd=256).to(dev, torch.bfloat16)
        ddp = DistributedDataParallel(model, pg, bucket_cap_mb=1.0, optimizer_in_backward=hp if fused else None)
        opt = None if fused else FusedAdamW(model.parameters(), **hp)
        g = torch.Generator().manual_seed(11 + pg.rank)
        for _ in range(3):
            idx = torch.randint(0, 512, (4, 128), generator=g).to(dev)
            tgt = torch.randint(0, 512, (4, 128), generator=g).to(dev)
            ddp.zero_grad()
            _, loss = ddp(idx, tgt)
            loss.backward()
            ddp.sync()
            if opt is not None:
                opt.step()
        torch.cuda.synchronize()
        kinds.append(pg.device_comm().impl.is_nvls(ddp._buckets[0].buffer))
        finals.append({n: p.detach().float().clone() for n, p in model.named_parameters()})
        if fused:
            assert ddp.unbucketed_parameters() == []
            st = ddp.optimizer_state_dict()
            assert st["step"] == 3 and len(st["buckets"]) == len(ddp._buckets)
    # Adam's first steps move an element by about lr whatever its gradient's size,
    # so a near-zero gradient whose sign flips under bf16 rounding (the fused
    # kernel does not round the reduced gradient to bf16) moves that element by
    # 2 lr: compare whole tensors by relative norm, not element by element.
    # The key third of the QKV bias has an exactly zero gradient (softmax is
    # invariant to a per-row constant), so its Adam steps follow rounding noise
    # and it is left out.
    width = 256
    for name, a in finals[0].items():
        b = finals[1][name]
        if name.endswith("qkv.bias"):
            a, b = torch.cat([a[:width], a[2 * width:]]), torch.cat([b[:width], b[2 * width:]])
        rel = ((a - b).norm() / (a.norm() + 1e-12)).item()
        assert rel <= 2e-2, (name, rel)
    flat = torch.cat([t.reshape(-1) for t in finals[1].values()])
    everyone = C.all_gather(pg, flat)
    assert all(torch.equal(o, everyone[0]) for o in everyone)  # identical replicas
    return "nvls" if kinds[1] else "peer"


@needs2
@pytest.mark.parametrize("nvls", ["1", "0"])
def test_ddp_optimizer_in_backward_matches_separate_optimizer(monkeypatch, nvls):
    monkeypatch.setenv("MINI_NCCL_DDP_NVLS", nvls)
    out = run(_ddp_fused_optimizer, 2, devices="cuda", timeout=600.0, op_timeout=60.0)
    assert out[0] in ("nvls", "peer"), out


def _host_staged(pg) -> None:
    from mini_nccl_b200 import device as D

    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = pg.world_size, pg.rank
    for fn in (lambda t: D.all_reduce_staged(pg, t), lambda t: D.all_reduce_pipelined(pg, t, chunk_bytes=1 << 16)):
        calls = []
        orig = torch.cuda.Stream.wait_stream

        def spy(self, other):
            calls.append(1)
            return orig(self, other)

        torch.cuda.Stream.wait_stream = spy
        try:
            t = torch.full((300_001,), float(r + 1), device=dev)
            fn(t)
        finally:
            torch.cuda.Stream.wait_stream = orig
        torch.cuda.synchronize()
        assert torch.equal(t, torch.full_like(t, W * (W + 1) / 2))
    # the pipelined ring ordered its copy stream behind compute on every exchange
    assert len(calls) >= 2 * (W - 1)


@needs2
def test_host_staged_paths_on_gpus():
    run(_host_staged, 2, timeout=300.0, devices="cuda")


def _fused_tp(pg) -> None:
    """GEMM->reduce-scatter and all-gather->GEMM kernels against fp32 torch."""
    from mini_nccl_b200.ops import kernels as K

    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = pg.world_size, pg.rank
    dc = pg.device_comm()

    def rnd(seed, *shape, scale=1.0):
        g = torch.Generator().manual_seed(seed)
        return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(dev)

    for M, Kd, N in ((2 * 200, 384, 640), (4096, 1024, 1536)):
        # row-parallel: partial sums on every rank, this rank keeps its rows
        for w_mn in (False, True):
            xs = [rnd(100 + q, M, Kd, scale=0.5) for q in range(W)]
            ws = [rnd(200 + q, N, Kd, scale=0.05) for q in range(W)]
            bias = rnd(300, N)
            rows = M // W
            resid = rnd(400 + r, rows, N)
            w_arg = ws[r].t().contiguous() if w_mn else ws[r]
            out = dc.gemm_reduce_scatter(xs[r], w_arg, w_mn=w_mn, bias=bias, resid=resid)
            dc.synchronize()
            K.check_status(dev)
            full = sum(xs[q].float() @ ws[q].float().t() for q in range(W))
            want = full[r * rows:(r + 1) * rows] + bias.float() + resid.float()
            err = (out.float() - want).abs().max().item()
            assert err <= 0.02 * want.abs().max().item() + 0.05, ("rs", M, Kd, N, w_mn, err)
        # column-parallel: gather the rows, multiply by this rank's weight slice
        for w_mn, gelu in ((False, False), (False, True), (True, False)):
            shards = [rnd(500 + q, M // W, Kd, scale=0.5) for q in range(W)]
            w = rnd(600 + r, N, Kd, scale=0.05)
            bias = rnd(700 + r, N)
            aux = torch.empty(M, N, dtype=torch.bfloat16, device=dev) if gelu else None
            out, gathered = dc.all_gather_gemm(shards[r], w.t().contiguous() if w_mn else w, w_mn=w_mn,
                                               bias=bias, gelu_out_aux=aux)
            dc.synchronize()
            K.check_status(dev)
            xfull = torch.cat(shards)
            assert torch.equal(gathered, xfull)
            pre = xfull.float() @ w.float().t() + bias.float()
            want = torch.nn.functional.gelu(pre) if gelu else pre
            err = (out.float() - want).abs().max().item()
            assert err <= 0.02 * want.abs().max().item() + 0.05, ("ag", M, Kd, N, w_mn, gelu, err)
            if gelu:
                assert (aux.float() - pre).abs().max().item() <= 0.02 * pre.abs().max().item() + 0.05
    # many calls in a row (parity halves, epochs) stay correct
    x = rnd(900 + r, 1024, 512, scale=0.5)
    w = rnd(901 + r, 768, 512, scale=0.05)
    ref = None
    for _ in range(6):
        out = dc.gemm_reduce_scatter(x, w)
        if ref is None:
            ref = out.clone()
        assert torch.equal(out, ref)
    dc.synchronize()


@needs2
def test_fused_gemm_collectives_on_gpus():
    run(_fused_tp, 2, timeout=600.0, devices="cuda", op_timeout=60.0)


def _fsdp_opt_in_backward(pg, recompute: bool = True) -> None:
    """FSDP with AdamW fused into the reduce-scatter kernel == FSDP + FusedAdamW."""
    import copy

    import torch.nn.functional as F
    from torch import nn

    from mini_nccl_b200.fsdp import FullyShardedDataParallel
    from mini_nccl_b200.ops.kernels import FusedAdamW

    dev = torch.device("cuda", torch.cuda.current_device())

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = nn.Linear(64, 256)
            self.fc2 = nn.Linear(256, 64)

        def forward(self, x):
            return x + self.fc2(torch.relu(self.fc1(x)))

    torch.manual_seed(0)
    base = nn.Sequential(Block(), Block()).to(dev, torch.bfloat16)
    hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    fused = FullyShardedDataParallel(copy.deepcopy(base), pg, unit_cls=Block, optimizer_in_backward=hp,
                                     recompute=recompute)
    plain = FullyShardedDataParallel(copy.deepcopy(base), pg, unit_cls=Block)
    opt = FusedAdamW(plain.parameters(), **hp)
    g = torch.Generator().manual_seed(5 + pg.rank)
    for _ in range(4):
        x = torch.randn(32, 64, generator=g).to(dev, torch.bfloat16)
        for model in (fused, plain):
            model.zero_grad()
            F.mse_loss(model(x).float(), torch.zeros(32, 64, device=dev)).backward()
            model.sync()
        opt.step()
    pg.device_comm().synchronize()
    a, b = fused.full_state_dict(), plain.full_state_dict()
    for name in a:
        err = (a[name].float() - b[name].float()).abs().max().item()
        assert err <= 2e-2 * (b[name].float().abs().max().item() + 1e-3), (name, err)


@needs2
@pytest.mark.parametrize("recompute", [True, False])
def test_fsdp_optimizer_in_backward_on_gpus(recompute):
    run(_fsdp_opt_in_backward, 2, recompute, timeout=600.0, devices="cuda", op_timeout=60.0)


needs4 = pytest.mark.skipif(n_gpus() < 4, reason="needs at least 4 GPUs")


@needs4
def test_device_collective_battery_four_ranks():
    """W=4 reaches the scatter + all-gather broadcast and 4-way push schedules."""
    run(_battery, 4, devices="cuda", timeout=900.0, op_timeout=60.0)


needs8 = pytest.mark.skipif(n_gpus() < 8, reason="needs 8 GPUs")


@needs8
def test_device_collective_battery_eight_ranks():
    """The whole battery on one 8-GPU NVSwitch box (every schedule, W=8)."""
    run(_battery, 8, devices="cuda", timeout=1200.0, op_timeout=60.0)


@needs8
def test_nvls_collectives_eight_ranks():
    out = run(_nvls_battery, 8, devices="cuda", timeout=900.0, op_timeout=60.0)
    if out[0].startswith("unavailable"):
        pytest.skip(out[0])
    assert all(o == "ok" for o in out), out


@needs8
def test_fused_gemm_collectives_eight_ranks():
    run(_fused_tp, 8, timeout=900.0, devices="cuda", op_timeout=60.0)


@needs8
def test_fsdp_fused_gather_eight_ranks():
    run(_fsdp_fused_vs_plain, 8, devices="cuda", timeout=900.0, op_timeout=60.0)


def _gpt_3d_gpu(pg) -> None:
    """The 3D configuration's model (fused sequence-parallel TP kernels, 1F1B over
    NCCL p2p, DP replicas) on 8 GPUs against one fp32 CPU process, same weights."""
    import types

    import mini_nccl_b200 as mn
    from mini_nccl_b200.models.tp_gpt import GPTStage, sync_tensor_parallel_grads

    dev = torch.device("cuda", torch.cuda.current_device())
    V, T, L, H, Cw = 512, 128, 2, 4, 256
    mesh = mn.ParallelMesh(pg, dp=2, pp=2, tp=2)
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
    stage = stage.to(dev, torch.bfloat16)
    g = torch.Generator().manual_seed(7)
    idx = torch.randint(0, V, (8, T), generator=g)  # 2 replicas x 2 microbatches x 2 sequences
    tgt = torch.randint(0, V, (8, T), generator=g)
    ref.loss(ref(idx), tgt).backward()
    pipe = mn.PipelineParallel(stage, pp, activation_shape=(T // 2, 2, Cw),
                               loss_fn=stage.loss if s == 1 else None, dtype=torch.bfloat16, device=dev)
    mine = slice(4 * d, 4 * d + 4)
    pipe.step(idx[mine].to(dev) if s == 0 else None, tgt[mine].to(dev) if s == 1 else None, n_microbatches=2)
    sync_tensor_parallel_grads(stage, tp)
    mn.average_gradients(dp, list(stage.parameters()))

    def check(got, want, what):
        got, want = got.float().cpu(), want.float()
        err = (got - want).abs().max().item()
        assert err <= 0.08 * want.abs().max().item() + 1e-4, (what, err, want.abs().max().item())

    for j, blk in enumerate(stage.blocks):
        rb = ref.blocks[s * per + j]
        check(blk.ln1.weight.grad, rb.ln1.weight.grad, f"block{j}.ln1")
        a, n = blk.mlp.up.shard_start, blk.mlp.up.shard_size
        check(blk.mlp.up.weight.grad, rb.mlp.up.weight.grad[a: a + n], f"block{j}.mlp.up")
        rows = blk.attn.qkv.shard_rows.cpu()
        check(blk.attn.qkv.weight.grad, rb.attn.qkv.weight.grad.index_select(0, rows), f"block{j}.qkv")
    if s == 1:
        check(stage.head.weight.grad, ref.head.weight.grad, "head")


@needs8
def test_gpt_3d_fused_tp_matches_single_process_on_eight_gpus():
    run(_gpt_3d_gpu, 8, devices="cuda", timeout=900.0, op_timeout=120.0)
