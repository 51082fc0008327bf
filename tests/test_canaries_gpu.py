"""Guard bands around kernel outputs: no kernel writes outside its output.

compute-sanitizer is not available on the GPU pool, so out-of-bounds writes
are caught the way the plan for this library asks: every output here is a
view into a larger buffer whose head and tail (the guard bands) hold a
sentinel, the kernel runs on odd sizes that exercise its clipped tiles and
tail loops, and afterwards the guard bands must still hold the sentinel
bit for bit -- and the output itself must be right.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU only to be deselected
    pytest.skip("needs a CUDA device", allow_module_level=True)

from mini_nccl_b200.launcher import run  # noqa: E402
from mini_nccl_b200.ops import kernels as K  # noqa: E402

DEV = torch.device("cuda", 0)
GUARD = 4096  # elements on each side (a multiple of 8: the view stays 16-byte aligned)
SENTINEL = -12345.0


def guarded(numel: int, dtype: torch.dtype, device=DEV) -> tuple[torch.Tensor, torch.Tensor]:
    """(whole buffer, the middle ``numel`` elements) with the guards set to SENTINEL."""
    buf = torch.full((numel + 2 * GUARD,), SENTINEL, dtype=dtype, device=device)
    return buf, buf[GUARD: GUARD + numel]


def guards_intact(buf: torch.Tensor) -> bool:
    want = torch.full((GUARD,), SENTINEL, dtype=buf.dtype, device=buf.device)
    return bool(torch.equal(buf[:GUARD], want) and torch.equal(buf[-GUARD:], want))


def rnd(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(DEV, torch.bfloat16)


@pytest.mark.parametrize("M,N,K_", [(300, 264, 200), (129, 136, 72), (1000, 520, 64)])
@pytest.mark.parametrize("epi", ["none", "bias", "gelu", "resid"])
def test_gemm_forward_stays_inside_its_output(M, N, K_, epi):
    a, b = rnd(M, K_, seed=1), rnd(N, K_, seed=2, scale=0.1)
    buf, out = guarded(M * N, torch.bfloat16)
    out = out.view(M, N)
    kw: dict = {}
    ref = a.float() @ b.float().t()
    aux_buf = None
    if epi in ("bias", "gelu"):
        kw["bias"] = rnd(N, seed=3)
        ref = ref + kw["bias"].float()
    if epi == "gelu":
        aux_buf, aux = guarded(M * N, torch.bfloat16)
        kw["gelu_out_aux"] = aux.view(M, N)
    if epi == "resid":
        kw["resid"] = rnd(M, N, seed=4)
        ref = ref + kw["resid"].float()
    K.gemm(a, b, out, **kw)
    torch.cuda.synchronize()
    K.check_status()
    assert guards_intact(buf)
    if aux_buf is not None:
        assert guards_intact(aux_buf)
        ref = torch.nn.functional.gelu(ref)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("M,N,splits", [(200, 136, 3), (264, 768, 5)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_split_k_weight_gradient_stays_inside_its_output(M, N, splits, dtype):
    gy, x = rnd(4096, M, seed=5), rnd(4096, N, seed=6)
    buf, out = guarded(M * N, dtype)
    out = out.view(M, N)
    K.gemm(gy, x, out, a_mn=True, b_mn=True, out_dtype=dtype, splits=splits)
    torch.cuda.synchronize()
    K.check_status()
    assert guards_intact(buf)
    ref = gy.float().t() @ x.float()
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err


def _collectives(pg) -> str:
    """Device all-reduce (every algorithm), reduce-scatter, all-gather and
    broadcast on odd sizes, outputs inside guard bands."""
    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = pg.world_size, pg.rank
    dc = pg.device_comm()
    for n in (1, 3, 1003, 262147):
        for algorithm in ("one_shot", "two_shot", "ring", "tree", "auto"):
            buf, t = guarded(n, torch.float32, dev)
            t.copy_(torch.arange(n, dtype=torch.float32, device=dev) + r)
            dc.all_reduce(t, algorithm=algorithm)
            torch.cuda.synchronize(dev)
            dc.check()
            want = W * torch.arange(n, dtype=torch.float32, device=dev) + W * (W - 1) / 2
            assert torch.equal(t, want), (n, algorithm)
            assert guards_intact(buf), (n, algorithm)
        m = n * W
        x = torch.arange(m, dtype=torch.float32, device=dev) * (r + 1)
        got = dc.reduce_scatter(x)
        torch.cuda.synchronize(dev)
        full = torch.arange(m, dtype=torch.float32, device=dev) * (W * (W + 1) / 2)
        assert torch.equal(got, full[r * n:(r + 1) * n]), n
        shard = torch.full((n,), float(r + 1), device=dev)
        buf, out = guarded(m, torch.float32, dev)
        dc.all_gather(shard, out.view(W, n))
        torch.cuda.synchronize(dev)
        assert guards_intact(buf), n
        assert torch.equal(out.view(W, n), torch.arange(1, W + 1, dtype=torch.float32, device=dev)[:, None].expand(W, n))
        buf, t = guarded(n, torch.float32, dev)
        t.fill_(float(r + 7))
        dc.broadcast(t, src=W - 1)
        torch.cuda.synchronize(dev)
        dc.check()
        assert guards_intact(buf), n
        assert bool((t == float(W + 6)).all()), n
    return "ok"


needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")


@needs2
@pytest.mark.multigpu
def test_device_collectives_stay_inside_their_outputs():
    assert run(_collectives, 2, devices="cuda", timeout=600.0, op_timeout=60.0) == ["ok", "ok"]
