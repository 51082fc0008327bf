"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference.

Shapes include odd sizes (rows that are not tile multiples, widths that are
not 256 multiples) so masking and tail paths run.  Tolerances are set for
bf16 inputs/outputs with fp32 accumulation.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU only to be deselected
    pytest.skip("needs a CUDA device", allow_module_level=True)

from mini_nccl_b200.ops import kernels as K  # noqa: E402

DEV = torch.device("cuda", 0)


def rnd(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(DEV, torch.bfloat16)


def close(got, want, tol):
    """Element-wise: |got - want| <= tol * |want| + (tol / 4) * max|want|.

    The relative term bounds every entry by its own magnitude (bf16 rounding
    of the result plus the error fp32 accumulation lets through); the small
    absolute floor, a quarter of the tolerance at the tensor's largest entry,
    covers entries that are near zero only because of cancellation.
    """
    g, w = got.float(), want.float()
    scale = w.abs().max().item() + 1e-6
    err = (g - w).abs()
    bound = tol * w.abs() + 0.25 * tol * scale
    bad = err > bound
    if bool(bad.any()):
        i = int(torch.argmax((err - bound).flatten()).item())
        raise AssertionError(
            f"{int(bad.sum())} of {err.numel()} entries out of tolerance; worst at flat index {i}: "
            f"got {g.flatten()[i].item():.5g}, want {w.flatten()[i].item():.5g} (tol {tol}, max |want| {scale:.4g})")


def test_extension_is_the_in_tree_build():
    from mini_nccl_b200 import _build

    mod = K.ext()
    assert str(_build.BUILD) in mod.__file__, mod.__file__


@pytest.mark.parametrize("M,N,K_", [(128, 256, 64), (256, 512, 128), (300, 264, 200), (1000, 768, 768),
                                    (64, 128, 64), (4096, 2304, 768)])
def test_gemm_forward_layout(M, N, K_):
    a = rnd(M, K_, seed=1)
    b = rnd(N, K_, seed=2)
    out = K.gemm(a, b)
    torch.cuda.synchronize()
    K.check_status()
    close(out, a.float() @ b.float().t(), 1e-2)


@pytest.mark.parametrize("M,N,K_", [(256, 256, 128), (300, 264, 200), (1024, 768, 3072)])
def test_gemm_data_grad_layout(M, N, K_):
    gy = rnd(M, N, seed=3)
    w = rnd(N, K_, seed=4)
    dx = K.gemm(gy, w, b_mn=True)  # [M, K] = gy @ w
    torch.cuda.synchronize()
    close(dx, gy.float() @ w.float(), 1e-2)


@pytest.mark.parametrize("T,N,K_", [(256, 128, 256), (1000, 264, 200), (4096, 768, 3072)])
def test_gemm_weight_grad_layout(T, N, K_):
    gy = rnd(T, N, seed=5)
    x = rnd(T, K_, seed=6)
    dw = K.gemm(gy, x, a_mn=True, b_mn=True)  # [N, K] = gy^T @ x (split-K when small)
    torch.cuda.synchronize()
    close(dw, gy.float().t() @ x.float(), 1e-2)


def test_gemm_epilogues():
    M, N, K_ = 384, 512, 256
    a, b = rnd(M, K_, seed=7), rnd(N, K_, seed=8, scale=0.1)
    bias = rnd(N, seed=9)
    resid = rnd(M, N, seed=10)
    ref = a.float() @ b.float().t() + bias.float()
    close(K.gemm(a, b, bias=bias), ref, 1e-2)
    close(K.gemm(a, b, bias=bias, resid=resid), ref + resid.float(), 1e-2)
    pre = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    h = K.gemm(a, b, bias=bias, gelu_out_aux=pre)
    close(pre, ref, 1e-2)
    close(h, F.gelu(ref), 1e-2)
    g = K.gemm(a, b, gelu_grad_aux=pre)
    x = pre.float().requires_grad_(True)
    F.gelu(x).backward(torch.ones_like(x))
    close(g, (a.float() @ b.float().t()) * x.grad, 2e-2)
    acc = rnd(M, N, seed=11)
    want = acc.float() + a.float() @ b.float().t()
    K.gemm(a, b, acc, accumulate=True)
    close(acc, want, 1e-2)
    f32 = K.gemm(a, b, out_dtype=torch.float32)
    close(f32, a.float() @ b.float().t(), 1e-3)


@pytest.mark.parametrize("M,N,splits", [(256, 192, 4), (200, 136, 3), (2304, 768, 8)])
def test_gemm_split_k_accumulate(M, N, splits):
    # split-K partial tiles are added into one fp32 workspace by TMA reduce-add;
    # M and N off the tile grid exercise the clipped boxes
    gy, x = rnd(8192, M, seed=12), rnd(8192, N, seed=13)
    dw = rnd(M, N, seed=14)
    want = dw.float() + gy.float().t() @ x.float()
    K.gemm(gy, x, dw, a_mn=True, b_mn=True, accumulate=True, splits=splits)
    close(dw, want, 1e-2)
    f32 = K.gemm(gy, x, a_mn=True, b_mn=True, out_dtype=torch.float32, splits=splits)
    close(f32, gy.float().t() @ x.float(), 1e-3)


@pytest.mark.parametrize("rows,C", [(1000, 768), (20000, 768), (5000, 256), (3000, 512), (3000, 1024),
                                    (777, 2048), (300, 4096), (64, 640)])
def test_layernorm_forward_backward(rows, C):
    x = rnd(rows, C, seed=15).requires_grad_(True)
    w = (1 + 0.1 * rnd(C, seed=16).float()).to(torch.bfloat16).requires_grad_(True)
    b = rnd(C, seed=17, scale=0.1).requires_grad_(True)
    gy = rnd(rows, C, seed=18)
    y = K.LayerNorm.apply(x, w, b, 1e-5)
    y.backward(gy)
    xr, wr, br = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    yr = F.layer_norm(xr, (C,), wr, br, 1e-5)
    yr.backward(gy.float())
    close(y, yr, 2e-2)
    close(x.grad, xr.grad, 3e-2)
    close(w.grad, wr.grad, 2e-2)
    close(b.grad, br.grad, 2e-2)


@pytest.mark.parametrize("rows,C", [(20000, 768), (3000, 1024), (500, 2048)])
def test_layernorm_residual_gradients_meet_in_one_kernel(rows, C):
    x = rnd(rows, C, seed=40).requires_grad_(True)
    w = (1 + 0.1 * rnd(C, seed=41).float()).to(torch.bfloat16).requires_grad_(True)
    b = rnd(C, seed=42, scale=0.1).requires_grad_(True)
    gy, gr = rnd(rows, C, seed=43), rnd(rows, C, seed=44)
    y, x_alias = K.LayerNormResidual.apply(x, w, b, 1e-5)
    torch.autograd.backward([y, x_alias], [gy, gr])
    xf, wf, bf = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    yf = F.layer_norm(xf, (C,), wf, bf, 1e-5)
    torch.autograd.backward([yf, xf * 1.0], [gy.float(), gr.float()])
    close(y, yf, 2e-2)
    close(x.grad, xf.grad, 3e-2)
    close(w.grad, wf.grad, 2e-2)
    close(b.grad, bf.grad, 2e-2)


@pytest.mark.parametrize("rows,C", [(16384, 768), (16384, 2304), (1000, 3072), (130, 40)])
def test_bias_grad_column_sums(rows, C):
    g = rnd(rows, C, seed=30)
    want = g.float().sum(0)
    got = K.bias_grad(g, torch.float32)
    close(got, want, 1e-2)
    got2 = K.bias_grad(g, torch.float32)  # the fold accumulator re-zeroes itself between calls
    close(got2, want, 1e-2)


def test_gelu_forward_backward():
    x = rnd(4096, 64, seed=19).requires_grad_(True)
    gy = rnd(4096, 64, seed=20)
    y = K.Gelu.apply(x)
    y.backward(gy)
    xr = x.detach().float().requires_grad_(True)
    F.gelu(xr).backward(gy.float())
    close(y, F.gelu(xr), 1e-2)
    close(x.grad, xr.grad, 2e-2)


@pytest.mark.parametrize("B,T,H,D", [(2, 64, 2, 64), (2, 200, 3, 64), (1, 256, 2, 128), (2, 130, 2, 32),
                                     (2, 512, 3, 64), (1, 1024, 2, 64), (2, 384, 2, 128),
                                     (1, 2048, 2, 128)])  # the FSDP / 3D configs' head dim and length
def test_flash_attention(B, T, H, D):
    C = H * D
    qkv = rnd(B, T, 3 * C, seed=21).requires_grad_(True)
    go = rnd(B, T, H, D, seed=22)
    y = K.FlashAttention.apply(qkv, H)
    y.backward(go)
    ref_in = qkv.detach().float().requires_grad_(True)
    q, k, v = (t.view(B, T, H, D).transpose(1, 2) for t in ref_in.split(C, -1))
    yr = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2)
    yr.backward(go.float())
    close(y, yr, 2e-2)
    close(qkv.grad, ref_in.grad, 3e-2)


@pytest.mark.parametrize("rise", [0.0, 2.0, 8.0])
def test_flash_attention_forward_with_scores_rising_along_the_keys(rise):
    """Scores that grow tile after tile exercise the online softmax's rescaling:
    every key tile raises the running maximum (rise=8: by ~11 log2 units per
    tile; rise=2: by ~3; rise=0: ordinary scores), so the output accumulated
    over earlier tiles is rescaled at each step."""
    B, T, H, D = 2, 1024, 2, 64
    C = H * D
    g = torch.Generator(device="cpu").manual_seed(31)
    q = torch.randn(B, T, H, D, generator=g) * 0.5 + 1.0
    k = torch.randn(B, T, H, D, generator=g) * 0.5
    k = k + rise * (torch.arange(T, dtype=torch.float32) / T).view(1, T, 1, 1)
    v = torch.randn(B, T, H, D, generator=g)
    qkv = torch.cat([t.reshape(B, T, C) for t in (q, k, v)], -1).to(DEV, torch.bfloat16)
    y = K.FlashAttention.apply(qkv, H)
    ref = qkv.float()
    qr, kr, vr = (t.view(B, T, H, D).transpose(1, 2) for t in ref.split(C, -1))
    yr = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True).transpose(1, 2)
    close(y, yr, 2e-2)


def test_softmax_polynomial_exp2_against_exp2():
    """The FMA-pipe exp2 of the attention softmax stays within bf16's half-ulp of exp2."""
    x = torch.cat([torch.linspace(-126.0, 0.0, 1 << 20, device=DEV),
                   -torch.rand(1 << 20, device=DEV) * 30.0, torch.tensor([0.0, -1.0, -0.5, -125.999], device=DEV)])
    y = torch.empty_like(x)
    K.ext().exp2_poly_eval(x, y)
    want = torch.exp2(x.double())
    rel = ((y.double() - want).abs() / want).max().item()
    assert rel < 2.0 ** -9, rel
    assert torch.all(y[-4:-2] == torch.tensor([1.0, 0.5], device=DEV))  # exact at integers


def test_cross_entropy_and_fused_head():
    M, V, C = 512, 1000, 256
    logits = rnd(M, V, seed=23, scale=2.0).requires_grad_(True)
    tgt = torch.randint(0, V, (M,), device=DEV)
    loss = K.CrossEntropy.apply(logits, tgt)
    loss.backward()
    lr = logits.detach().float().requires_grad_(True)
    F.cross_entropy(lr, tgt).backward()
    assert abs(loss.item() - F.cross_entropy(lr, tgt).item()) < 2e-2
    close(logits.grad, lr.grad, 3e-2)
    x = rnd(M, C, seed=24).requires_grad_(True)
    w = rnd(1008, C, seed=25, scale=0.05).requires_grad_(True)
    tgt = torch.randint(0, 1008, (M,), device=DEV)
    loss = K.HeadCrossEntropy.apply(x, w, tgt)
    loss.backward()
    xr, wr = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lref = F.cross_entropy(xr @ wr.t(), tgt)
    lref.backward()
    assert abs(loss.item() - lref.item()) < 2e-2
    close(x.grad, xr.grad, 3e-2)
    close(w.grad, wr.grad, 3e-2)


def test_embedding():
    V, T, C, B = 1000, 64, 128, 4
    wte = rnd(V, C, seed=26).requires_grad_(True)
    wpe = rnd(T, C, seed=27).requires_grad_(True)
    idx = torch.randint(0, V, (B, T), device=DEV)
    gy = rnd(B, T, C, seed=28)
    y = K.Embedding.apply(idx, wte, wpe)
    y.backward(gy)
    wr, pr = wte.detach().float().requires_grad_(True), wpe.detach().float().requires_grad_(True)
    (wr[idx] + pr[None]).backward(gy.float())
    close(y, wr[idx] + pr[None], 1e-2)
    close(wte.grad, wr.grad, 2e-2)
    close(wpe.grad, pr.grad, 2e-2)


def test_fused_adamw_matches_torch():
    torch.manual_seed(0)
    ps = [torch.randn(300, 7, device=DEV).to(torch.bfloat16).float(), torch.randn(1001, device=DEV).to(torch.bfloat16).float()]
    ref = [p.clone().requires_grad_(True) for p in ps]
    mine = [p.to(torch.bfloat16).requires_grad_(True) for p in ps]
    opt = K.FusedAdamW(mine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    ropt = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, eps=1e-8)
    for step in range(5):
        grads = [torch.randn_like(p) for p in ps]
        for p, g in zip(mine, grads):
            p.grad = g.to(torch.bfloat16)
        for p, g in zip(ref, grads):
            p.grad = g.to(torch.bfloat16).float()
        opt.step()
        ropt.step()
    for p, r in zip(mine, ref):
        close(p.detach(), r.detach(), 2e-2)
        close(opt.state[p]["master"].view_as(r), r.detach(), 1e-4)


def test_gpt_block_matches_cpu_reference():
    from mini_nccl_b200.models.gpt import GPT

    torch.manual_seed(0)
    cpu = GPT(vocab_size=512, block_size=128, n_layer=2, n_head=4, n_embd=256)
    gpu = GPT(vocab_size=512, block_size=128, n_layer=2, n_head=4, n_embd=256)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.to(DEV, torch.bfloat16)
    idx = torch.randint(0, 512, (4, 128))
    tgt = torch.randint(0, 512, (4, 128))
    _, lc = cpu(idx, tgt)
    lc.backward()
    _, lg = gpu(idx.to(DEV), tgt.to(DEV))
    lg.backward()
    assert abs(lg.item() - lc.item()) < 3e-2, (lg.item(), lc.item())
    for (name, pc), pg in zip(cpu.named_parameters(), gpu.parameters()):
        if pc.grad is None:
            continue
        err = (pg.grad.float().cpu() - pc.grad).abs().max().item()
        ref = pc.grad.abs().max().item() + 1e-8
        assert err <= 0.06 * ref, f"{name}: grad err {err:.3g} vs {ref:.3g}"


def test_gemm_throughput_is_tensor_core_class():
    """Not a benchmark: catches a silently broken (e.g. serialised) pipeline."""
    M = N = K_ = 4096
    a, b = rnd(M, K_, seed=30), rnd(N, K_, seed=31)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    for _ in range(3):
        K.gemm(a, b, out)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(10):
        K.gemm(a, b, out)
    e.record()
    torch.cuda.synchronize()
    tflops = 2 * M * N * K_ * 10 / (s.elapsed_time(e) / 1e3) / 1e12
    print(f"tcgen05 GEMM 4096^3: {tflops:.0f} TFLOP/s")
    assert tflops > 200, tflops
    assert math.isfinite(tflops)
