"""Autograd wrappers around the sm_100a kernels.

Every function here requires CUDA bf16 tensors and calls the compiled
extension; if the extension is missing this raises rather than falling back.
GEMM layouts follow ``csrc/cuda/gemm.cu``:

=============  =====================  ============================
product        A operand              B operand
=============  =====================  ============================
Y  = X W^T     X  [M, K] (K-major)    W [N, K] (K-major)
dX = dY W      dY [M, N] (K-major)    W [N, K] read MN-major
dW = dY^T X    dY [M, N] MN-major     X [M, K] MN-major
=============  =====================  ============================
"""

from __future__ import annotations

import math
import os

import torch

EPI_BIAS, EPI_GELU, EPI_RESID, EPI_GELU_GRAD, EPI_ACCUM = 1, 2, 4, 8, 16

#: Head dims whose attention forward runs on tcgen05 (others use mma.sync).
TC_ATTENTION_HEAD_DIMS = (64, 128)
#: tcgen05 backward on/off (``MNB_ATTN_BWD=mma`` selects the mma.sync kernel, for comparisons)
TC_ATTENTION_BWD = os.environ.get("MNB_ATTN_BWD", "tc") != "mma"

_EXT = None
_STATUS: dict[int, torch.Tensor] = {}
NUM_SMS = 148


def ext():
    """The compiled extension, wrapped so every launch is counted."""
    global _EXT
    if _EXT is None:
        from .._build import cuda_ext
        from ..utils.launches import CountingProxy

        _EXT = CountingProxy(cuda_ext())
    return _EXT


def status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _STATUS.get(idx)
    if st is None:
        st = torch.zeros(4, dtype=torch.int32, device=device)
        _STATUS[idx] = st
    return st


_FOLD: dict[int, torch.Tensor] = {}


def fold_accumulator(device: torch.device, n: int) -> torch.Tensor:
    """Persistent zeroed fp32 accumulator (n values + an arrival counter) for the
    single-kernel column reductions; every call leaves it zeroed again, and the
    calls are ordered on the device's stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _FOLD.get(idx)
    if buf is None or buf.numel() < n + 1:
        buf = _FOLD[idx] = torch.zeros(max(n + 1, 1 << 16), dtype=torch.float32, device=device)
    return buf


def check_status(device: torch.device | None = None) -> None:
    """Raise if a GEMM pipeline wait ran out of budget (device sync)."""
    for idx, st in _STATUS.items():
        if device is not None and device.index not in (None, idx):
            continue
        v = int(st[0].item())
        if v:
            st.zero_()
            raise RuntimeError(f"GEMM kernel on cuda:{idx} reported pipeline status {v}")


def supports_gemm(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (
        x.dtype == torch.bfloat16
        and w.dtype == torch.bfloat16
        and w.dim() == 2
        and w.shape[0] % 8 == 0
        and w.shape[1] % 8 == 0
    )


# Split-K cost model: one 128 x BN x 64 k-block of MMAs on one SM at the
# sustained bf16 rate, and the reduction pass reading every fp32 partial slice.
_SUSTAINED_FLOPS = 1.36e15
_HBM_BYTES_PER_S = 6.5e12


def _splits_for(m: int, n: int, k: int) -> int:
    """Split-K factor for small-output / long-K GEMMs (the weight gradients).

    The persistent kernel runs ``tiles * splits`` work units in waves of
    NUM_SMS; the split minimising (waves x k-blocks per unit) plus the
    partial tiles' fp32 traffic (reduce-adds into one workspace) wins.  A
    grid that already fills the machine is never split: the LM head's data
    gradient (384 tiles, 2.6 waves) measured 1.094 ms unsplit and 1.109 ms in
    5 splits, although whole waves alone predicted 13 % less.  Counting whole
    waves matters: 54 output tiles in 3 splits are 162 units, two waves of
    86 k-blocks, where 5 splits run two waves of 52.
    """
    bn = 256 if n >= 256 else 128
    tiles = math.ceil(m / 128) * math.ceil(n / bn)
    k_blocks = math.ceil(k / 64)
    if tiles >= NUM_SMS or k_blocks < 16:
        return 1
    kb_seconds = 128 * bn * 64 * 2 / (_SUSTAINED_FLOPS / NUM_SMS)
    best, best_t = 1, float("inf")
    for s in range(1, min(32, k_blocks // 4) + 1):
        per = math.ceil(k_blocks / s)
        s_eff = math.ceil(k_blocks / per)  # the kernel drops empty splits
        waves = math.ceil(tiles * s_eff / NUM_SMS)
        t = waves * per * kb_seconds + (s_eff * m * n * 4 / _HBM_BYTES_PER_S if s_eff > 1 else 0.0)
        if t < best_t * (1 - 1e-6):
            best, best_t = s_eff, t
    return best


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    bias: torch.Tensor | None = None,
    gelu_out_aux: torch.Tensor | None = None,
    gelu_grad_aux: torch.Tensor | None = None,
    resid: torch.Tensor | None = None,
    accumulate: bool = False,
    out_dtype: torch.dtype = torch.bfloat16,
    splits: int | None = None,
) -> torch.Tensor:
    """``out = epilogue(A B^T)`` on the tcgen05 tensor cores (layouts in the module doc)."""
    M = a.shape[1] if a_mn else a.shape[0]
    K = a.shape[0] if a_mn else a.shape[1]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    epi = 0
    aux = None
    if gelu_out_aux is not None:
        epi |= EPI_GELU
        aux = gelu_out_aux
    if gelu_grad_aux is not None:
        epi |= EPI_GELU_GRAD
        aux = gelu_grad_aux
    if accumulate:
        epi |= EPI_ACCUM
    if splits is None:
        splits = _splits_for(M, N, K) if (epi & ~EPI_ACCUM) == 0 and bias is None and resid is None else 1
    ws = None
    if splits > 1:  # the kernel zeroes it and adds every split's partial tiles into it
        ws = torch.empty(M * N, dtype=torch.float32, device=a.device)
    ext().gemm(a, b, out, a_mn, b_mn, bias, aux, resid, epi, splits, ws, status_word(a.device))
    return out


def _rows(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.stride(-1) == 1 else x2.contiguous()


def bias_grad(g2: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    rows, C = g2.shape
    out = torch.empty(C, dtype=dtype, device=g2.device)
    ext().bias_grad(g2, out, fold_accumulator(g2.device, C), False)
    return out


class Linear(torch.autograd.Function):
    """``y = x W^T + b (+ resid)``; the residual add rides in the GEMM epilogue."""

    @staticmethod
    def forward(ctx, x, weight, bias, resid=None):
        x2 = _rows(x)
        r2 = _rows(resid) if resid is not None else None
        y = gemm(x2, weight, bias=bias, resid=r2)
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        ctx.has_resid = resid is not None
        ctx.x_shape = x.shape
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w = ctx.saved_tensors
        g2 = _rows(gy).contiguous()
        dx = dw = db = dr = None
        if ctx.needs_input_grad[0]:
            dx = gemm(g2, w, b_mn=True).view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            dw = gemm(g2, x2, a_mn=True, b_mn=True)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = bias_grad(g2, w.dtype)
        if ctx.has_resid:
            dr = gy
        return dx, dw, db, dr


class GatheredLinear(torch.autograd.Function):
    """``y = x W^T + b`` where computing it also gathers W's sharded parameter buffer.

    ``gather_gemm(x2)`` runs the fused kernel (FSDP's first GEMM of a unit,
    :meth:`DeviceComm.gather_weight_gemm`) and returns ``x2 W^T + b``; by the
    time it returns (in stream order) ``weight`` -- a view into the gathered
    buffer -- holds its values.  The backward is :class:`Linear`'s.
    """

    @staticmethod
    def forward(ctx, x, weight, bias, gather_gemm):
        x2 = _rows(x)
        y = gather_gemm(x2)
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        ctx.has_resid = False
        ctx.x_shape = x.shape
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, gy):
        dx, dw, db, _ = Linear.backward(ctx, gy)
        return dx, dw, db, None


class LinearGelu(torch.autograd.Function):
    """``gelu(x W^T + b)``: GELU in the forward epilogue, GELU' in the backward one."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        x2 = _rows(x)
        M, N = x2.shape[0], weight.shape[0]
        pre = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
        h = gemm(x2, weight, bias=bias, gelu_out_aux=pre)
        ctx.save_for_backward(x2, weight, pre)
        ctx.has_bias = bias is not None
        ctx.x_shape = x.shape
        return h.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, gh):
        x2, w, pre = ctx.saved_tensors
        g = _rows(gh).contiguous()
        dpre = torch.empty_like(pre)
        ext().gelu_bwd(pre, g, dpre)
        dx = gemm(dpre, w, b_mn=True).view(ctx.x_shape)
        dw = gemm(dpre, x2, a_mn=True, b_mn=True)
        db = bias_grad(dpre, w.dtype) if ctx.has_bias else None
        return dx, dw, db


class MLP(torch.autograd.Function):
    """``resid + gelu(x W1^T + b1) W2^T + b2`` with GELU and GELU' fused into GEMMs."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, resid):
        x2 = _rows(x)
        M = x2.shape[0]
        pre = torch.empty((M, w1.shape[0]), dtype=torch.bfloat16, device=x.device)
        h = gemm(x2, w1, bias=b1, gelu_out_aux=pre)
        y = gemm(h, w2, bias=b2, resid=_rows(resid) if resid is not None else None)
        ctx.save_for_backward(x2, w1, w2, pre, h)
        ctx.x_shape = x.shape
        ctx.has_resid = resid is not None
        return y.view(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w1, w2, pre, h = ctx.saved_tensors
        g = _rows(gy).contiguous()
        dw2 = gemm(g, h, a_mn=True, b_mn=True)
        db2 = bias_grad(g, w2.dtype)
        dpre = gemm(g, w2, b_mn=True, gelu_grad_aux=pre)  # (dY W2) * gelu'(pre)
        dw1 = gemm(dpre, x2, a_mn=True, b_mn=True)
        db1 = bias_grad(dpre, w1.dtype)
        dx = gemm(dpre, w1, b_mn=True).view(ctx.x_shape)
        return dx, dw1, db1, dw2, db2, (gy if ctx.has_resid else None)


class Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        ext().gelu_fwd(xc, y)
        ctx.save_for_backward(xc)
        return y

    @staticmethod
    def backward(ctx, gy):
        (x,) = ctx.saved_tensors
        dx = torch.empty_like(x)
        ext().gelu_bwd(x, gy.contiguous(), dx)
        return dx


class LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps: float):
        xc = x.contiguous()
        rows = xc.numel() // xc.shape[-1]
        y = torch.empty_like(xc)
        mean = torch.empty(rows, dtype=torch.float32, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        ext().layernorm_fwd(xc, weight, bias, y, mean, rstd, eps)
        ctx.save_for_backward(xc, weight, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w, mean, rstd = ctx.saved_tensors
        C = x.shape[-1]
        rows = x.numel() // C
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        db = torch.empty_like(w)
        ext().layernorm_bwd(gy.contiguous(), x, w, mean, rstd, dx, dw, db, fold_accumulator(x.device, 2 * C), False)
        return dx, dw, db, None


class LayerNormResidual(torch.autograd.Function):
    """``(LayerNorm(x), x)``: the second output is the residual branch's copy of x.

    Its gradient and the LayerNorm's input gradient are summed inside the
    LayerNorm backward kernel, instead of by autograd with a separate add
    kernel (x feeds both the norm and the block's residual connection).
    """

    @staticmethod
    def forward(ctx, x, weight, bias, eps: float):
        xc = x.contiguous()
        rows = xc.numel() // xc.shape[-1]
        y = torch.empty_like(xc)
        mean = torch.empty(rows, dtype=torch.float32, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        ext().layernorm_fwd(xc, weight, bias, y, mean, rstd, eps)
        ctx.save_for_backward(xc, weight, mean, rstd)
        return y, x.view_as(x)

    @staticmethod
    def backward(ctx, gy, gres):
        x, w, mean, rstd = ctx.saved_tensors
        C = x.shape[-1]
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        db = torch.empty_like(w)
        acc = fold_accumulator(x.device, 2 * C)
        if gy is None:
            gy = torch.zeros_like(x)
        if gres is None:
            ext().layernorm_bwd(gy.contiguous(), x, w, mean, rstd, dx, dw, db, acc, False)
        else:
            ext().layernorm_bwd_add(gy.contiguous(), x, w, mean, rstd, gres.contiguous(), dx, dw, db, acc, False)
        return dx, dw, db, None


class FlashAttention(torch.autograd.Function):
    """Causal attention straight out of a fused ``[B, T, 3*H*D]`` QKV tensor.

    Returns ``[B, T, H, D]``; the backward returns one contiguous ``dqkv`` so
    the QKV projection's backward GEMMs read it without a concatenation.
    """

    @staticmethod
    def forward(ctx, qkv, n_head: int):
        B, T, C3 = qkv.shape
        C = C3 // 3
        D = C // n_head
        scale = 1.0 / math.sqrt(D)
        q, k, v = qkv[..., :C], qkv[..., C : 2 * C], qkv[..., 2 * C :]
        o = torch.empty((B, T, C), dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty((B, n_head, T), dtype=torch.float32, device=qkv.device)
        if D in TC_ATTENTION_HEAD_DIMS and qkv.is_contiguous():
            ext().flash_attn_fwd_tc(qkv, o, lse, n_head, scale, status_word(qkv.device))
        else:
            ext().flash_attn_fwd(q, k, v, o, lse, n_head, scale)
        ctx.save_for_backward(qkv, o, lse)
        ctx.n_head, ctx.scale = n_head, scale
        return o.view(B, T, n_head, D)

    @staticmethod
    def backward(ctx, go):
        qkv, o, lse = ctx.saved_tensors
        B, T, C3 = qkv.shape
        C = C3 // 3
        q, k, v = qkv[..., :C], qkv[..., C : 2 * C], qkv[..., 2 * C :]
        go = go.reshape(B, T, C).contiguous()
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = dqkv[..., :C], dqkv[..., C : 2 * C], dqkv[..., 2 * C :]
        dq_acc = torch.empty((B, T, C), dtype=torch.float32, device=qkv.device)
        delta = torch.empty((B, ctx.n_head, T), dtype=torch.float32, device=qkv.device)
        D = C // ctx.n_head
        if D in TC_ATTENTION_HEAD_DIMS and T % 128 == 0 and qkv.is_contiguous() and TC_ATTENTION_BWD:
            ext().flash_attn_bwd_tc(qkv, o, go, lse, dqkv, dq_acc, delta, ctx.n_head, ctx.scale,
                                    status_word(qkv.device))
        else:
            ext().flash_attn_bwd(q, k, v, o, go, lse, dq, dk, dv, dq_acc, delta, ctx.n_head, ctx.scale)
        return dqkv, None


class CrossEntropy(torch.autograd.Function):
    """Mean softmax cross-entropy over rows of bf16 logits."""

    @staticmethod
    def forward(ctx, logits, targets):
        z = logits.reshape(-1, logits.shape[-1]).contiguous().clone()
        t = targets.reshape(-1).contiguous()
        loss = torch.empty(z.shape[0], dtype=torch.float32, device=z.device)
        ext().xent_fwd_bwd(z, t, loss, 1.0 / z.shape[0], -100)
        ctx.save_for_backward(z)
        ctx.shape = logits.shape
        return loss.mean()

    @staticmethod
    def backward(ctx, g):
        (z,) = ctx.saved_tensors
        return (z * g.to(z.dtype)).view(ctx.shape), None


class HeadCrossEntropy(torch.autograd.Function):
    """Tied LM head + cross-entropy, gradients computed in the forward pass.

    ``logits = x W^T`` (tcgen05), then one kernel per row turns the logits into
    the loss and, in place, into ``dlogits``; ``dX`` and ``dW`` follow as two
    more GEMMs.  The ``[rows, V]`` logits never exist in fp32 and are freed
    before backward, so peak memory is one bf16 logits chunk.
    """

    @staticmethod
    def forward(ctx, x, weight, targets, chunk_rows: int = 16384):
        x2 = _rows(x)
        t = targets.reshape(-1)
        M, C = x2.shape
        V = weight.shape[0]
        loss = torch.empty(M, dtype=torch.float32, device=x.device)
        dx = torch.empty_like(x2)
        dw = torch.empty((V, C), dtype=torch.float32 if M > chunk_rows else torch.bfloat16, device=x.device)
        for r0 in range(0, M, chunk_rows):
            r1 = min(M, r0 + chunk_rows)
            logits = gemm(x2[r0:r1], weight)
            ext().xent_fwd_bwd(logits, t[r0:r1], loss[r0:r1], 1.0 / M, -100)
            gemm(logits, weight, dx[r0:r1], b_mn=True)
            gemm(logits, x2[r0:r1], dw, a_mn=True, b_mn=True, accumulate=r0 > 0,
                 out_dtype=dw.dtype)
            del logits
        ctx.save_for_backward(dx, dw)
        ctx.x_shape = x.shape
        ctx.w_dtype = weight.dtype
        return loss.mean()

    @staticmethod
    def backward(ctx, g):
        dx, dw = ctx.saved_tensors
        # In place: the gradients were computed for a unit upstream gradient.
        dx.mul_(g.to(dx.dtype))
        if dw.dtype != ctx.w_dtype:
            dw = dw.mul_(g.to(dw.dtype)).to(ctx.w_dtype)
        else:
            dw.mul_(g.to(dw.dtype))
        return dx.view(ctx.x_shape), dw, None, None


class Embedding(torch.autograd.Function):
    """``wte[idx] + wpe[:T]`` for ``idx`` of shape ``[B, T]``."""

    @staticmethod
    def forward(ctx, idx, wte, wpe):
        B, T = idx.shape
        y = torch.empty((B, T, wte.shape[1]), dtype=wte.dtype, device=wte.device)
        ext().embed_fwd(idx.contiguous(), wte, wpe, y)
        ctx.save_for_backward(idx)
        ctx.shapes = (wte.shape, wpe.shape)
        return y

    @staticmethod
    def backward(ctx, gy):
        (idx,) = ctx.saved_tensors
        wte_shape, wpe_shape = ctx.shapes
        dwte = torch.zeros(wte_shape, dtype=gy.dtype, device=gy.device)
        dwpe = torch.zeros(wpe_shape, dtype=gy.dtype, device=gy.device)
        ext().embed_bwd(idx, gy.contiguous(), dwte, dwpe.view(-1, wte_shape[1]), False)
        return None, dwte, dwpe


class FusedAdamW(torch.optim.Optimizer):
    """AdamW over bf16 (or fp32) parameters with fp32 master weights and moments.

    One multi-tensor kernel per step for every parameter: it reads the
    gradient, updates the fp32 master copy and both moments, and writes the
    rounded parameter back.  The pointer table is rebuilt only when a
    gradient's storage moves.
    """

    def __init__(self, params, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, master_weights=True):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.master_weights = master_weights
        self._tables: dict[int, tuple] = {}
        self._step = 0

    def _prepare(self, gi: int, group):
        params = [p for p in group["params"] if p.grad is not None]
        key = tuple((p.data_ptr(), p.grad.data_ptr(), p.grad.dtype) for p in params)
        cached = self._tables.get(gi)
        if cached is not None and cached[0] == key:
            return cached[1:]
        rows, chunks = [], []
        CH = 1 << 16
        pdt = {p.dtype for p in params}
        gdt = {p.grad.dtype for p in params}
        if len(pdt) != 1 or len(gdt) != 1:
            raise ValueError("FusedAdamW needs one parameter dtype and one gradient dtype per group")
        for p in params:
            st = self.state[p]
            if "m" not in st:
                st["m"] = torch.zeros(p.numel(), dtype=torch.float32, device=p.device)
                st["v"] = torch.zeros(p.numel(), dtype=torch.float32, device=p.device)
                if self.master_weights and p.dtype != torch.float32:
                    st["master"] = p.detach().float().reshape(-1).clone()
            master = st.get("master")
            rows.append([p.data_ptr(), p.grad.data_ptr(), master.data_ptr() if master is not None else 0,
                         st["m"].data_ptr(), st["v"].data_ptr(), p.numel()])
            for s0 in range(0, p.numel(), CH):
                chunks.append([len(rows) - 1, s0, min(CH, p.numel() - s0)])
        dev = params[0].device
        table = torch.tensor(rows, dtype=torch.int64).to(dev)
        chunks_t = torch.tensor(chunks, dtype=torch.int64).to(dev)
        out = (table, chunks_t, next(iter(pdt)) == torch.bfloat16, next(iter(gdt)) == torch.bfloat16)
        self._tables[gi] = (key, *out)
        return out

    def state_dict(self) -> dict:
        """torch's optimizer state dict plus the shared step count.

        Moments and master weights are saved as fp32, whatever the
        parameters' dtype."""
        sd = super().state_dict()
        sd["fused_adamw_step"] = self._step
        return sd

    def load_state_dict(self, state_dict: dict) -> None:
        """Restore a :meth:`state_dict`, keeping moments and masters in fp32.

        (``torch.optim.Optimizer.load_state_dict`` would cast them to each
        parameter's dtype, rounding fp32 masters of bf16 parameters.)"""
        saved_groups = state_dict["param_groups"]
        if len(saved_groups) != len(self.param_groups):
            raise ValueError("the state dict has a different number of parameter groups")
        by_index = {}
        for group, saved in zip(self.param_groups, saved_groups, strict=True):
            if len(group["params"]) != len(saved["params"]):
                raise ValueError("a parameter group has a different number of parameters")
            by_index.update(zip(saved["params"], group["params"], strict=True))
            group.update({k: v for k, v in saved.items() if k != "params"})
        self.state.clear()
        for index, st in state_dict["state"].items():
            p = by_index[index]
            self.state[p] = {k: v.detach().to(device=p.device, dtype=torch.float32).clone().contiguous()
                             if torch.is_tensor(v) else v for k, v in st.items()}
        self._step = int(state_dict.get("fused_adamw_step", 0))
        self._tables.clear()  # the cached pointer tables name the old state tensors

    @torch.no_grad()
    def step(self, closure=None, grad_scale: float = 1.0):
        loss = closure() if closure is not None else None
        self._step += 1
        for gi, group in enumerate(self.param_groups):
            if not any(p.grad is not None for p in group["params"]):
                continue
            table, chunks, p_bf16, g_bf16 = self._prepare(gi, group)
            b1, b2 = group["betas"]
            ext().adamw_step(table, chunks, p_bf16, g_bf16, group["lr"], b1, b2, group["eps"],
                             group["weight_decay"], 1 - b1 ** self._step, 1 - b2 ** self._step, grad_scale)
        return loss
