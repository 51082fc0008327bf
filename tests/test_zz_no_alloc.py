"""The allocation-free C entry point for the bias gradient.

Some callers of this library may not allocate device memory themselves (a
plugin inside another runtime that owns all device memory, a service that has
reserved the device for its own pool, a loop that cannot afford cudaMalloc's
possible device-wide wait).  ``mnb_bias_grad_noalloc`` serves them: it takes
the caller's input and output and keeps its scratch in a fixed array built
into the library.  This test calls it through its exported C symbol and
checks it against the allocating entry point (``bias_grad``) on two calls in
a row, since every call reuses the same built-in scratch.

Named so that pytest collects it last: a failure here leaves every other test
already run.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from mini_nccl_b200 import _build  # noqa: E402
from mini_nccl_b200.ops import kernels as K  # noqa: E402

DEV = torch.device("cuda", 0)


def _lib() -> ctypes.CDLL:
    K.ext()  # load the extension (and torch's libraries) the normal way first
    lib = ctypes.CDLL(str(_build.cuda_lib_path()))
    fn = lib.mnb_bias_grad_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    lib.mnb_noalloc_last_error.restype = ctypes.c_char_p
    lib.mnb_noalloc_max_scratch_floats.restype = ctypes.c_longlong
    return lib


def _call(lib, g: torch.Tensor, out: torch.Tensor, accumulate: bool = False) -> int:
    stream = torch.cuda.current_stream(DEV).cuda_stream
    return lib.mnb_bias_grad_noalloc(g.data_ptr(), out.data_ptr(), g.shape[0], g.shape[1],
                                     int(out.dtype == torch.float32), int(accumulate), stream)


@pytest.mark.parametrize("rows,cols,dtype", [(16384, 768, torch.bfloat16), (1000, 3072, torch.float32),
                                             (37, 264, torch.bfloat16)])
def test_no_alloc_entry_matches_allocating_entry(rows, cols, dtype):
    lib = _lib()
    g = (torch.randn(rows, cols, generator=torch.Generator().manual_seed(rows)) * 0.5).to(DEV, torch.bfloat16)
    want = K.bias_grad(g, dtype).float()
    for call in range(2):  # the second call reuses scratch the first one left behind
        out = torch.full((cols,), float("nan"), dtype=dtype, device=DEV)
        rc = _call(lib, g, out)
        torch.cuda.synchronize()
        assert rc == 0, lib.mnb_noalloc_last_error().decode()
        err = (out.float() - want).abs().max().item()
        assert err <= 1e-2 * (want.abs().max().item() + 1e-6), f"call {call}: max err {err}"


def test_no_alloc_entry_bf16_accumulate_and_near_limit():
    """Accumulate into a bf16 output, on a shape that uses most of the scratch."""
    lib = _lib()
    limit = lib.mnb_noalloc_max_scratch_floats()
    cols = 4096
    rows = (limit // cols) * 128 - 5  # ceil(rows/128) * cols is just inside the limit
    g = (torch.randn(rows, cols, device=DEV) * 0.25).to(torch.bfloat16)
    base = (torch.randn(cols, device=DEV)).to(torch.bfloat16)
    want = base.float() + K.bias_grad(g, torch.float32)
    for call in range(2):
        out = base.clone()
        assert _call(lib, g, out, accumulate=True) == 0, lib.mnb_noalloc_last_error().decode()
        torch.cuda.synchronize()
        err = (out.float() - want).abs().max().item()
        assert err <= 1e-2 * want.abs().max().item(), f"call {call}: max err {err}"


def test_no_alloc_entry_more_bands_than_grid_rows():
    """More than 65,535 bands of 128 rows: CTAs walk several bands each."""
    lib = _lib()
    cols = 8
    rows = 65535 * 128 + 3 * 128 + 17  # 65,539 bands
    g = (torch.rand(rows, cols, device=DEV) - 0.5).to(torch.bfloat16)
    want = g.float().sum(0)
    out = torch.zeros(cols, dtype=torch.float32, device=DEV)
    rc = _call(lib, g, out)
    torch.cuda.synchronize()
    assert rc == 0, lib.mnb_noalloc_last_error().decode()
    assert (out - want).abs().max().item() <= 1e-3 * rows ** 0.5


def test_no_alloc_entry_accumulates_and_rejects_oversize():
    lib = _lib()
    g = torch.randn(512, 256, device=DEV).to(torch.bfloat16)
    out = torch.ones(256, dtype=torch.float32, device=DEV)
    assert _call(lib, g, out, accumulate=True) == 0
    torch.cuda.synchronize()
    want = 1.0 + g.float().sum(0)
    assert (out - want).abs().max().item() < 1e-2 * want.abs().max().item()
    limit = lib.mnb_noalloc_max_scratch_floats()
    cols = 4096
    too_many_rows = (limit // cols + 1) * 128
    big = torch.empty(1, cols, dtype=torch.bfloat16, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.mnb_bias_grad_noalloc(big.data_ptr(), out.data_ptr(), too_many_rows, cols, 1, 0, stream)
    assert rc == 2
    assert b"maximum" in lib.mnb_noalloc_last_error()
