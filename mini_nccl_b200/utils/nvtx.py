"""NVTX ranges for the device collectives and fused kernels.

Every collective a :class:`~mini_nccl_b200.device.DeviceComm` launches (the
fused GEMM + collective kernels, the reduce-scatter + AdamW kernel and the DDP
bucket all-reduces among them) and every pipeline stage transfer is wrapped in
an NVTX range named ``mnb:<op>[<algorithm>] <bytes>B``, so an Nsight Systems
timeline labels the communication kernels and shows which ones overlapped
compute.  The ranges mark host issue time (where the launch happened); the
kernel rows of the same timeline show when the GPU ran them.

Without a profiler attached an NVTX push/pop is a call into a no-op stub.
``MINI_NCCL_NVTX=0`` turns the ranges off entirely.
"""

from __future__ import annotations

import os
from contextlib import contextmanager

ENABLED = os.environ.get("MINI_NCCL_NVTX", "1") != "0"

_push = _pop = None


def _bind() -> bool:
    global _push, _pop
    if _push is None:
        try:
            import torch

            if not torch.cuda.is_available():
                raise RuntimeError("no CUDA")
            _push, _pop = torch.cuda.nvtx.range_push, torch.cuda.nvtx.range_pop
        except Exception:
            _push = _pop = False  # type: ignore[assignment]
    return bool(_push)


def push(name: str) -> bool:
    """Open a range; returns whether one was opened (pass it to :func:`pop`)."""
    if ENABLED and _bind():
        _push(name)
        return True
    return False


def pop(opened: bool) -> None:
    if opened:
        _pop()


def label(op: str, algorithm: str = "", nbytes: int = 0) -> str:
    return f"mnb:{op}[{algorithm}] {nbytes}B" if algorithm else f"mnb:{op} {nbytes}B"


@contextmanager
def nvtx_range(name: str):
    opened = push(name)
    try:
        yield
    finally:
        pop(opened)
