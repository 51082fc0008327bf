"""Count this library's own kernel launches (reported by bench.py).

Every call into the compiled extension goes through :func:`counted`, which
adds the number of kernels that entry point launches.  Library kernels
(cuBLAS, torch's own elementwise ops) are not counted: the figure is how many
of *our* kernels ran.
"""

from __future__ import annotations

import threading

_lock = threading.Lock()
_count = 0

# Kernels launched per call of each extension entry point.
KERNELS_PER_CALL = {
    "gemm": 1,
    "layernorm_fwd": 1,
    "layernorm_bwd": 1,
    "layernorm_bwd_add": 1,
    "bias_grad": 1,
    "gelu_fwd": 1,
    "gelu_bwd": 1,
    "embed_fwd": 1,
    "embed_bwd": 2,
    "xent_fwd_bwd": 1,
    "adamw_step": 1,
    "flash_attn_fwd": 1,
    "flash_attn_fwd_tc": 1,
    "flash_attn_bwd": 3,
    "flash_attn_bwd_tc": 3,
    "all_reduce": 1,
    "reduce_scatter": 1,
    "move": 1,
    "barrier": 1,
    "stepped_all_reduce": 1,
    "gemm_rs": 1,
    "reduce_scatter_adamw": 1,
    "ag_gemm": 1,
}


def add(n: int) -> None:
    global _count
    with _lock:
        _count += n


def count() -> int:
    return _count


def reset() -> None:
    global _count
    with _lock:
        _count = 0


class CountingProxy:
    """Wraps the extension module (or a native object) and counts launches.

    The counting wrapper of each entry point is built once and cached on the
    proxy, so a launch costs one dict lookup and one counter update.
    """

    def __init__(self, target) -> None:
        object.__setattr__(self, "_t", target)

    def __getattr__(self, name):
        attr = getattr(self._t, name)
        per = KERNELS_PER_CALL.get(name)
        if per is None or not callable(attr):
            return attr
        if name == "gemm":
            def call(*args, **kwargs):
                global _count
                out = attr(*args, **kwargs)
                _count += per + (1 if len(args) > 9 and isinstance(args[9], int) and args[9] > 1 else 0)
                return out
        else:
            def call(*args, **kwargs):
                global _count
                out = attr(*args, **kwargs)
                _count += per
                return out
        if isinstance(self._t, __import__("types").ModuleType):
            object.__setattr__(self, name, call)  # module functions are stable: cache the wrapper
        return call
