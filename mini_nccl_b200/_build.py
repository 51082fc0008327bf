"""In-tree builder for the native extensions.

Two extensions, both built inside the package directory so they travel with
the source tree and are found without any install step:

* ``_host``: the C++ TCP transport (pybind11 only, no torch headers, no CUDA).
  It is what CPU-tensor collectives and every CPU test run on.
* ``_cuda``: every sm_100a kernel (collectives over peer memory, tcgen05 GEMM,
  attention, LayerNorm, cross-entropy, AdamW, embedding) plus the device
  communicator runtime.  Compiled with ``-gencode arch=compute_100a,code=sm_100a``
  only; there is no other architecture.

Both are rebuilt only when a source file is newer than the built library.
"""

from __future__ import annotations

import fcntl
import glob
import hashlib
import importlib.machinery
import importlib.util
import os
import subprocess
import sys
import sysconfig
from contextlib import contextmanager
from pathlib import Path

PKG = Path(__file__).resolve().parent
BUILD = PKG / "_build"
HOST_SRC = sorted((PKG / "csrc" / "host").glob("*.cpp"))
CUDA_DIR = PKG / "csrc" / "cuda"
INCLUDE_DIR = PKG / "csrc" / "include"

SM100A = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *SM100A,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]


def _ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def host_lib_path() -> Path:
    return BUILD / "host" / f"_host{_ext_suffix()}"


def cuda_lib_path() -> Path:
    return BUILD / "cuda" / "_cuda.so"


@contextmanager
def _lock(name: str):
    BUILD.mkdir(parents=True, exist_ok=True)
    with open(BUILD / f".{name}.lock", "w") as fh:
        fcntl.flock(fh, fcntl.LOCK_EX)
        try:
            yield
        finally:
            fcntl.flock(fh, fcntl.LOCK_UN)


def _digest(sources: list[Path], extra: str = "") -> str:
    h = hashlib.sha256(extra.encode())
    for s in sources:
        h.update(s.name.encode())
        h.update(s.read_bytes())
    return h.hexdigest()


def _stale(target: Path, sources: list[Path], extra: str = "") -> bool:
    """Content-hash staleness: copies of the tree keep their built libraries."""
    stamp = target.with_name(target.name + ".sha256")
    if not target.exists() or not stamp.exists():
        return True
    return stamp.read_text().strip() != _digest(sources, extra)


def _stamp(target: Path, digest: str) -> None:
    """Record the digest the build started from (an edit made during the
    build then leaves the library stale, as it is)."""
    target.with_name(target.name + ".sha256").write_text(digest)


def _cxx() -> str:
    """The system C++ compiler.

    ``$CXX`` is deliberately not honoured: on the images this runs on it can
    point at a wrapper that links a different unwinder, and a C++ exception
    crossing the pybind11 boundary then crashes instead of raising.
    """
    for cand in ("/usr/bin/g++", "/usr/bin/c++"):
        if os.path.exists(cand):
            return cand
    return "g++"


def build_host(force: bool = False, verbose: bool = False) -> Path:
    """Compile the pybind11 TCP transport with the system C++ compiler."""
    import pybind11

    out = host_lib_path()
    with _lock("host"):
        if not force and not _stale(out, HOST_SRC):
            return out
        digest = _digest(HOST_SRC)
        out.parent.mkdir(parents=True, exist_ok=True)
        cmd = [
            _cxx(),
            "-O2",
            "-std=c++17",
            "-shared",
            "-fPIC",
            "-Wall",
            "-fvisibility=hidden",
            f"-I{pybind11.get_include()}",
            f"-I{sysconfig.get_paths()['include']}",
            *[str(s) for s in HOST_SRC],
            "-o",
            str(out) + ".tmp",
            "-lpthread",
        ]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(str(out) + ".tmp", out)
        _stamp(out, digest)
    return out


def cuda_sources() -> list[Path]:
    return sorted(CUDA_DIR.glob("*.cu")) + sorted(CUDA_DIR.glob("*.cpp"))


def cuda_headers() -> list[Path]:
    return sorted(CUDA_DIR.glob("*.cuh")) + sorted(CUDA_DIR.glob("*.h")) + sorted(INCLUDE_DIR.glob("*.h"))


def build_cuda(force: bool = False, verbose: bool = False) -> Path:
    """Compile every sm_100a kernel into one torch extension (ninja, parallel)."""
    from torch.utils import cpp_extension

    out = cuda_lib_path()
    with _lock("cuda"):
        deps = cuda_sources() + cuda_headers()
        if not force and not _stale(out, deps, " ".join(NVCC_FLAGS)):
            return out
        digest = _digest(deps, " ".join(NVCC_FLAGS))
        os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
        os.environ["CXX"] = _cxx()
        os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
        bdir = out.parent
        bdir.mkdir(parents=True, exist_ok=True)
        if force:
            for f in glob.glob(str(bdir / "*.o")):
                os.remove(f)
        cpp_extension.load(
            name="_cuda",
            sources=[str(s) for s in cuda_sources()],
            extra_cflags=["-O3", "-std=c++17"],
            extra_cuda_cflags=NVCC_FLAGS + [f"-I{CUDA_DIR}"],
            extra_ldflags=["-lcuda"],
            extra_include_paths=[str(CUDA_DIR)],
            build_directory=str(bdir),
            verbose=verbose,
            with_cuda=True,
            is_python_module=True,
        )
        _stamp(out, digest)
    return out


def _import_from(path: Path, name: str):
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    assert spec is not None
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


_HOST = None
_CUDA = None


def host_ext():
    """The native transport module, built on first use if absent or stale."""
    global _HOST
    if _HOST is None:
        path = host_lib_path()
        if _stale(path, HOST_SRC):
            build_host()
        _HOST = _import_from(path, "_host")
    return _HOST


def cuda_ext():
    """The sm_100a kernel module.  Raises if it cannot be built or loaded."""
    global _CUDA
    if _CUDA is None:
        import torch  # noqa: F401  (the extension links against torch's libraries)

        path = cuda_lib_path()
        if _stale(path, cuda_sources() + cuda_headers(), " ".join(NVCC_FLAGS)):
            build_cuda()
        _CUDA = _import_from(path, "_cuda")
    return _CUDA


if __name__ == "__main__":
    build_host(force="--force" in sys.argv, verbose=True)
    if "--host-only" not in sys.argv:
        build_cuda(force="--force" in sys.argv, verbose=True)
    print("built", host_lib_path(), cuda_lib_path())
