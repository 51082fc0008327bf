"""setuptools hook: compile both native extensions before the package is copied.

``pip install --no-build-isolation .`` runs :func:`mini_nccl_b200._build.build_host`
(the C++ TCP transport) and, when a CUDA toolkit is present,
:func:`mini_nccl_b200._build.build_cuda` (every sm_100a kernel, nvcc
``-gencode arch=compute_100a,code=sm_100a``; no GPU is needed to compile).
The libraries land in ``mini_nccl_b200/_build`` and ship as package data.
Set ``MNB_SKIP_CUDA_BUILD=1`` to install the CPU-only part.
"""

from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

from setuptools import setup
from setuptools.command.build_py import build_py

ROOT = Path(__file__).resolve().parent


class BuildNative(build_py):
    def run(self) -> None:
        sys.path.insert(0, str(ROOT))
        from mini_nccl_b200 import _build

        _build.build_host()
        if os.environ.get("MNB_SKIP_CUDA_BUILD") != "1" and shutil.which("nvcc") is not None:
            _build.build_cuda()
        super().run()


setup(cmdclass={"build_py": BuildNative})
