"""Shared pytest configuration.

Markers:
  gpu       needs a CUDA device (B200, sm_100a); excluded with -m "not gpu"
  multigpu  needs at least two CUDA devices (also marked gpu)
  examples  end-to-end example scripts (slower)
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
# Spawned workers import the package from the repository root too.
os.environ["PYTHONPATH"] = os.pathsep.join(
    [str(ROOT)] + [p for p in os.environ.get("PYTHONPATH", "").split(os.pathsep) if p]
)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")
    config.addinivalue_line("markers", "examples: runs an example script end to end")


def pytest_collection_modifyitems(config, items):
    for item in items:
        if "multigpu" in item.keywords and "gpu" not in item.keywords:
            item.add_marker(pytest.mark.gpu)
