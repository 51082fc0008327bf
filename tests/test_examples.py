"""Smoke-run every example with a tiny config (CPU ranks, synthetic corpus).

Asserts each command exits cleanly and prints the line proving it did its
work; the parity tests cover correctness (reference strategy:
tests/test_examples.py:1-138).
"""

from __future__ import annotations

import ast
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
TINY = "--steps 2 --n-layer 2 --n-embd 32 --batch-size 4 --block-size 16"

EXAMPLES = [
    pytest.param(f"examples/train_gpt.py --world-size 2 {TINY}", "final loss:", id="train_gpt_ddp"),
    pytest.param(f"examples/train_gpt.py --world-size 2 --fsdp {TINY}", "peak while training", id="train_gpt_fsdp"),
    pytest.param(f"examples/tensor_parallel_gpt.py --world-size 2 {TINY}", "max disagreement:", id="tensor_parallel"),
    pytest.param(f"examples/tensor_parallel_gpt.py --world-size 2 --sequence-parallel {TINY}", "max disagreement:",
                 id="tensor_parallel_sp"),
    pytest.param(f"examples/pipeline_gpt.py --world-size 2 --microbatches 2 {TINY}",
                 "microbatches in flight per stage", id="pipeline"),
    pytest.param(f"examples/two_dimensional_gpt.py --world-size 2 --tp 2 {TINY}", "loss across the tensor group",
                 id="two_dimensional"),
]


def run_example(command: str, expect: str, timeout: float = 420.0) -> str:
    proc = subprocess.run([sys.executable, *command.split()], cwd=ROOT, capture_output=True, text=True,
                          timeout=timeout)
    if proc.returncode != 0:
        tail = "\n".join((proc.stdout + proc.stderr).splitlines()[-25:])
        pytest.fail(f"`{command}` exited {proc.returncode}:\n{tail}")
    if expect not in proc.stdout:
        pytest.fail(f"`{command}` never printed {expect!r}:\n" + "\n".join(proc.stdout.splitlines()[-25:]))
    return proc.stdout


@pytest.mark.examples
@pytest.mark.parametrize(("command", "expect"), EXAMPLES)
def test_example_runs(command: str, expect: str) -> None:
    run_example(command, expect)


@pytest.mark.examples
def test_desync_demo_produces_a_diagnosis() -> None:
    out = run_example("examples/desync_demo.py", "DESYNC at collective")
    assert "rank 2: barrier" in out, out[-800:]
    assert "CollectiveTimeoutError" in out, out[-800:]


@pytest.mark.examples
def test_three_dimensional_mesh_is_orthogonal() -> None:
    out = run_example(f"examples/three_dimensional_gpt.py --world-size 4 --pp 2 --tp 2 --microbatches 2 {TINY}",
                      "pipeline group")
    line = next(line for line in out.splitlines() if "pipeline group" in line)
    groups = [set(ast.literal_eval(part.split("group")[1].strip())) for part in line.split("|")]
    assert len(set.intersection(*groups)) == 1, line


@pytest.mark.examples
def test_multinode_allreduce_env_bootstrap() -> None:
    import os

    from mini_nccl_b200.launcher import _free_ports

    hosts = ",".join(f"127.0.0.1:{p}" for p in _free_ports(2))
    procs = [subprocess.Popen([sys.executable, "examples/multinode_allreduce.py", "--max-mib", "1", "--iters", "1"],
                              cwd=ROOT, env=dict(os.environ, MINI_NCCL_HOSTS=hosts, WORLD_SIZE="2", RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    assert "world_size=2" in outs[0] and "1048576" in outs[0], outs[0]


@pytest.mark.examples
def test_launch_multinode_script_runs_local_ranks(tmp_path) -> None:
    """The ssh launcher with every rank on this host (no ssh needed)."""
    from mini_nccl_b200.launcher import _free_ports

    port = _free_ports(1)[0]
    hosts = tmp_path / "hosts.txt"
    hosts.write_text(f"# two ranks on this machine\n127.0.0.1:{port}:2\n")
    out = subprocess.run(["bash", "examples/launch_multinode.sh", str(hosts), "examples/multinode_allreduce.py",
                          "--max-mib", "1", "--iters", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert f"hosts=127.0.0.1:{port},127.0.0.1:{port + 1}" in out.stdout
    assert "world_size=2" in out.stdout and "1048576" in out.stdout
