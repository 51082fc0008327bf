"""Environment bootstrap: the multi-node contract and torchrun compatibility."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

from mini_nccl_b200 import _hosts_from_env
from mini_nccl_b200.launcher import _free_ports

WORKER = """
import torch
import mini_nccl_b200 as mn

pg = mn.init_process_group()
try:
    assert pg.world_size == 2, pg.world_size
    t = torch.full((300,), float(pg.rank + 1))
    mn.all_reduce(t)
    assert torch.all(t == 3.0), t
    got = mn.all_gather(torch.tensor([float(pg.rank)]))
    assert [g.item() for g in got] == [0.0, 1.0], got
    mn.barrier()
finally:
    mn.destroy_process_group()
print("OK", pg.rank)
"""


def test_hosts_from_env_parsing(monkeypatch) -> None:
    monkeypatch.setenv("MINI_NCCL_HOSTS", "10.1.2.3:29500, node-b:4000 ,")
    assert _hosts_from_env() == [("10.1.2.3", 29500), ("node-b", 4000)]
    monkeypatch.setenv("MINI_NCCL_HOSTS", "no-port-here")
    with pytest.raises(ValueError, match="host:port"):
        _hosts_from_env()
    monkeypatch.delenv("MINI_NCCL_HOSTS")
    assert _hosts_from_env() is None


def _spawn(env_for_rank) -> None:
    procs = []
    for rank in range(2):
        env = dict(os.environ, **env_for_rank(rank))
        env.pop("CUDA_VISIBLE_DEVICES", None)
        procs.append(subprocess.Popen(
            [sys.executable, "-c", WORKER], env=env,
            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
        ))
    for rank, p in enumerate(procs):
        out, _ = p.communicate(timeout=240)
        assert p.returncode == 0, f"rank {rank} failed:\n{out}"
        assert f"OK {rank}" in out, out


def test_two_independent_processes_rendezvous() -> None:
    hosts = ",".join(f"127.0.0.1:{p}" for p in _free_ports(2))
    _spawn(lambda r: {"MINI_NCCL_HOSTS": hosts, "WORLD_SIZE": "2", "RANK": str(r), "LOCAL_RANK": ""})


def test_torchrun_style_store_rendezvous() -> None:
    """Under torchrun, ranks exchange their ports through the launcher's store."""
    from datetime import timedelta

    import torch.distributed as dist

    port = _free_ports(1)[0]
    store = dist.TCPStore("127.0.0.1", port, 3, is_master=True, timeout=timedelta(seconds=60),
                          wait_for_workers=False)
    try:
        _spawn(lambda r: {
            "WORLD_SIZE": "2", "RANK": str(r), "MASTER_ADDR": "127.0.0.1",
            "MASTER_PORT": str(port), "TORCHELASTIC_RUN_ID": "unit-test",
            "MINI_NCCL_HOSTS": "",
        })
    finally:
        del store
