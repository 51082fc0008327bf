#!/usr/bin/env python
"""Mutation check: plant one real bug at a time and demand that a test catches it.

    python tests/mutation_check.py            # every mutation that can run here
    python tests/mutation_check.py --strict   # also fail on anchors that no longer match
    python tests/mutation_check.py --list
    python tests/mutation_check.py --only ring-wrong-block,ddp-no-average

Each mutation is an exact-text patch of one source file plus the tests that
must fail once it is applied.  The checker applies the patch, runs those tests
(``pytest -x -q``), restores the file byte for byte, and reports the mutation
as *caught* (tests failed) or *survived*.  One control mutation changes
nothing observable and must survive: it proves the harness does not report
every patch as caught.  Mutations of CUDA-only code are skipped without a GPU.
(Same idea as the reference's scripts/mutation_check.py:59-397; the mutations
here are this library's own.)

Exit status: non-zero if any real mutation survives, if the control is
caught, or (``--strict``) if an anchor is missing.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import time
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


@dataclass
class Mutation:
    name: str
    path: str
    old: str
    new: str
    tests: list[str]
    why: str
    control: bool = False
    needs_gpu: bool = False


M = Mutation
MUTATIONS: list[Mutation] = [
    M("ring-wrong-block", "mini_nccl_b200/collectives.py",
      "            in_b = blocks[(r - s - 1) % W]\n",
      "            in_b = blocks[(r - s) % W]\n",
      ["tests/test_collectives.py::test_collective_battery"],
      "the reduce-scatter half folds the incoming partial into the wrong block"),
    M("ring-allgather-off-by-one", "mini_nccl_b200/collectives.py",
      "            out_b = blocks[(r + 1 - s) % W]\n",
      "            out_b = blocks[(r - s) % W]\n",
      ["tests/test_collectives.py::test_collective_battery"],
      "the all-gather half forwards a block this rank does not own yet"),
    M("tree-skips-a-child", "mini_nccl_b200/collectives.py",
      "        child = v + step\n        if child < W:\n",
      "        child = v + step\n        if child < W - 1:\n",
      ["tests/test_collectives.py::test_collective_battery"],
      "the last rank's contribution never reaches the root"),
    M("halving-wrong-half", "mini_nccl_b200/collectives.py",
      "        keep = padded[mid:hi] if upper else padded[lo:mid]\n",
      "        keep = padded[lo:mid] if upper else padded[mid:hi]\n",
      ["tests/test_collectives.py::test_collective_battery"],
      "both partners keep the same half"),
    M("naive-no-broadcast", "mini_nccl_b200/collectives.py",
      "    for dst in range(1, W):\n        pg.send(flat, dst)\n",
      "    for dst in range(1, W):\n        pg.send(flat.clone().zero_(), dst)\n",
      ["tests/test_collectives.py::test_collective_battery"],
      "rank 0 sends garbage instead of the result"),
    M("split-drops-remainder", "mini_nccl_b200/collectives.py",
      "    sizes = [q + (i < extra) for i in range(parts)]\n    return list(torch.split(flat, sizes))\n",
      "    sizes = [q for i in range(parts)]\n    return list(torch.split(flat[: q * parts], sizes))\n",
      ["tests/test_collectives.py::test_multichannel_large_allreduce"],
      "the last n % channels elements of a multi-channel all-reduce are never reduced"),
    M("wire-not-rounded", "mini_nccl_b200/collectives.py",
      "        view = self.out[: x.numel()]\n        view.copy_(x)\n        return view\n",
      "        return x\n",
      ["tests/test_low_precision.py"],
      "the narrow wire silently sends full precision"),
    M("ddp-no-average", "mini_nccl_b200/parallel/ddp.py",
      "                bucket.buffer.div_(self.pg.world_size)\n",
      "                pass\n",
      ["tests/test_ddp.py::test_tied_lm_trains_like_one_process"],
      "gradients are summed, not averaged"),
    M("ddp-no-sync-ignored", "mini_nccl_b200/parallel/ddp.py",
      "            if self._accumulating:\n                return  # inside no_sync()",
      "            if False:\n                return  # inside no_sync()",
      ["tests/test_ddp.py::test_no_sync_accumulates_three_microbatches"],
      "no_sync() still communicates"),
    M("ddp-bucket-order", "mini_nccl_b200/parallel/ddp.py",
      "        for p in reversed(list(self.module.parameters())):\n",
      "        for p in list(self.module.parameters()):\n",
      ["tests/test_ddp.py::test_a_dtype_change_starts_a_new_bucket"],
      "buckets follow registration order, so the first bucket to fill is reduced last"),
    M("fsdp-rng-not-replayed", "mini_nccl_b200/parallel/fsdp.py",
      "            torch.set_rng_state(self.cpu_state)\n",
      "            pass\n",
      ["tests/test_fsdp.py::test_recompute_replays_randomness"],
      "the recompute draws a fresh dropout mask"),
    M("fsdp-sum-not-mean", "mini_nccl_b200/parallel/fsdp.py",
      "        return collectives.reduce_scatter(self.pg, flat, op=\"sum\").div_(W)\n",
      "        return collectives.reduce_scatter(self.pg, flat, op=\"sum\")\n",
      ["tests/test_fsdp.py::test_fsdp_matches_single_process"],
      "shard gradients are summed over ranks"),
    M("tp-f-backward-no-allreduce", "mini_nccl_b200/parallel/tensor_parallel.py",
      "        if pg.world_size > 1:\n            grad = grad.contiguous()\n            collectives.all_reduce(pg, grad)\n"
      "        return None, grad\n",
      "        return None, grad\n",
      ["tests/test_tensor_parallel.py::test_parallel_mlp_matches_reference_world2"],
      "each rank's input gradient misses the other ranks' contributions"),
    M("tp-sp-grads-not-summed", "mini_nccl_b200/parallel/tensor_parallel.py",
      "    if pg.world_size == 1 or not grads:\n        return 0\n",
      "    if True:\n        return 0\n",
      ["tests/test_tensor_parallel.py::test_sequence_parallel_grads_match_single_process"],
      "replicated LayerNorm / bias gradients under sequence parallelism stay partial"),
    M("pipeline-lifo", "mini_nccl_b200/parallel/pipeline.py",
      "            x, out = self._queue.popleft()\n",
      "            x, out = self._queue.pop()\n",
      ["tests/test_pipeline.py::test_gradients_match_one_process"],
      "gradients are matched to the newest microbatch instead of the oldest"),
    M("pipeline-warmup-too-deep", "mini_nccl_b200/parallel/pipeline.py",
      "        warm = min(self.n_stages - 1 - self.rank, n)\n",
      "        warm = min(self.n_stages - self.rank, n)\n",
      ["tests/test_pipeline.py::test_1f1b_bounds_in_flight_microbatches"],
      "1F1B holds one microbatch more than W - s in flight"),
    M("mesh-first-dim-fastest", "mini_nccl_b200/mesh.py",
      "math.prod(sizes[i + 1:])",
      "math.prod(sizes[:i])",
      ["tests/test_mesh.py::test_mesh_layout_last_dimension_fastest"],
      "the rank layout no longer matches the documented last-dimension-fastest order"),
    M("recorder-seq-frozen", "mini_nccl_b200/recorder.py",
      "        self._next_seq[channel] = seq + 1\n",
      "        self._next_seq[channel] = seq\n",
      ["tests/test_faults.py::test_desync_times_out_with_diagnosis"],
      "every collective gets the same sequence number, so desyncs are invisible"),
    M("staging-no-stream-order", "mini_nccl_b200/device.py",
      "    staging.order_after_compute()\n",
      "    pass\n",
      ["tests/test_device_staging.py::test_every_exchange_orders_the_copy_stream_behind_compute"],
      "the copy stream may read a block before the compute stream has reduced into it"),
    M("ddp-comm-stream-no-producer-wait", "mini_nccl_b200/parallel/ddp.py",
      "                self._comm_stream.wait_event(produced)\n",
      "                pass\n",
      ["tests/test_stream_order_gpu.py::test_ddp_comm_stream_waits_for_every_bucket"],
      "a bucket's all-reduce may read the bucket before backward finished writing it", needs_gpu=True),
    M("fsdp-prefetch-no-wait", "mini_nccl_b200/parallel/fsdp.py",
      "        self._side.wait_stream(cur)\n        with torch.cuda.stream(self._side):\n"
      "            flat = nxt._gather(nxt.shard)\n",
      "        with torch.cuda.stream(self._side):\n            flat = nxt._gather(nxt.shard)\n",
      ["tests/test_stream_order_gpu.py::test_fsdp_side_and_comm_streams_wait_for_their_producers"],
      "the prefetched gather may run ahead of the compute stream it must follow", needs_gpu=True),
    M("fsdp-prefetched-used-unawaited", "mini_nccl_b200/parallel/fsdp.py",
      "        torch.cuda.current_stream(unit.device).wait_event(done)\n        return flat\n",
      "        return flat\n",
      ["tests/test_stream_order_gpu.py::test_fsdp_side_and_comm_streams_wait_for_their_producers"],
      "the compute stream may read prefetched parameters before their gather finished", needs_gpu=True),
    M("fsdp-reduce-scatter-no-wait", "mini_nccl_b200/parallel/fsdp.py",
      "            side.wait_stream(cur)\n            with torch.cuda.stream(side):\n",
      "            with torch.cuda.stream(side):\n",
      ["tests/test_stream_order_gpu.py::test_fsdp_side_and_comm_streams_wait_for_their_producers"],
      "a unit's gradient reduce-scatter may read gradients backward has not written yet", needs_gpu=True),
    M("splitk-ignores-partial-waves", "mini_nccl_b200/ops/kernels.py",
      "        waves = math.ceil(tiles * s_eff / NUM_SMS)\n",
      "        waves = tiles * s_eff / NUM_SMS\n",
      ["tests/test_gemm_planning.py"],
      "the split-K plan counts fractional waves, so a nearly empty last wave looks free"),
    M("host-batches-single-buffer", "bench.py",
      "        self.turn ^= 1\n",
      "        self.turn ^= 0\n",
      ["tests/test_bench_host_batches.py"],
      "the next batch is drawn into the buffer whose copy the current step just enqueued"),
    M("control-docstring", "mini_nccl_b200/collectives.py",
      "    \"\"\"Deterministic contiguous split; the first ``n % parts`` pieces get one extra.\"\"\"\n",
      "    \"\"\"Deterministic contiguous split (the first n % parts pieces get one extra).\"\"\"\n",
      ["tests/test_collectives.py::test_single_channel_still_correct"],
      "changes nothing observable: must survive", control=True),
]


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def run_one(m: Mutation, timeout: float) -> tuple[str, float]:
    path = ROOT / m.path
    original = path.read_bytes()
    text = original.decode()
    if text.count(m.old) != 1:
        return "stale-anchor", 0.0
    path.write_bytes(text.replace(m.old, m.new, 1).encode())
    t0 = time.perf_counter()
    try:
        proc = subprocess.run(
            [sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider", *m.tests],
            cwd=ROOT, capture_output=True, text=True, timeout=timeout,
            env={**os.environ, "PYTHONDONTWRITEBYTECODE": "1"},
        )
        failed = proc.returncode != 0
    except subprocess.TimeoutExpired:
        failed = True  # a hang introduced by the mutation counts as caught
    finally:
        path.write_bytes(original)
    return ("caught" if failed else "survived"), time.perf_counter() - t0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--strict", action="store_true")
    ap.add_argument("--list", action="store_true")
    ap.add_argument("--only", default="")
    ap.add_argument("--timeout", type=float, default=600.0)
    args = ap.parse_args()
    chosen = [m for m in MUTATIONS if not args.only or m.name in args.only.split(",")]
    if args.list:
        for m in chosen:
            print(f"{m.name:28s} {m.path:45s} {m.why}")
        return 0
    gpu = gpu_available()
    bad = 0
    for m in chosen:
        if m.needs_gpu and not gpu:
            print(f"SKIP      {m.name} (needs a GPU)")
            continue
        status, dt = run_one(m, args.timeout)
        expected = "survived" if m.control else "caught"
        ok = status == expected or (status == "stale-anchor" and not args.strict)
        bad += 0 if ok else 1
        print(f"{'OK' if ok else 'FAIL':9s} {m.name:28s} {status:12s} {dt:6.1f}s  {m.why}", flush=True)
    print(f"\n{len(chosen)} mutations, {bad} problem(s)")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
