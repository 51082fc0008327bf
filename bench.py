#!/usr/bin/env python
"""Headline benchmark: GPT training tokens/s per box (DDP).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|torch]

Model: decoder-only GPT, 12 layers, d_model 768, 12 heads, vocab 50304,
sequence 1024, learned positions, MLP 4x, tied head (124M parameters),
random init.  Data: synthetic uniform token ids.  Micro-batch 16 sequences
per GPU, data parallel over N GPUs with 25 MB gradient buckets, AdamW
(0.9, 0.95, wd 0.1), bf16 compute with fp32 master weights.

For N > 1 launch with torchrun (one process per GPU):

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port P bench.py --gpus N

Two timed phases, each of exactly K steps after W warm-up steps, bracketed
by a barrier and torch.cuda.synchronize() on both sides, max over ranks:

1. ``value``: device time (CUDA events) of K training steps whose batches
   are already resident on the device;
2. ``e2e``: wall time of K steps through the public API where every step
   copies that step's inputs from pinned host memory and reads the loss back
   to the host.  The synthetic batches are made the way a data loader makes
   them: batch i+1 is drawn on the CPU while step i runs on the GPU (two
   pinned buffers per input), the same in every arm.

``--mode 3d`` runs BASELINE config 5: GPT 32 layers, d_model 4096, 32 heads,
sequence 2048, on a tp x pp x dp mesh (N=8: 2 x 2 x 2; N=4: 2 x 2 x 1; N=2:
2 x 1 x 1), 1F1B over 8 microbatches of 2 sequences per pipeline, sequence-
parallel TP whose GEMM / collective pairs run as fused kernels, stage
send/recv over NCCL p2p; total work per step is fixed (strong scaling).

``--mode fsdp`` runs BASELINE config 4 instead: GPT 24 layers, d_model 2048,
16 heads, sequence 2048, micro-batch 4 per GPU, one FSDP unit per block with
parameters, gradients and AdamW state sharded N ways (fp32 master weights;
ours fuses each block's AdamW step into its gradient reduce-scatter, and
keeps activations rather than recomputing -- torch FSDP2's default).

Arms: ``ours`` (this library: sm_100a kernels, peer-memory DDP all-reduce),
``reference`` (the unmodified reference package from baseline/_ref with its
own example GPT; gradients averaged with its GPU entry point
``mini_nccl.device.all_reduce_staged``), ``torch`` (torch DDP over NCCL with
the same model in autocast -- the NCCL+cuBLAS baseline).
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REF_ROOT = ROOT / "baseline" / "_ref"

VOCAB = 50304
BUCKET_MB = 25.0
# (layers, d_model, heads, seq, micro-batch per GPU) of each BASELINE config
MODES = {
    "ddp": dict(layers=12, embd=768, heads=12, seq=1024, micro=16, metric="GPT tok/s/box (DDP)"),
    "fsdp": dict(layers=24, embd=2048, heads=16, seq=2048, micro=4, metric="GPT tok/s/box (FSDP)"),
    # 3D: micro = sequences per microbatch; MICROBATCHES of them per pipeline per step
    "3d": dict(layers=32, embd=4096, heads=32, seq=2048, micro=2, metric="GPT tok/s/box (3D TPxPPxDP)"),
}
MICROBATCHES = 8


def mesh_dims(world: int) -> tuple[int, int, int]:
    """(dp, pp, tp) for the 3D config on N GPUs: tp first, then pp, then dp."""
    return {1: (1, 1, 1), 2: (1, 1, 2), 4: (1, 2, 2), 8: (2, 2, 2)}[world]
LAYERS, EMBD, HEADS, SEQ, MICRO_BATCH = 12, 768, 12, 1024, 16  # the default (DDP) config
METRIC = MODES["ddp"]["metric"]


def set_mode(mode: str) -> None:
    """Point the module-level config at one BASELINE config."""
    global LAYERS, EMBD, HEADS, SEQ, MICRO_BATCH, METRIC
    m = MODES[mode]
    LAYERS, EMBD, HEADS, SEQ, MICRO_BATCH, METRIC = m["layers"], m["embd"], m["heads"], m["seq"], m["micro"], m["metric"]


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "torch"], default="ours")
    ap.add_argument("--mode", choices=sorted(MODES), default="ddp",
                    help="ddp: config 3 (default); fsdp: config 4; 3d: config 5 (N in 1, 2, 4, 8)")
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end phase")
    ap.add_argument("--ddp-optimizer", choices=["fused", "separate"], default="separate",
                    help="--mode ddp, N > 1: AdamW inside each gradient bucket's reduction on 1/N of the "
                         "parameters per rank (fused), or one AdamW step over all parameters after backward")
    ap.add_argument("--fsdp-gather", choices=["fused", "prefetch"], default="fused",
                    help="--mode fsdp: gather each block's parameters inside its first GEMM (fused) or "
                         "with a separate all-gather prefetched on a side stream")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks: NVML sampled in a thread during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(2.0)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        mhz = [s for s, _ in self.samples]
        seen = 0
        for _, r in self.samples:
            seen |= r
        names = sorted(n for n, bit in self.REASONS.items() if seen & bit and n != "gpu_idle")
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(mhz)}


# ---------------------------------------------------------------------------
# shared harness
# ---------------------------------------------------------------------------
def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def batches_on_device(torch, n, B, dev, seed):
    g = torch.Generator().manual_seed(seed)
    xs = [torch.randint(0, VOCAB, (B, SEQ), generator=g).to(dev) for _ in range(n)]
    ys = [torch.randint(0, VOCAB, (B, SEQ), generator=g).to(dev) for _ in range(n)]
    return xs, ys


class HostBatches:
    """Random (x, y) token batches in pinned host memory, one step ahead.

    ``current()`` is this step's pair; ``advance()`` (called once the step's
    work is enqueued) draws the next pair on the CPU while the GPU runs.  Two
    buffers per input: the pair being drawn was last copied to the device by
    the previous step, whose result the caller has already read back.
    """

    def __init__(self, torch, rows: int, seq: int, vocab: int, seed: int) -> None:
        self.torch = torch
        self.vocab = vocab
        self.gen = torch.Generator().manual_seed(seed)
        self.bufs = [tuple(torch.empty((rows, seq), dtype=torch.int64).pin_memory() for _ in range(2))
                     for _ in range(2)]
        self.turn = 0
        self._draw(0)

    def _draw(self, k: int) -> None:
        for t in self.bufs[k]:
            self.torch.randint(0, self.vocab, t.shape, generator=self.gen, out=t)

    def current(self):
        return self.bufs[self.turn]

    def advance(self) -> None:
        self.turn ^= 1
        self._draw(self.turn)


def run_phases(torch, args, step_fn, barrier, reduce_max, dev, clocks: ClockSampler, e2e_step=None):
    """Warm-up, device-timed phase, optional e2e phase.  Returns (ms, e2e_ms, launches)."""
    from mini_nccl_b200.utils import launches

    for i in range(args.warmup):
        step_fn(i)
    barrier()
    torch.cuda.synchronize()
    launches.reset()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clocks:
        barrier()
        torch.cuda.synchronize()
        start.record()
        for i in range(args.steps):
            step_fn(i)
        end.record()
        torch.cuda.synchronize()
        barrier()
    n_launch = launches.count()
    ms = reduce_max(start.elapsed_time(end))
    e2e_ms = None
    if e2e_step is not None and not args.no_e2e:
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = reduce_max((time.perf_counter() - t0) * 1e3)
    return ms, e2e_ms, n_launch


def emit(args, world, impl, ms, e2e_ms, clocks, launches, extra=None):
    if args.mode == "3d":
        dp, pp, tp = mesh_dims(world)
        seqs = dp * MICROBATCHES * args.micro_batch  # per step, whole job
    else:
        seqs = world * args.micro_batch
    tokens = seqs * SEQ * args.steps
    value = tokens / (ms / 1e3)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "strong" if args.mode == "3d" else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic uniform token ids, random-init weights",
        "config": {
            "model": f"GPT {LAYERS}L/{EMBD}/{HEADS}H V{VOCAB} T{SEQ}"
                     + (" (head untied: it lives on the last pipeline stage)" if args.mode == "3d" else " (tied head)"),
            "global_batch": seqs,
            "micro_batch_per_gpu": args.micro_batch,
            "seq_len": SEQ,
            "parallelism": (("tp{2}xpp{1}xdp{0}, 1F1B x{3} microbatches, sequence parallel".format(
                *mesh_dims(world), MICROBATCHES)) if args.mode == "3d"
                else f"{args.mode if args.mode != 'ddp' else 'dp'}{world}"),
            "bucket_mb": BUCKET_MB if args.mode == "ddp" else None,
            "optimizer": "AdamW(0.9,0.95,wd0.1), fp32 master" + (
                ", inside each bucket's reduction on 1/N of the parameters per rank"
                if args.mode == "ddp" and getattr(args, "ddp_optimizer", "") == "fused" and world > 1
                and impl == "ours" else ""),
            "l2": "no flush: per-step working set (activations, params, grads, Adam state) >> 126 MB L2",
        },
        "clocks": clocks.summary(),
        "impl": impl,
    }
    if e2e_ms is not None:
        line["e2e"] = {
            "value": round(tokens / (e2e_ms / 1e3), 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": (2 * MICROBATCHES if args.mode == "3d" else 2) * args.micro_batch * SEQ * 8,
            "d2h_bytes_per_step": 4,
            "ms_per_step": round(e2e_ms / args.steps, 3),
        }
    if launches is not None:
        line["gpu_launches"] = launches
    if extra:
        line.update(extra)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# ours
# ---------------------------------------------------------------------------
def run_ours_3d(args):
    """Config 5: tensor x pipeline x data parallel GPT (fused TP kernels, 1F1B over NCCL p2p)."""
    import torch

    sys.path.insert(0, str(ROOT))
    import mini_nccl_b200 as mn
    from mini_nccl_b200.models.tp_gpt import GPTStage, sync_tensor_parallel_grads
    from mini_nccl_b200.ops.kernels import FusedAdamW

    rank, world, local = env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dp, pp, tp = mesh_dims(world)
    if world > 1:
        pg = mn.init_process_group(rank, world, device=dev, op_timeout=300.0, nccl_p2p=pp > 1)
    else:
        pg = mn.ProcessGroup(0, 1, device=dev)
    mesh = mn.ParallelMesh(pg, dp=dp, pp=pp, tp=tp)
    dpg, ppg, tpg = mesh.group("dp"), mesh.group("pp"), mesh.group("tp")
    d, s = mesh.coordinate("dp"), mesh.coordinate("pp")
    torch.manual_seed(1000 + s)  # replicated parameters identical across the tp group and the replicas
    with torch.device(dev):  # billions of parameters: initialise on the GPU
        stage = GPTStage(VOCAB, SEQ, LAYERS, HEADS, EMBD, tpg, s, pp, sequence_parallel=tp > 1)
    stage = stage.to(torch.bfloat16)
    B = args.micro_batch
    act = (SEQ // tp, B, EMBD) if tp > 1 else (B, SEQ, EMBD)
    pipe = mn.PipelineParallel(stage, ppg, activation_shape=act, loss_fn=stage.loss if s == pp - 1 else None,
                               schedule="1f1b", dtype=torch.bfloat16, device=dev)
    opt = FusedAdamW(stage.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    first, last = s == 0, s == pp - 1
    n_seq = MICROBATCHES * B
    xs, ys = batches_on_device(torch, 2, n_seq, dev, seed=1000 + d)
    params = list(stage.parameters())

    def train(x, y):
        opt.zero_grad(set_to_none=True)
        loss = pipe.step(x if first else None, y if last else None, n_microbatches=MICROBATCHES)
        sync_tensor_parallel_grads(stage, tpg)
        if dp > 1:
            mn.average_gradients(dpg, params)
        opt.step()
        return loss

    def step(i):
        train(xs[i % 2], ys[i % 2])

    host = HostBatches(torch, n_seq, SEQ, VOCAB, seed=77 + d)
    losses = []

    def e2e_step(i):
        hx, hy = host.current()
        x = hx.to(dev, non_blocking=True) if first else None
        y = hy.to(dev, non_blocking=True) if last else None
        loss = train(x, y)  # the pipeline returns the loss as a host float on the last stage
        host.advance()
        losses.append(loss)

    def barrier():
        if world > 1:
            mn.collectives.barrier(pg)

    def reduce_max(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        mn.collectives.all_reduce(pg, t, op="max")
        return float(t.item())

    clocks = ClockSampler(dev.index)
    ms, e2e_ms, n_launch = run_phases(torch, args, step, barrier, reduce_max, dev, clocks, e2e_step)
    if world > 1:
        pg.device_comm().synchronize()
    final = torch.tensor([losses[-1] if (losses and last) else 0.0], dtype=torch.float64)
    if world > 1:
        mn.collectives.all_reduce(pg, final, op="max")
    if rank == 0:
        emit(args, world, "ours", ms, e2e_ms, clocks, n_launch, {"final_loss": round(float(final.item()), 4)})
    pg.close()


def run_ours(args):
    import torch

    if args.mode == "3d":
        return run_ours_3d(args)
    sys.path.insert(0, str(ROOT))
    import mini_nccl_b200 as mn
    from mini_nccl_b200.models.gpt import GPT
    from mini_nccl_b200.ops.kernels import FusedAdamW

    rank, world, local = env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        pg = mn.init_process_group(rank, world, device=dev, op_timeout=120.0)
    else:
        pg = mn.ProcessGroup(0, 1, device=dev)
    torch.manual_seed(0)
    model = GPT(VOCAB, SEQ, LAYERS, HEADS, EMBD).to(dev, torch.bfloat16)
    hp = dict(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    if args.mode == "fsdp":
        from mini_nccl_b200.models.gpt import Block

        # one unit per block; each block's AdamW runs inside its gradient reduce-scatter
        # activations saved (as torch FSDP2 does by default); parameters still freed after each
        # block's forward and gathered again for its backward
        # fused: each block's parameter all-gather runs inside its QKV GEMM (one kernel);
        # prefetch: a separate all-gather of the next block on a side stream
        ddp = mn.FullyShardedDataParallel(model, pg, unit_cls=Block, prefetch=True, recompute=False,
                                          optimizer_in_backward=dict(hp, eps=1e-8),
                                          fuse_gather_gemm=args.fsdp_gather == "fused" and world > 1)
        shard_ids = {id(u.shard) for u in ddp.units}
        opt = FusedAdamW([p for p in ddp.parameters() if id(p) not in shard_ids], **hp)
    elif args.ddp_optimizer == "fused" and world > 1:
        # AdamW inside each bucket's reduction: every rank updates its 1/W slice, new parameters by all-gather
        ddp = mn.DistributedDataParallel(model, pg, bucket_cap_mb=BUCKET_MB, overlap=True, algorithm="auto",
                                         optimizer_in_backward=dict(hp, eps=1e-8))
        rest = ddp.unbucketed_parameters()
        opt = FusedAdamW(rest, **hp) if rest else None
    else:
        ddp = mn.DistributedDataParallel(model, pg, bucket_cap_mb=BUCKET_MB, overlap=True, algorithm="auto")
        opt = FusedAdamW(model.parameters(), **hp)
    B = args.micro_batch
    xs, ys = batches_on_device(torch, 4, B, dev, seed=1000 + rank)

    def step(i):
        ddp.zero_grad()
        _, loss = ddp(xs[i % 4], ys[i % 4])
        loss.backward()
        ddp.sync()
        if opt is not None:
            opt.step()
        return loss

    host = HostBatches(torch, B, SEQ, VOCAB, seed=77 + rank)
    losses = []

    def e2e_step(i):
        hx, hy = host.current()
        x = hx.to(dev, non_blocking=True)
        y = hy.to(dev, non_blocking=True)
        ddp.zero_grad()
        _, loss = ddp(x, y)
        loss.backward()
        ddp.sync()
        if opt is not None:
            opt.step()
        host.advance()
        losses.append(loss.item())

    def barrier():
        if world > 1:
            mn.collectives.barrier(pg)

    def reduce_max(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        mn.collectives.all_reduce(pg, t, op="max")
        return float(t.item())

    clocks = ClockSampler(dev.index)
    ms, e2e_ms, n_launch = run_phases(torch, args, step, barrier, reduce_max, dev, clocks, e2e_step)
    if world > 1:
        pg.device_comm().synchronize()
    if rank == 0:
        emit(args, world, "ours", ms, e2e_ms, clocks, n_launch,
             {"final_loss": round(losses[-1], 4) if losses else None})
    pg.close()


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def _store_addrs(torch, rank, world):
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from mini_nccl_b200.launcher import _free_ports

    store = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"]), world,
                          is_master=False, timeout=timedelta(seconds=300))
    run_id = os.environ.get("TORCHELASTIC_RUN_ID", "bench")
    store.set(f"ref/{run_id}/{rank}", str(_free_ports(1)[0]))
    ports = []
    for r in range(world):
        store.wait([f"ref/{run_id}/{r}"])
        ports.append(int(store.get(f"ref/{run_id}/{r}")))
    return [("127.0.0.1", p) for p in ports]


def run_reference(args):
    rank, world, local = env_rank()
    if args.mode != "ddp":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable":
                              f"the reference's {args.mode} path moves tensors over TCP from host memory only "
                              "(mini_nccl/transport.py byte_view); it has no GPU path for this config"}))
        return
    if not (REF_ROOT / "mini_nccl" / "__init__.py").exists() or not (REF_ROOT / "examples" / "model.py").exists():
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable":
                              "baseline/_ref not installed (pip install --target baseline/_ref of the reference)"}))
        return
    import torch

    sys.path.insert(0, str(REF_ROOT))
    import mini_nccl as rmn
    from mini_nccl import device as rdev

    spec = importlib.util.spec_from_file_location("ref_example_model", REF_ROOT / "examples" / "model.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        pg = rmn.ProcessGroup(rank, world, addrs=_store_addrs(torch, rank, world))
    torch.manual_seed(0)
    model = mod.GPT(vocab_size=VOCAB, block_size=SEQ, n_layer=LAYERS, n_head=HEADS, n_embd=EMBD).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    B = args.micro_batch
    xs, ys = batches_on_device(torch, 4, B, dev, seed=1000 + rank)
    params = [p for p in model.parameters()]

    def train(x, y):
        opt.zero_grad(set_to_none=False)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = model(x, y)
        loss.backward()
        if world > 1:
            grads = [p.grad for p in params if p.grad is not None]
            flat = torch.cat([g.reshape(-1) for g in grads])
            rdev.all_reduce_staged(pg, flat)
            flat.div_(world)
            at = 0
            for g in grads:
                g.copy_(flat[at : at + g.numel()].view_as(g))
                at += g.numel()
        opt.step()
        return loss

    def step(i):
        return train(xs[i % 4], ys[i % 4])

    host = HostBatches(torch, B, SEQ, VOCAB, seed=77 + rank)

    def e2e_step(i):
        hx, hy = host.current()
        loss = train(hx.to(dev, non_blocking=True), hy.to(dev, non_blocking=True))
        host.advance()
        loss.item()

    def barrier():
        if pg is not None:
            rmn.collectives.barrier(pg)

    def reduce_max(v):
        if pg is None:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        rmn.collectives.all_reduce(pg, t, op="max")
        return float(t.item())

    clocks = ClockSampler(dev.index)
    sys.path.insert(0, str(ROOT))
    ms, e2e_ms, _ = run_phases(torch, args, step, barrier, reduce_max, dev, clocks, e2e_step)
    if rank == 0:
        emit(args, world, "reference", ms, e2e_ms, clocks, None,
             {"reference_path": "examples/model.py GPT + torch.optim.AdamW; grads via mini_nccl.device.all_reduce_staged"})
    if pg is not None:
        pg.close()


# ---------------------------------------------------------------------------
# torch DDP + NCCL baseline
# ---------------------------------------------------------------------------
def run_torch(args):
    import torch
    import torch.distributed as dist

    if args.mode == "3d":
        return run_torch_3d(args)

    sys.path.insert(0, str(ROOT))
    from mini_nccl_b200.models.gpt import GPT

    rank, world, local = env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    torch.manual_seed(0)
    model = GPT(VOCAB, SEQ, LAYERS, HEADS, EMBD).to(dev)  # fp32 params, autocast bf16 compute
    B = args.micro_batch
    xs, ys = batches_on_device(torch, 4, B, dev, seed=1000 + rank)
    import torch.nn.functional as F

    class StockBlock(torch.nn.Module):
        """One block of the same parameters through stock torch ops (cuBLAS, SDPA)."""

        def __init__(self, blk):
            super().__init__()
            self.ln1, self.qkv, self.proj, self.ln2, self.mlp = blk.ln1, blk.qkv, blk.proj, blk.ln2, blk.mlp
            self.n_head = blk.n_head

        def forward(self, h):
            Bq, T, C = h.shape
            q, k, v = self.qkv(self.ln1(h)).split(C, dim=-1)
            q, k, v = (t.view(Bq, T, self.n_head, C // self.n_head).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            h = h + self.proj(a.transpose(1, 2).reshape(Bq, T, C))
            return h + self.mlp(self.ln2(h))

    class StockGPT(torch.nn.Module):
        def __init__(self, m):
            super().__init__()
            self.tok_emb, self.pos_emb, self.ln_f, self.head = m.tok_emb, m.pos_emb, m.ln_f, m.head
            self.blocks = torch.nn.ModuleList(StockBlock(b) for b in m.blocks)

        def forward(self, x, y):
            T = x.shape[1]
            h = self.tok_emb(x) + self.pos_emb[:, :T]
            for blk in self.blocks:
                h = blk(h)
            logits = self.head(self.ln_f(h))
            return F.cross_entropy(logits.view(-1, logits.shape[-1]).float(), y.view(-1))

    net = StockGPT(model)
    if world > 1 and args.mode == "fsdp":
        from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

        mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
        for blk in net.blocks:
            fully_shard(blk, mp_policy=mp)
        fully_shard(net, mp_policy=mp)
    elif world > 1:
        net = torch.nn.parallel.DistributedDataParallel(net, bucket_cap_mb=BUCKET_MB)
    opt = torch.optim.AdamW(net.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)

    def train(x, y):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = net(x, y)
        loss.backward()
        opt.step()
        return loss

    def step(i):
        return train(xs[i % 4], ys[i % 4])

    host = HostBatches(torch, B, SEQ, VOCAB, seed=77 + rank)

    def e2e_step(i):
        hx, hy = host.current()
        loss = train(hx.to(dev, non_blocking=True), hy.to(dev, non_blocking=True))
        host.advance()
        loss.item()

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce_max(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(dev.index)
    ms, e2e_ms, _ = run_phases(torch, args, step, barrier, reduce_max, dev, clocks, e2e_step)
    if rank == 0:
        emit(args, world, "torch", ms, e2e_ms, clocks, None)
    if world > 1:
        dist.destroy_process_group()



def run_torch_3d(args):
    """Config 5 on stock torch + NCCL: the Megatron-style baseline.

    Same mesh, model shape, microbatching and optimizer as ``run_ours_3d``;
    every op is stock PyTorch under bf16 autocast (cuBLAS GEMMs, SDPA flash
    attention, fused AdamW) and every transfer is NCCL through
    torch.distributed: tensor parallelism as Megatron's column / row split
    with an all-reduce after each row-parallel GEMM (forward) and before each
    column-parallel one (backward), 1F1B over NCCL send / recv on the pp
    group, and a data-parallel all-reduce of the gradients after the
    pipeline drains.
    """
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    from torch import nn

    rank, world, local = env_rank()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dp, pp, tp = mesh_dims(world)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    # rank = (d * pp + s) * tp + t  (last dimension fastest, as ParallelMesh lays it out)
    d, s, t = rank // (pp * tp), (rank // tp) % pp, rank % tp
    groups = {}
    if world > 1:
        for name, members in (("tp", [[(dd * pp + ss) * tp + tt for tt in range(tp)] for dd in range(dp)
                                      for ss in range(pp)]),
                              ("pp", [[(dd * pp + ss) * tp + tt for ss in range(pp)] for dd in range(dp)
                                      for tt in range(tp)]),
                              ("dp", [[(dd * pp + ss) * tp + tt for dd in range(dp)] for ss in range(pp)
                                      for tt in range(tp)])):
            for m in members:
                g = dist.new_group(m)  # every rank creates every group, in the same order
                if rank in m:
                    groups[name] = (g, m)

    class ToTP(torch.autograd.Function):  # identity forward, all-reduce of the input gradient
        @staticmethod
        def forward(ctx, x):
            return x

        @staticmethod
        def backward(ctx, g):
            g = g.contiguous()
            dist.all_reduce(g, group=groups["tp"][0])
            return g

    class FromTP(torch.autograd.Function):  # all-reduce of the partial sums, identity backward
        @staticmethod
        def forward(ctx, x):
            x = x.contiguous()
            dist.all_reduce(x, group=groups["tp"][0])
            return x

        @staticmethod
        def backward(ctx, g):
            return g

    C, H = EMBD, HEADS
    hl = H // tp  # heads on this rank

    class TPBlock(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln1, self.ln2 = nn.LayerNorm(C), nn.LayerNorm(C)
            self.qkv = nn.Linear(C, 3 * C // tp)           # column parallel: this rank's q, k, v heads
            self.proj = nn.Linear(C // tp, C, bias=False)  # row parallel (bias added once, after the sum)
            self.proj_b = nn.Parameter(torch.zeros(C))
            self.fc1 = nn.Linear(C, 4 * C // tp)
            self.fc2 = nn.Linear(4 * C // tp, C, bias=False)
            self.fc2_b = nn.Parameter(torch.zeros(C))

        def forward(self, h):  # h [B, T, C], replicated over the tp group
            Bq, T, _ = h.shape
            x = self.ln1(h)
            if tp > 1:
                x = ToTP.apply(x)
            q, k, v = self.qkv(x).view(Bq, T, 3, hl, C // H).permute(2, 0, 3, 1, 4)
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(Bq, T, C // tp)
            y = self.proj(a)
            h = h + (FromTP.apply(y) if tp > 1 else y) + self.proj_b
            x = self.ln2(h)
            if tp > 1:
                x = ToTP.apply(x)
            y = self.fc2(F.gelu(self.fc1(x)))
            return h + (FromTP.apply(y) if tp > 1 else y) + self.fc2_b

    class Stage(nn.Module):
        def __init__(self):
            super().__init__()
            self.first, self.last = s == 0, s == pp - 1
            if self.first:
                self.tok_emb = nn.Embedding(VOCAB, C)
                self.pos_emb = nn.Parameter(torch.zeros(1, SEQ, C))
            self.blocks = nn.ModuleList(TPBlock() for _ in range(LAYERS // pp))
            if self.last:
                self.ln_f = nn.LayerNorm(C)
                self.head = nn.Linear(C, VOCAB, bias=False)

        def forward(self, x):
            h = self.tok_emb(x) + self.pos_emb if self.first else x
            for blk in self.blocks:
                h = blk(h)
            return self.head(self.ln_f(h)) if self.last else h

    torch.manual_seed(1000 + s)  # replicated parameters identical across the tp group and the replicas
    torch.cuda.manual_seed(1000 + s)
    with torch.device(dev):
        stage = Stage()
    for p in stage.parameters():  # N(0, 0.02) like the model of the other arms; LayerNorm stays (1, 0)
        if p.dim() > 1:
            nn.init.normal_(p, 0.0, 0.02)
    opt = torch.optim.AdamW(stage.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    B = args.micro_batch
    M = MICROBATCHES
    n_seq = M * B
    xs, ys = batches_on_device(torch, 2, n_seq, dev, seed=1000 + d)
    params = [p for p in stage.parameters()]
    pp_group, pp_ranks = groups.get("pp", (None, [rank]))
    prev_rank = pp_ranks[s - 1] if s > 0 else None
    next_rank = pp_ranks[s + 1] if s < pp - 1 else None
    act_shape = (B, SEQ, C)

    def p2p(send=None, to=None, recv_from=None):
        ops, buf = [], None
        if send is not None:
            ops.append(dist.P2POp(dist.isend, send.contiguous(), to, group=pp_group))
        if recv_from is not None:
            buf = torch.empty(act_shape, dtype=torch.bfloat16, device=dev)
            ops.append(dist.P2POp(dist.irecv, buf, recv_from, group=pp_group))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        return buf

    first, last = s == 0, s == pp - 1

    # Paired NCCL point-to-point steps of the 1F1B schedule (every send is
    # posted together with the receive its neighbour pairs it with).
    def recv_forward():
        return None if first else p2p(recv_from=prev_rank)

    def send_forward(out):
        if not last:
            p2p(send=out.detach().to(torch.bfloat16), to=next_rank)

    def send_forward_recv_backward(out):
        return None if last else p2p(send=out.detach().to(torch.bfloat16), to=next_rank, recv_from=next_rank)

    def send_backward_recv_forward(g):
        return None if first else p2p(send=g.to(torch.bfloat16), to=prev_rank, recv_from=prev_rank)

    def send_backward(g):
        if not first:
            p2p(send=g.to(torch.bfloat16), to=prev_rank)

    def recv_backward():
        return None if last else p2p(recv_from=next_rank)

    def train(x, y):
        opt.zero_grad(set_to_none=True)
        queue = []
        losses = []

        def forward(k, inp):
            if inp is not None:
                inp.requires_grad_(True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = stage(x[k * B:(k + 1) * B] if first else inp)
                if last:
                    out = F.cross_entropy(out.float().view(-1, VOCAB), y[k * B:(k + 1) * B].reshape(-1)) / M
                    losses.append(out.detach())
            queue.append((inp, out))
            return out

        def backward(grad):
            inp, out = queue.pop(0)  # the oldest microbatch in flight
            if last:
                out.backward()
            else:
                out.backward(grad.to(out.dtype))
            return inp.grad if inp is not None else None

        warm = min(pp - 1 - s, M)
        for k in range(warm):
            send_forward(forward(k, recv_forward()))
        inp = recv_forward() if warm < M else None
        for k in range(warm, M):
            g_out = send_forward_recv_backward(forward(k, inp))
            g_in = backward(g_out)
            if k == M - 1:
                send_backward(g_in)
                inp = None
            else:
                inp = send_backward_recv_forward(g_in)
        for _ in range(warm):
            send_backward(backward(recv_backward()))
        if dp > 1:  # average over the data-parallel replicas: NCCL all-reduces queued back to back
            works = [dist.all_reduce(p.grad, group=groups["dp"][0], async_op=True) for p in params
                     if p.grad is not None]
            for w in works:
                w.wait()
            torch._foreach_div_([p.grad for p in params if p.grad is not None], float(dp))
        opt.step()
        return torch.stack(losses).sum() if losses else None

    def step(i):
        train(xs[i % 2], ys[i % 2])

    host = HostBatches(torch, n_seq, SEQ, VOCAB, seed=77 + d)
    final = [0.0]

    def e2e_step(i):
        hx, hy = host.current()
        loss = train(hx.to(dev, non_blocking=True) if s == 0 else None,
                     hy.to(dev, non_blocking=True) if s == pp - 1 else None)
        host.advance()
        if loss is not None:
            final[0] = float(loss.item())

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce_max(v):
        if world == 1:
            return v
        tt = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    clocks = ClockSampler(dev.index)
    ms, e2e_ms, _ = run_phases(torch, args, step, barrier, reduce_max, dev, clocks, e2e_step)
    loss_max = reduce_max(final[0])
    if rank == 0:
        emit(args, world, "torch", ms, e2e_ms, clocks, None, {"final_loss": round(loss_max, 4)})
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    set_mode(args.mode)
    if args.micro_batch is None:
        args.micro_batch = MICRO_BATCH
    _, world, _ = env_rank()
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    {"ours": run_ours, "reference": run_reference, "torch": run_torch}[args.impl](args)


if __name__ == "__main__":
    main()
