"""Train a character-level GPT data-parallel (DDP) or fully sharded (FSDP).

    python examples/train_gpt.py --world-size 4 --steps 200 --sample
    python examples/train_gpt.py --world-size 8 --device cuda --fsdp

Every gradient byte moves through this library: on CPU over its native TCP
mesh, on GPUs through its peer-memory all-reduce / reduce-scatter kernels.
Each rank samples its own batches (seed ``step*W + rank``); the loss printed
every 20 steps is averaged across ranks (reference:
examples/train_gpt.py:43-179).
"""

from __future__ import annotations

import argparse
import time

import torch

from _common import batch, encode, load_corpus, to_device

import mini_nccl_b200 as mn
from mini_nccl_b200 import collectives
from mini_nccl_b200.models.gpt import GPT, Block


def worker(pg, data: torch.Tensor, vocab: str, cfg: dict) -> float:
    torch.manual_seed(0)
    model = GPT(len(vocab), cfg["block_size"], cfg["n_layer"], cfg["n_head"], cfg["n_embd"])
    n_params = sum(p.numel() for p in model.parameters())
    model, dev = to_device(model, cfg["device"])
    if cfg["fsdp"]:
        wrapped = mn.FullyShardedDataParallel(model, pg, unit_cls=Block)
    else:
        wrapped = mn.DistributedDataParallel(model, pg, bucket_cap_mb=cfg["bucket_mb"],
                                             overlap=not cfg["no_overlap"], algorithm=cfg["algorithm"])
    if dev.type == "cuda":
        from mini_nccl_b200.ops.kernels import FusedAdamW

        opt = FusedAdamW(wrapped.parameters(), lr=cfg["lr"], betas=(0.9, 0.95), weight_decay=0.1)
    else:
        opt = torch.optim.AdamW(wrapped.parameters(), lr=cfg["lr"], betas=(0.9, 0.95), weight_decay=0.1)
    if pg.rank == 0:
        mode = "FSDP" if cfg["fsdp"] else "DDP"
        print(f"model: {n_params / 1e6:.2f}M params | {mode} | world_size={pg.world_size} | "
              f"device={dev} | per-rank batch={cfg['batch_size']}", flush=True)
    B, T = cfg["batch_size"], cfg["block_size"]
    t0, tokens, final = time.perf_counter(), 0, 0.0
    for step in range(cfg["steps"]):
        x, y = batch(data, T, B, seed=step * pg.world_size + pg.rank)
        x, y = x.to(dev), y.to(dev)
        wrapped.zero_grad()
        _, loss = wrapped(x, y)
        loss.backward()
        wrapped.sync()
        opt.step()
        tokens += B * T * pg.world_size
        if step % 20 == 0 or step == cfg["steps"] - 1:
            g = loss.detach().float().reshape(1).cpu()
            collectives.all_reduce(pg, g)
            final = g.item() / pg.world_size
            if pg.rank == 0:
                dt = time.perf_counter() - t0
                print(f"step {step:4d} | loss {final:.4f} | {tokens / dt:,.0f} tok/s", flush=True)
                t0, tokens = time.perf_counter(), 0
    if cfg["fsdp"] and pg.rank == 0:
        rows = (("replica a DDP rank would hold", "ddp_equivalent"),
                ("shards resident between steps", "sharded_params_resident"),
                ("parameters kept whole on every rank", "replicated_params"),
                ("largest gathered unit in flight", "peak_transient"),
                ("peak while training", "fsdp_peak"))
        report = wrapped.memory_report()
        print("\nFSDP parameter memory on rank 0 (MiB):", flush=True)
        for label, key in rows:
            print(f"  {label:<38s}{report[key] / 2**20:10.2f}", flush=True)
    state = wrapped.full_state_dict() if cfg["fsdp"] else None
    if pg.rank == 0 and cfg["sample"]:
        if state is not None:
            model.load_state_dict(state)
        prompt = torch.zeros((1, 1), dtype=torch.long, device=dev)
        out = model.generate(prompt, 200)
        print("\n--- sample ---\n" + "".join(vocab[i] for i in out[0].tolist()) + "\n--------------")
    return final


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--world-size", type=int, default=2)
    ap.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--batch-size", type=int, default=16, help="per-rank batch")
    ap.add_argument("--block-size", type=int, default=128)
    ap.add_argument("--n-layer", type=int, default=4)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=128)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--bucket-mb", type=float, default=0.5)
    ap.add_argument("--no-overlap", action="store_true")
    ap.add_argument("--fsdp", action="store_true", help="shard the transformer blocks instead of replicating")
    ap.add_argument("--algorithm", default="auto", choices=["auto", "ring", "tree", "halving", "naive",
                                                              "one_shot", "two_shot"])
    ap.add_argument("--data", help="text file to train on (default: synthetic corpus)")
    ap.add_argument("--sample", action="store_true")
    ap.add_argument("--trace-dir", help="record every collective; then python -m mini_nccl_b200.diagnose DIR")
    args = ap.parse_args()
    data, vocab = encode(load_corpus(args.data))
    print(f"corpus: {len(data):,} chars, vocab {len(vocab)}", flush=True)
    cfg = vars(args).copy()
    world, trace_dir = cfg.pop("world_size"), cfg.pop("trace_dir")
    losses = mn.run(worker, world, data, vocab, cfg, timeout=3600.0, trace_dir=trace_dir,
                    devices="cuda" if args.device == "cuda" else None)
    print(f"final loss: {losses[0]:.4f}")
    if trace_dir:
        print(f"\ntrace written to {trace_dir}\n  python -m mini_nccl_b200.diagnose {trace_dir} --trace {trace_dir}/merged.json")


if __name__ == "__main__":
    main()
