"""Shared helpers for the examples: a character corpus and batch sampling.

There is no network access assumed: ``--data PATH`` trains on any local text
file; without it a synthetic corpus (a repeated paragraph with some noise) is
generated, which is enough to watch the loss fall.
"""

from __future__ import annotations

import random
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

_PARAGRAPH = (
    "To be, or not to be, that is the question: Whether 'tis nobler in the mind to suffer "
    "the slings and arrows of outrageous fortune, or to take arms against a sea of troubles "
    "and by opposing end them. To die, to sleep, no more; and by a sleep to say we end the "
    "heart-ache and the thousand natural shocks that flesh is heir to.\n"
)


def load_corpus(path: str | None, n_chars: int = 200_000) -> str:
    if path:
        return Path(path).read_text(encoding="utf-8")
    rng = random.Random(0)
    out, words = [], _PARAGRAPH.split(" ")
    while sum(len(w) + 1 for w in out) < n_chars:
        w = words[rng.randrange(len(words))] if rng.random() < 0.2 else words[len(out) % len(words)]
        out.append(w)
    return " ".join(out)


def encode(text: str) -> tuple[torch.Tensor, str]:
    vocab = "".join(sorted(set(text)))
    stoi = {c: i for i, c in enumerate(vocab)}
    return torch.tensor([stoi[c] for c in text], dtype=torch.long), vocab


def batch(data: torch.Tensor, block: int, size: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    ix = torch.randint(len(data) - block - 1, (size,), generator=g)
    x = torch.stack([data[i : i + block] for i in ix])
    y = torch.stack([data[i + 1 : i + block + 1] for i in ix])
    return x, y


def to_device(model: torch.nn.Module, device: str):
    """Model placement: CUDA runs bf16 on the sm_100a kernels, CPU stays fp32."""
    if device == "cuda":
        dev = torch.device("cuda", torch.cuda.current_device())
        return model.to(dev, torch.bfloat16), dev
    return model, torch.device("cpu")
