"""Table printing and input generation shared by the benchmarks."""
from __future__ import annotations

import json
import os

import torch

IGNORE_INDEX = -100


def fmt_float(value: float) -> str:
    return "0" if value == 0.0 else f"{value:.6e}"


def print_table(headers: list[str], rows: list[list[str]], *, title: str = "") -> None:
    widths = [max(len(h), *(len(r[i]) for r in rows)) if rows else len(h) for i, h in enumerate(headers)]
    if title:
        print(f"\n {title}")
    print(" " + " | ".join(h.ljust(w) for h, w in zip(headers, widths)))
    print(" " + "-|-".join("-" * w for w in widths))
    for r in rows:
        print(" " + " | ".join(c.rjust(w) if i >= 2 else c.ljust(w) for i, (c, w) in enumerate(zip(r, widths))))


def seeded_randn(shape, *, seed: int, device, scale: float = 1.0) -> torch.Tensor:
    """fp32 N(0, scale^2) values from a per-tensor generator (identical on every run and device count)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(device)


def seeded_labels(n: int, vocab: int, *, seed: int, device, ignore_every: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    labels = torch.randint(0, vocab, (n,), generator=g)
    labels[:: max(1, ignore_every)] = IGNORE_INDEX
    return labels.to(device)


def write_json(path: str | None, payload: dict) -> None:
    if not path:
        return
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        json.dump(payload, f, indent=1)
