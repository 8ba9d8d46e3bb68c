"""Reader for the committed golden vectors in ``tests/golden/*.npz``."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def cases():
    """The training-step fixtures (the weight-init fixture ``init_weights.npz`` has its own reader)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith("init_"))


def load_init():
    """[(dims, seed, [W_0 .. W_{L-1}])] from ``init_weights.npz`` (the reference's ``init_weights``)."""
    z = np.load(GOLDEN / "init_weights.npz")
    meta = json.loads(str(z["meta"]))
    out = []
    for c, m in enumerate(meta["cases"]):
        L = len(m["dims"]) - 1
        out.append((tuple(m["dims"]), m["seed"], [torch.from_numpy(z[f"case{c}_w{l}"].copy()) for l in range(L)]))
    return out


def load(name: str):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    L = len(meta["dims"]) - 1
    t = lambda k: torch.from_numpy(z[k].copy())  # noqa: E731
    w_in = [t(f"w_in_{i}") for i in range(L)]
    w_out = [t(f"w_out_{i}") for i in range(L)]
    x_out = [t(f"x_out_{i}") for i in range(L + 1)]
    batches = [(t(f"xb_{j}"), t(f"yb_{j}")) for j in range(meta["batches"])]
    return meta, w_in, batches, w_out, x_out
