"""Generate the golden iPC vectors by running the REFERENCE's own pure-PyTorch code.

Run in a container that has the reference checkout (default
``/root/reference``; override with ``LICH_REF``):

    python tests/golden/make_golden.py

It imports ``ipc_tilelang.reference.ipc_step`` / ``ReferenceState`` /
``one_hot`` and ``ipc_tilelang.activations.get_activation`` from the
reference (``src/ipc_tilelang/reference.py:42-59``,
``src/ipc_tilelang/activations.py:33-35``), drives them with the
"T inference iterations + 1 weight update" schedule after a forward-init
sweep (``scripts/validate_reference.py:27-30``), and writes the inputs and
outputs to ``tests/golden/*.npz``.  ``init_weights.npz`` holds the reference's
own weight init (``init_weights``, ``src/ipc_tilelang/reference.py:15-22``) for
a few (dims, seed) pairs on the CPU generator.  The reference is NOT needed to
run the tests: they only read the committed ``.npz`` files.
"""
from __future__ import annotations

import json
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LICH_REF", "/root/reference")) / "src"


def _load_reference():
    sys.path.insert(0, str(REF))
    from ipc_tilelang.activations import get_activation  # noqa: E402
    from ipc_tilelang.reference import ReferenceState, ipc_step, one_hot  # noqa: E402
    return get_activation, ReferenceState, ipc_step, one_hot


def _weights(dims, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn((a, b), generator=g) / math.sqrt(b) for a, b in zip(dims[:-1], dims[1:])]


def _batches(dims, B, count, seed, one_hot):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(count):
        x = torch.rand((dims[-1], B), generator=g)
        labels = torch.randint(0, dims[0], (B,), generator=g)
        out.append((x, one_hot(labels, dims[0], dtype=torch.float32)))
    return out


def run_case(name, dims, B, act_name, alpha, gamma, T, steps, batches_n, seed, *, single_step_no_w=False):
    get_activation, ReferenceState, ipc_step, one_hot = _load_reference()
    act = get_activation(act_name)
    w0 = _weights(dims, seed)
    batches = _batches(dims, B, batches_n, seed + 1, one_hot)
    arrays = {}
    for i, wi in enumerate(w0):
        arrays[f"w_in_{i}"] = wi.numpy()
    for j, (xb, yb) in enumerate(batches):
        arrays[f"xb_{j}"] = xb.numpy()
        arrays[f"yb_{j}"] = yb.numpy()
    w = [t.clone() for t in w0]
    L = len(w)
    metrics = None
    st = None
    for s in range(steps):
        x_in, y = batches[s % batches_n]
        # forward-init sweep, as scripts/validate_reference.py:27-30
        x = [torch.zeros((d, B)) for d in dims]
        x[-1].copy_(x_in)
        for l in reversed(range(L)):
            pred = w[l] @ act.forward(x[l + 1])
            if l > 0:
                x[l].copy_(pred)
        x[0].copy_(y)
        st = ReferenceState(x=x, w=w)
        if single_step_no_w:
            st, metrics = ipc_step(st, act=act, alpha=alpha, gamma=gamma, fixed_low=y, fixed_high=x_in,
                                   update_weights=False)
        else:
            for t in range(T):
                st, metrics = ipc_step(st, act=act, alpha=alpha, gamma=gamma, fixed_low=y, fixed_high=x_in,
                                       update_weights=(t == T - 1))
        w = st.w
    for i, wi in enumerate(st.w):
        arrays[f"w_out_{i}"] = wi.numpy()
    for i, xi in enumerate(st.x):
        arrays[f"x_out_{i}"] = xi.numpy()
    meta = {
        "name": name, "dims": list(dims), "B": B, "activation": act_name, "alpha": alpha, "gamma": gamma,
        "T": T, "steps": steps, "batches": batches_n, "seed": seed, "single_step_no_w": single_step_no_w,
        "energy": float(metrics["energy"]), "max_abs_error": float(metrics["max_abs_error"]),
        "generator": "tests/golden/make_golden.py (reference ipc_step, src/ipc_tilelang/reference.py:42-59)",
    }
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(name, {k: v.shape for k, v in arrays.items() if k != "meta"}, meta["energy"])


def run_init(name, cases):
    """The reference's weight init (``init_weights``, ``src/ipc_tilelang/reference.py:15-22``:
    ``kaiming_uniform_(a=sqrt(5))`` in layer order from one generator) on the CPU, for (dims, seed) pairs."""
    sys.path.insert(0, str(REF))
    from ipc_tilelang.reference import init_weights  # noqa: E402
    arrays, meta = {}, []
    for c, (dims, seed) in enumerate(cases):
        for l, w in enumerate(init_weights(dims, dtype=torch.float32, device=torch.device("cpu"), seed=seed)):
            arrays[f"case{c}_w{l}"] = w.numpy()
        meta.append({"dims": list(dims), "seed": seed})
    arrays["meta"] = np.array(json.dumps({"cases": meta, "generator": "reference init_weights"}))
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(name, len(arrays) - 1, "weight tensors")


def main():
    torch.set_num_threads(1)
    run_init("init_weights", [((10, 64, 64, 784), 0), ((10, 64, 64, 64, 64, 64, 64, 784), 3), ((10, 16, 24), 7)])
    # configs[0] of the baseline: dims (10,64,64,784), tanh, alpha 1e-4, gamma 0.5, T=4
    # (batch reduced from 128 to 8 to keep the fixture small; 2 training steps).
    run_case("c1_dims_b8", (10, 64, 64, 784), 8, "tanh", 1e-4, 0.5, 4, 2, 1, seed=11)
    # Larger alpha so the weight update is far above the fp32 noise floor.
    for act in ("relu", "tanh", "sigmoid", "silu", "gelu"):
        run_case(f"small_{act}", (10, 16, 16, 24), 4, act, 0.05, 0.5, 2, 2, 2, seed=23)
    run_case("small_tanh_no_w", (10, 16, 16, 16, 24), 4, "tanh", 0.05, 0.5, 1, 1, 1, seed=37, single_step_no_w=True)


if __name__ == "__main__":
    main()
