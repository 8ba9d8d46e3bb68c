"""Seeded synthetic inputs for the iPC configurations.

MNIST / FashionMNIST (the reference downloads them at run time,
``scripts/train_mnist.py:47``, ``scripts/train_paper_efficiency.py:43``) are
not available offline, so every workload here uses seeded synthetic data of
the same shapes and value ranges:

* inputs ``x_L ~ U[0, 1]`` (784-dim images in [0, 1]; 4096-dim for the wide
  configuration), feature-major ``[d_L, B]``;
* labels uniform over the classes, one-hot ``[C, B]`` targets;
* weights ``W[l] ~ N(0, 1/fan_in)``, ``fan_in = d_{l+1}``, drawn in layer order;
* the per-kernel microbenchmark uses ``x ~ N(0, 1)`` and ``W ~ N(0, 1/K)``.

All draws come from a CPU ``torch.Generator`` (weight seed ``s``, data seed
``s + 1``), so the CPU oracle and the GPU path see the same numbers.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch


def fan_in_normal(dims: Sequence[int], *, seed: int, dtype: torch.dtype = torch.float32) -> list[torch.Tensor]:
    """``W[l] ~ N(0, 1/d_{l+1})`` of shape ``[d_l, d_{l+1}]`` for ``l = 0..L-1`` (CPU)."""
    g = torch.Generator().manual_seed(int(seed))
    out = []
    for n_l, n_u in zip(dims[:-1], dims[1:]):
        w = torch.randn((n_l, n_u), generator=g, dtype=torch.float32) / math.sqrt(n_u)
        out.append(w.to(dtype))
    return out


def one_hot_cb(labels: torch.Tensor, num_classes: int, dtype: torch.dtype) -> torch.Tensor:
    """``[C, B]`` one-hot of integer labels (same layout as the reference ``one_hot``)."""
    y = torch.zeros((num_classes, labels.numel()), dtype=dtype, device=labels.device)
    y.scatter_(0, labels.view(1, -1).long(), 1.0)
    return y


def batch_pool(d_in: int, classes: int, batch: int, *, count: int, seed: int,
               dtype: torch.dtype = torch.float32) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """``count`` batches ``(x [d_in, B] ~ U[0,1], y one-hot [classes, B])`` on the CPU."""
    g = torch.Generator().manual_seed(int(seed))
    out = []
    for _ in range(count):
        x = torch.rand((d_in, batch), generator=g, dtype=torch.float32)
        labels = torch.randint(0, classes, (batch,), generator=g)
        out.append((x.to(dtype), one_hot_cb(labels, classes, dtype)))
    return out


def stacked_pool(d_in: int, classes: int, batch: int, *, count: int, nets: int, seed: int,
                 dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """Pool for ``nets`` independent networks: ``x [count, nets, d_in, B]``, ``y [count, nets, C, B]``."""
    g = torch.Generator().manual_seed(int(seed))
    x = torch.rand((count, nets, d_in, batch), generator=g, dtype=torch.float32).to(dtype)
    labels = torch.randint(0, classes, (count, nets, batch), generator=g)
    y = torch.zeros((count, nets, classes, batch), dtype=dtype)
    y.scatter_(2, labels.unsqueeze(2), 1.0)
    return x, y


def microbench_operands(M: int, K: int, B: int, *, seed: int, dtype: torch.dtype):
    """Operands of one isolated P / I / W launch: ``x ~ N(0,1)``, ``W ~ N(0, 1/K)``.

    Returns a dict with ``x_up [K,B]``, ``w [M,K]``, ``x_lo [M,B]``,
    ``w_low [K,M]`` and ``e_low [K,B]`` (CPU tensors in ``dtype``)."""
    g = torch.Generator().manual_seed(int(seed))
    s = 1.0 / math.sqrt(K)
    return {
        "x_up": torch.randn((K, B), generator=g).to(dtype),
        "w": (torch.randn((M, K), generator=g) * s).to(dtype),
        "x_lo": torch.randn((M, B), generator=g).to(dtype),
        "w_low": (torch.randn((K, M), generator=g) * (1.0 / math.sqrt(M))).to(dtype),
        "e_low": torch.randn((K, B), generator=g).to(dtype),
    }


def paper_dims(depth: int, hidden: int = 64, d_in: int = 784, classes: int = 10) -> tuple[int, ...]:
    """``(classes,) + (hidden,)*depth + (d_in,)``: depth counts hidden layers, ``L = depth + 1``
    (reference ``scripts/train_paper_efficiency.py:54``)."""
    return (classes,) + (hidden,) * depth + (d_in,)
