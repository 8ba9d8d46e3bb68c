"""Activation registry (names and codes of the activations the kernels fuse).

Mirrors ``src/ipc_tilelang/activations.py:6-35`` of the reference: the same
five names plus ``identity``.  ``forward`` runs the library's own
element-wise kernel on CUDA tensors (the trainer uses it for the saved input
activation, ``trainer.py:510-511``); there is no CPU path.  ``derivative``
is a convenience on CUDA tensors for inspection only -- every kernel fuses
f' itself.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as N


@dataclass(frozen=True)
class ActivationSpec:
    name: str

    @property
    def code(self) -> int:
        return N.act_code(self.name)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("lich_b200 activations run on CUDA tensors only")
        x = x.contiguous()
        out = torch.empty_like(x)
        N.check(N.load().ipc_activate(N.ptr(out), N.ptr(x), x.numel(), self.code, N.dtype_code(x.dtype),
                                      N.stream_handle(x.device)))
        return out

    def derivative(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("lich_b200 activations run on CUDA tensors only")
        xf = x.float()
        n = self.name
        if n == "relu":
            d = (xf > 0).float()
        elif n == "tanh":
            y = torch.tanh(xf)
            d = 1 - y * y
        elif n == "sigmoid":
            y = torch.sigmoid(xf)
            d = y * (1 - y)
        elif n == "silu":
            s = torch.sigmoid(xf)
            d = s * (1 + xf * (1 - s))
        elif n == "gelu":
            c, k = 0.044715, 0.7978845608028654
            u = k * (xf + c * xf ** 3)
            t = torch.tanh(u)
            d = 0.5 * (1 + t) + 0.5 * xf * (1 - t * t) * k * (1 + 3 * c * xf * xf)
        else:
            d = torch.ones_like(xf)
        return d.to(x.dtype)


ACTIVATIONS = {n: ActivationSpec(n) for n in ("relu", "tanh", "sigmoid", "silu", "gelu", "identity")}


def get_activation(name: str) -> ActivationSpec:
    """Reference ``activations.py:33-35``: ValueError for an unknown name."""
    try:
        return ACTIVATIONS[name.lower()]
    except KeyError as exc:
        raise ValueError(f"Unknown activation {name!r}") from exc
