"""Small-batch weight update -- the drop-in for ``ipc_tilelang.weight_update_specialization``.

The reference forms a ``[B, M, K]`` temporary with ``torch.bmm`` and reduces
it (``src/ipc_tilelang/weight_update_specialization.py:90-104``).  Here the
update is one sm_100a kernel (``ipc_weight_update`` with
``IPC_ALGO_OUTER``) that reads W once and writes it once, with E and f(X)
staged in shared memory; it supports every activation, not only relu /
identity.

Sign: the reference's eager path subtracts (``w.add_(-alpha*grad)``,
``weight_update_specialization.py:102``) while its GEMM kernel and its
oracle add (``tilelang_kernels.py:320``, ``reference.py:57``).  This module
follows the oracle: ``W += alpha * E @ f(X)^T``, so switching backends never
changes the result.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from .tilelang_kernels import KernelConfig, WeightUpdateKernel


def _dtype_name(dtype: Any) -> str:
    return str(dtype).split(".")[-1]


@dataclass(frozen=True)
class WeightPolicyKey:
    M: int
    K: int
    B: int
    activation: str = "relu"
    dtype: str = "float16"


class SmallBWeightPolicy:
    """Read-only exact-shape backend table (``gemm`` / ``outer``), same JSON schema as the reference
    (``weight_update_specialization.py:24-60``)."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        with self.path.open("r", encoding="utf-8") as f:
            data = json.load(f)
        if not isinstance(data, dict):
            raise ValueError(f"Invalid weight-update policy: {self.path}")
        self.data = data
        self.entries: dict[tuple[int, int, int, int, str, str], str] = {}
        for row in data.get("entries", []):
            if not isinstance(row, dict):
                continue
            try:
                key = (int(row["M"]), int(row["K"]), int(row["B"]), int(row.get("count", 1)),
                       str(row.get("activation", "relu")), str(row.get("dtype", "float16")))
            except (KeyError, TypeError, ValueError):
                continue
            backend = str(row.get("backend", "gemm")).lower()
            if backend in {"gemm", "outer"}:
                self.entries[key] = backend

    def backend(self, *, M: int, K: int, B: int, activation: str, dtype: Any, count: int = 1) -> str:
        return self.entries.get((int(M), int(K), int(B), int(count), str(activation), _dtype_name(dtype)), "gemm")


class SmallBWeightUpdater:
    """Factory of small-B outer-product updaters: ``updater(w, e, src)`` with
    ``w [M,K]``, ``e [M,B]``, ``src [K,B]`` (``f`` applied to ``src``)."""

    def __init__(self, *, alpha: float):
        self.alpha = float(alpha)
        self._single_cache: dict[tuple, object] = {}
        self._group_cache: dict[tuple, object] = {}

    @staticmethod
    def _supported_activation(name: str) -> bool:
        return str(name).lower() in {"relu", "tanh", "sigmoid", "silu", "gelu", "identity", "linear"}

    def _make(self, *, M, K, B, activation, dtype, count):
        if not self._supported_activation(activation):
            return None
        cfg = KernelConfig(backend="outer")
        act = "identity" if str(activation).lower() == "linear" else str(activation).lower()
        return WeightUpdateKernel(M, K, B, act, _dtype_name(dtype), cfg, self.alpha, True, groups=count)

    def make_singleton(self, *, M: int, K: int, B: int, activation: str, dtype: Any):
        key = (int(M), int(K), int(B), str(activation), _dtype_name(dtype), "single")
        if key not in self._single_cache:
            self._single_cache[key] = self._make(M=M, K=K, B=B, activation=activation, dtype=dtype, count=1)
        return self._single_cache[key]

    def make_grouped(self, *, count: int, M: int, K: int, B: int, activation: str, dtype: Any):
        """Grouped small-B update over ``[count, M, K]`` stacks (the reference leaves this disabled,
        ``weight_update_specialization.py:106-112``; the kernel here covers it)."""
        key = (int(count), int(M), int(K), int(B), str(activation), _dtype_name(dtype), "group")
        if key not in self._group_cache:
            self._group_cache[key] = self._make(M=M, K=K, B=B, activation=activation, dtype=dtype, count=count)
        return self._group_cache[key]
