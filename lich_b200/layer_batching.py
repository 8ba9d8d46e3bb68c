"""Layer-batched ("grid.z") operators -- the drop-in for ``ipc_tilelang.layer_batching``.

A run of identical square internal layers is stored as one contiguous
``[G(+1), D, B]`` buffer so one launch covers all of them; the kernels take a
leading ``groups`` dimension (reference ``src/ipc_tilelang/layer_batching.py``).
The sm_100a kernels are the same as the singleton ones with ``groups > 1``
(one CTA grid slice per group).
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

from .tilelang_kernels import (
    ForwardKernel,
    InferenceUpdateKernel,
    KernelConfig,
    PredictionErrorKernel,
    WeightUpdateKernel,
    _validate,
)


@dataclass(frozen=True)
class LayerBatchGroup:
    """Edges ``start..end`` (inclusive) of equal width, states ``start..end+1``.

    Endpoints are never included, so the inference update never touches x[0]
    or x[L] (reference ``layer_batching.py:16-43``)."""

    start: int
    end: int
    width: int

    @property
    def count(self) -> int:
        return self.end - self.start + 1

    @property
    def state_count(self) -> int:
        return self.count + 1

    @property
    def edge_indices(self) -> tuple[int, ...]:
        return tuple(range(self.start, self.end + 1))

    @property
    def state_indices(self) -> tuple[int, ...]:
        return tuple(range(self.start, self.end + 2))


def find_internal_square_groups(dims: tuple[int, ...], *, max_group_count: int = 2) -> tuple[LayerBatchGroup, ...]:
    """Non-overlapping groups of consecutive square internal edges.

    Same contract as the reference (``layer_batching.py:46-86``): only edges
    ``1 <= l <= L-2`` with ``dims[l] == dims[l+1]`` qualify; a maximal run of
    such edges is cut into groups of at most ``max_group_count`` edges, a
    group needs at least two edges, and one edge is left out after each group
    so neighbouring groups never share a state buffer.
    """
    L = len(dims) - 1
    if L < 3 or max_group_count < 2:
        return ()
    square = [1 <= l <= L - 2 and int(dims[l]) == int(dims[l + 1]) for l in range(L)]
    groups: list[LayerBatchGroup] = []
    l = 1
    while l <= L - 2:
        if not square[l]:
            l += 1
            continue
        width = int(dims[l])
        run_end = l
        while run_end + 1 <= L - 2 and square[run_end + 1] and int(dims[run_end + 1]) == width:
            run_end += 1
        start = l
        while start <= run_end:
            stop = min(start + max_group_count - 1, run_end)
            if stop > start:
                groups.append(LayerBatchGroup(start=start, end=stop, width=width))
                start = stop + 2
            else:
                start += 1
        l = run_end + 1
    return tuple(groups)


def _check_groups(groups: int, M: int, K: int, what: str) -> None:
    if groups < 2:
        raise ValueError(f"batched {what} kernel requires groups >= 2")
    if M != K:
        raise ValueError("layer batching covers only square internal layers")


@lru_cache(maxsize=128)
def build_prediction_error_batched(M: int, K: int, B: int, groups: int, activation: str, dtype: str,
                                   cfg: KernelConfig):
    """``E[g] = X_lower[g] - W[g] @ f(X_upper[g])`` (reference ``layer_batching.py:89-150``)."""
    _check_groups(groups, M, K, "prediction")
    _validate(M, K, B, activation, dtype)
    return PredictionErrorKernel(M, K, B, activation, dtype, cfg, groups=groups)


@lru_cache(maxsize=128)
def build_inference_update_batched(M: int, K: int, B: int, groups: int, activation: str, dtype: str,
                                   cfg: KernelConfig, gamma: float, save_activation: bool = False):
    """Batched inference update (reference ``layer_batching.py:153-248``)."""
    _check_groups(groups, M, K, "inference")
    _validate(M, K, B, activation, dtype)
    return InferenceUpdateKernel(M, K, B, activation, dtype, cfg, gamma, save_activation, groups=groups)


@lru_cache(maxsize=128)
def build_weight_update_batched(M: int, K: int, B: int, groups: int, activation: str, dtype: str,
                                cfg: KernelConfig, alpha: float, recompute_activation: bool = True):
    """Batched ``W[g] += alpha * E[g] @ A[g].T`` (reference ``layer_batching.py:251-346``)."""
    _check_groups(groups, M, K, "weight")
    _validate(M, K, B, activation, dtype)
    return WeightUpdateKernel(M, K, B, activation, dtype, cfg, alpha, recompute_activation, groups=groups)


@lru_cache(maxsize=128)
def build_forward_batched(M: int, K: int, B: int, groups: int, activation: str, dtype: str, cfg: KernelConfig):
    _check_groups(groups, M, K, "forward")
    _validate(M, K, B, activation, dtype)
    return ForwardKernel(M, K, B, activation, dtype, cfg, groups=groups)
