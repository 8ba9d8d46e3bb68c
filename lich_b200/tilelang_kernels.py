"""Fused iPC operator builders -- the drop-in for ``ipc_tilelang.tilelang_kernels``.

Same names, arguments and call convention as the reference
(``src/ipc_tilelang/tilelang_kernels.py:8-17,114-353``): each ``build_*``
returns a cached callable specialised for ``(M, K, B, activation, dtype,
cfg, ...)`` that mutates its tensor arguments in place on the current CUDA
stream.  The callables run hand-written sm_100a kernels through the C ABI in
``include/ipc_b200.h``; nothing is JIT-compiled at build time, so a builder
returns immediately.  On tensor-core shapes an operator with f on its B operand
(prediction error, forward, recompute-mode weight update) first stores
``cast(f(B))`` once into a workspace it allocates on its first call on a
device, then runs the tcgen05 GEMM on it (``ipc_fused_gemm_ws``).

Errors follow the reference: an unknown activation or dtype raises
``ValueError`` at build time; calling a kernel with tensors of the wrong
shape, dtype, device or layout raises ``ValueError`` before anything is
launched; a missing native library raises ``RuntimeError`` at import.
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

import torch

from . import _native as N

N.load()  # fail loudly at import if the native library is missing


@dataclass(frozen=True)
class KernelConfig:
    """Tile knobs of the reference (``tilelang_kernels.py:8-17``) plus ``backend``.

    The sm_100a kernels choose their own tiles (128-row tcgen05 tiles, 64x64
    mma.sync tiles); the reference's fields are kept so configs, tuning
    tables and positional constructions such as
    ``KernelConfig(64, 128, 16, 128, 2, True, 8, False)`` stay valid.
    ``backend`` selects the algorithm: ``"auto"``, ``"simt"`` (generic
    CUDA-core / mma.sync), ``"tcgen05"`` or ``"outer"`` (weight update only);
    the ``tc_*`` fields override the tcgen05 kernel's launch heuristics (tuning
    tables measured on B200 set them, ``lich_b200.tuning``).
    """

    block_m: int = 128
    block_n: int = 128
    block_k: int = 32
    threads: int = 128
    num_stages: int = 2
    swizzle: bool = True
    swizzle_panel: int = 8
    shared_swizzle: bool = False
    backend: str = "auto"
    # launch knobs of the tcgen05 kernel (ipc_gemm_tune_t; 0 = the library's heuristic): output tile
    # width (128 / 256), split-K ranges of a weight update (1 = none), M-tiles per raster band, CTAs
    tc_bn: int = 0
    tc_splits: int = 0
    tc_raster: int = 0
    tc_max_ctas: int = 0
    tc_pair: int = 0  # CTA pairs (cta_group::2, 256 x 256 tiles): 0 launcher's choice, 1 single CTAs, 2 pairs

    def tune(self):
        """The ``ipc_gemm_tune_t`` of this config, or None when every knob is the heuristic's."""
        if not (self.tc_bn or self.tc_splits or self.tc_raster or self.tc_max_ctas or self.tc_pair):
            return None
        t = N.IpcGemmTune()
        t.bn, t.splits, t.raster, t.max_ctas = int(self.tc_bn), int(self.tc_splits), int(self.tc_raster), \
            int(self.tc_max_ctas)
        t.pair = int(self.tc_pair)
        return t


def _algo(cfg: KernelConfig) -> int:
    try:
        return N.ALGO_CODES[str(getattr(cfg, "backend", "auto")).lower()]
    except KeyError as exc:
        raise ValueError(f"Unknown backend {cfg.backend!r}") from exc


class _FusedOp:
    """Shape-specialised callable over the C ABI; validates its tensors, then launches."""

    kind = "op"

    def __init__(self, shapes, activation: str, dtype: str, cfg: KernelConfig, groups: int = 1):
        self.activation = str(activation).lower()
        self.act = N.act_code(self.activation)
        self.torch_dtype = N.torch_dtype(dtype)
        self.dt = N.dtype_code(self.torch_dtype)
        self.cfg = cfg
        self.algo = _algo(cfg)
        self.groups = int(groups)
        self.shapes = [((self.groups,) + tuple(s)) if self.groups > 1 else tuple(s) for s in shapes]
        self._ws: dict = {}

    def _workspace(self, dev: torch.device, mode: int, flags: int):
        """This operator's workspace for the current stream of ``dev`` (allocated on its first call there),
        or None when the call needs none.  With f on the B operand of a tensor-core shape it holds the
        stored activation ``cast(f(B))`` the GEMM reads (plus split-K partials for a weight update).  One
        workspace per stream: calls of one (cached) operator on two streams may overlap."""
        key = (dev, N.stream_handle(dev), mode, flags)
        if key not in self._ws:
            with torch.cuda.device(dev):
                n = N.workspace_bytes(mode, M=self.M, K=self.K, B=self.B, groups=self.groups, flags=flags,
                                      dtype=self.torch_dtype, algo=str(getattr(self.cfg, "backend", "auto")).lower())
            self._ws[key] = torch.empty((n + 15) // 16 * 4, device=dev, dtype=torch.float32) if n > 0 else None
        return self._ws[key]

    def _check(self, tensors):
        if len(tensors) != len(self.shapes):
            raise ValueError(f"{self.kind}: expected {len(self.shapes)} tensors, got {len(tensors)}")
        dev = None
        for i, (t, shape) in enumerate(zip(tensors, self.shapes)):
            if not isinstance(t, torch.Tensor):
                raise ValueError(f"{self.kind}: argument {i} is not a tensor")
            if not t.is_cuda:
                raise ValueError(f"{self.kind}: argument {i} is not a CUDA tensor")
            if tuple(t.shape) != shape:
                raise ValueError(f"{self.kind}: argument {i} has shape {tuple(t.shape)}, kernel was built for {shape}")
            if t.dtype != self.torch_dtype:
                raise ValueError(f"{self.kind}: argument {i} is {t.dtype}, kernel was built for {self.torch_dtype}")
            if not t.is_contiguous():
                raise ValueError(f"{self.kind}: argument {i} is not contiguous")
            if dev is None:
                dev = t.device
            elif t.device != dev:
                raise ValueError(f"{self.kind}: tensors on different devices")
        return dev

    def _algo_name(self) -> str:
        return str(getattr(self.cfg, "backend", "auto")).lower()

    def get_kernel_source(self) -> str:
        return (f"lich_b200 {self.kind} M/K/B shapes={self.shapes} act={self.activation} dtype={self.torch_dtype} "
                f"backend={getattr(self.cfg, 'backend', 'auto')} (prebuilt sm_100a kernel, include/ipc_b200.h)")


class PredictionErrorKernel(_FusedOp):
    kind = "prediction_error"

    def __init__(self, M, K, B, activation, dtype, cfg, groups=1, saved_activation=False):
        super().__init__([(K, B), (M, K), (M, B), (M, B)], activation, dtype, cfg, groups)
        self.M, self.K, self.B = int(M), int(K), int(B)
        self.saved = bool(saved_activation)

    def __call__(self, x_upper, w, x_lower, e):
        dev = self._check((x_upper, w, x_lower, e))
        s = N.stream_handle(dev)
        lib = N.load()
        flags = 0 if self.saved else N.FLAG_ACTIVATE_B
        ws = self._workspace(dev, N.MODE_PRED, flags)
        if ws is not None or self.cfg.tune() is not None:  # tensor cores: f(X_upper) stored once, then tcgen05
            N.fused_gemm(N.MODE_PRED, w, x_upper, e, x_lower, M=self.M, K=self.K, B=self.B, groups=self.groups,
                         flags=flags, act=self.activation, dtype=self.torch_dtype, algo=self._algo_name(),
                         device=dev, workspace=ws, tune=self.cfg.tune())
            return
        if self.saved:
            rc = lib.ipc_pred_err_saved(N.ptr(x_upper), N.ptr(w), N.ptr(x_lower), N.ptr(e), self.M, self.K, self.B,
                                        self.groups, self.dt, self.algo, s)
        else:
            rc = lib.ipc_pred_err(N.ptr(x_upper), N.ptr(w), N.ptr(x_lower), N.ptr(e), self.M, self.K, self.B,
                                  self.groups, self.act, self.dt, self.algo, s)
        N.check(rc)


class InferenceUpdateKernel(_FusedOp):
    kind = "inference_update"

    def __init__(self, M, K, B, activation, dtype, cfg, gamma, save_activation=False, groups=1):
        shapes = [(M, B), (M, B), (K, M), (K, B)] + ([(M, B)] if save_activation else [])
        super().__init__(shapes, activation, dtype, cfg, groups)
        self.M, self.K, self.B = int(M), int(K), int(B)
        self.gamma = float(gamma)
        self.save_activation = bool(save_activation)

    def __call__(self, x, e, w_lower, e_lower, a_out=None):
        tensors = (x, e, w_lower, e_lower) + ((a_out,) if self.save_activation else ())
        if not self.save_activation and a_out is not None:
            raise ValueError("inference_update: kernel built without save_activation takes 4 tensors")
        dev = self._check(tensors)
        tune = self.cfg.tune()
        if tune is not None:
            N.fused_gemm(N.MODE_INFER, w_lower, e_lower, x, e, a_out, M=self.M, K=self.K, B=self.B, groups=self.groups,
                         scale=self.gamma, act=self.activation, dtype=self.torch_dtype, algo=self._algo_name(),
                         device=dev, tune=tune)
            return
        N.check(N.load().ipc_infer_update(N.ptr(x), N.ptr(e), N.ptr(w_lower), N.ptr(e_lower), N.ptr(a_out),
                                          self.M, self.K, self.B, self.groups, self.gamma, self.act, self.dt,
                                          self.algo, N.stream_handle(dev)))


class WeightUpdateKernel(_FusedOp):
    kind = "weight_update"

    def __init__(self, M, K, B, activation, dtype, cfg, alpha, recompute_activation=True, groups=1):
        super().__init__([(M, K), (M, B), (K, B)], activation, dtype, cfg, groups)
        self.M, self.K, self.B = int(M), int(K), int(B)
        self.alpha = float(alpha)
        self.recompute = bool(recompute_activation)

    def __call__(self, w, e, x_or_a_upper):
        dev = self._check((w, e, x_or_a_upper))
        flags = N.FLAG_ACTIVATE_B if self.recompute else 0
        ws = self._workspace(dev, N.MODE_WEIGHT, flags)
        if ws is not None or self.cfg.tune() is not None:  # tensor cores: stored activation / split-K partials
            N.fused_gemm(N.MODE_WEIGHT, e, x_or_a_upper, w, M=self.M, K=self.K, B=self.B, groups=self.groups,
                         scale=self.alpha, flags=flags, act=self.activation, dtype=self.torch_dtype,
                         algo=self._algo_name(), device=dev, workspace=ws, tune=self.cfg.tune())
            return
        N.check(N.load().ipc_weight_update(N.ptr(w), N.ptr(e), N.ptr(x_or_a_upper), self.M, self.K, self.B,
                                           self.groups, self.alpha, int(self.recompute), self.act, self.dt,
                                           self.algo, N.stream_handle(dev)))


class ForwardKernel(_FusedOp):
    """``out = cast(W @ f(x_upper))``: the forward sweep of ``initialize_batch`` / ``predict``."""

    kind = "forward"

    def __init__(self, M, K, B, activation, dtype, cfg, groups=1):
        super().__init__([(K, B), (M, K), (M, B)], activation, dtype, cfg, groups)
        self.M, self.K, self.B = int(M), int(K), int(B)

    def __call__(self, x_upper, w, out):
        dev = self._check((x_upper, w, out))
        ws = self._workspace(dev, N.MODE_FORWARD, N.FLAG_ACTIVATE_B)
        if ws is not None or self.cfg.tune() is not None:
            N.fused_gemm(N.MODE_FORWARD, w, x_upper, out, M=self.M, K=self.K, B=self.B, groups=self.groups,
                         flags=N.FLAG_ACTIVATE_B, act=self.activation, dtype=self.torch_dtype,
                         algo=self._algo_name(), device=dev, workspace=ws, tune=self.cfg.tune())
            return
        N.check(N.load().ipc_forward(N.ptr(x_upper), N.ptr(w), N.ptr(out), self.M, self.K, self.B, self.groups,
                                     self.act, self.dt, self.algo, N.stream_handle(dev)))


def _validate(M, K, B, activation, dtype):
    if min(int(M), int(K), int(B)) < 0:
        raise ValueError(f"negative shape M={M} K={K} B={B}")
    N.act_code(activation)
    N.dtype_code(N.torch_dtype(dtype))


@lru_cache(maxsize=256)
def build_prediction_error(M: int, K: int, B: int, activation: str, dtype: str, cfg: KernelConfig):
    """``E = X_lower - W[M,K] @ f(X_upper[K,B])`` (reference ``tilelang_kernels.py:114-177``)."""
    _validate(M, K, B, activation, dtype)
    return PredictionErrorKernel(M, K, B, activation, dtype, cfg)


@lru_cache(maxsize=256)
def build_inference_update(M: int, K: int, B: int, activation: str, dtype: str, cfg: KernelConfig, gamma: float,
                           save_activation: bool = False):
    """``X += gamma*(-E + f'(X) * W_lower.T @ E_lower)``, optionally ``A_out = f(X)``
    (reference ``tilelang_kernels.py:180-265``)."""
    _validate(M, K, B, activation, dtype)
    return InferenceUpdateKernel(M, K, B, activation, dtype, cfg, gamma, save_activation)


@lru_cache(maxsize=256)
def build_weight_update(M: int, K: int, B: int, activation: str, dtype: str, cfg: KernelConfig, alpha: float,
                        recompute_activation: bool = True):
    """``W += alpha * E @ A.T`` with ``A = f(X_upper)`` or a saved activation
    (reference ``tilelang_kernels.py:268-349``)."""
    _validate(M, K, B, activation, dtype)
    return WeightUpdateKernel(M, K, B, activation, dtype, cfg, alpha, recompute_activation)


@lru_cache(maxsize=256)
def build_forward(M: int, K: int, B: int, activation: str, dtype: str, cfg: KernelConfig = KernelConfig()):
    """``out = W @ f(x)`` (no reference builder: the reference does this step in eager torch)."""
    _validate(M, K, B, activation, dtype)
    return ForwardKernel(M, K, B, activation, dtype, cfg)


def kernel_call(kernel, *tensors: torch.Tensor) -> None:
    """Reference ``tilelang_kernels.py:352-353``."""
    kernel(*tensors)
