"""ctypes binding of the C ABI in ``include/ipc_b200.h`` (``lich_b200/_lib/libipc_b200.so``).

The library is the product: there is no CPU or eager-torch fallback.  If it is
missing, importing the operators raises immediately with the build command.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_longlong, c_size_t, c_ulonglong, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libipc_b200.so"

IPC_OK = 0
IPC_ERR_ARG = -1
IPC_ERR_UNSUPPORTED = -2
IPC_ERR_CUDA = -3
IPC_ERR_TIMEOUT = -4
IPC_ERR_DEVICE = -5

ACT_CODES = {"relu": 0, "tanh": 1, "sigmoid": 2, "silu": 3, "gelu": 4, "identity": 5, "linear": 5}
DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
DTYPE_NAMES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
               "fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16,
               "half": torch.float16}
ALGO_CODES = {"auto": 0, "simt": 1, "generic": 1, "tcgen05": 2, "outer": 3}

MODE_PRED, MODE_INFER, MODE_WEIGHT, MODE_WDELTA, MODE_FORWARD = 0, 1, 2, 3, 4
FLAG_ACTIVATE_B, FLAG_AOUT_STORED, FLAG_ACCUMULATE, FLAG_MULTIMEM_RED = 1, 2, 4, 8

# Split-K scratch that covers every shape the weight update splits: a split happens only with fewer
# than half the SMs' worth of 128 x 128 output tiles, and splits x tiles stays below 148 + tiles, so the
# fp32 partials never exceed 222 tiles x 64 KiB.
SPLITK_WORKSPACE_BYTES = 16 << 20

NET_MAX_LAYERS = 8
NET_TRACE_STEPS = 64
NET_TRACE_PHASES = 12
NET_SYNC_BYTES = 64

EXPORTED = (
    "ipc_abi_version", "ipc_last_error", "ipc_launch_count", "ipc_pred_err", "ipc_pred_err_saved",
    "ipc_forward", "ipc_infer_update", "ipc_weight_update", "ipc_weight_delta", "ipc_weight_apply",
    "ipc_activate", "ipc_net_train", "ipc_net_plan", "ipc_fused_gemm", "ipc_device_status",
    "ipc_fused_gemm_ws", "ipc_weight_update_noalloc", "ipc_selftest_barrier_timeout", "ipc_set_max_ctas",
    "ipc_fused_gemm_ws_bytes", "ipc_fused_gemm_tuned", "ipc_weight_update_opt", "ipc_count_correct",
)


class IpcNet(Structure):
    _fields_ = [
        ("L", c_int),
        ("dims", c_int * (NET_MAX_LAYERS + 1)),
        ("B", c_int),
        ("nets", c_int),
        ("w", c_void_p * NET_MAX_LAYERS),
        ("x", c_void_p * (NET_MAX_LAYERS + 1)),
        ("e", c_void_p * (NET_MAX_LAYERS + 1)),
        ("a", c_void_p * (NET_MAX_LAYERS + 1)),
    ]


class IpcNetRun(Structure):
    _fields_ = [
        ("pool_x", c_void_p),
        ("pool_y", c_void_p),
        ("pool_batches", c_int),
        ("first_batch", c_int),
        ("steps", c_int),
        ("T", c_int),
        ("forward_init", c_int),
        ("update_weights", c_int),
        ("recompute", c_int),
        ("alpha", c_float),
        ("gamma", c_float),
        ("act", c_int),
        ("dtype", c_int),
        ("cluster", c_int),
        ("energy", c_void_p),
        ("phase_ns", c_void_p),
        ("sync", c_void_p),
    ]


OPT_KINDS = {"sgd": 1, "adamw": 2}


class IpcOptim(Structure):
    _fields_ = [("kind", c_int), ("lr", c_float), ("momentum", c_float), ("weight_decay", c_float),
                ("beta1", c_float), ("beta2", c_float), ("eps", c_float), ("step", c_int),
                ("m", c_void_p), ("v", c_void_p)]


class IpcGemmTune(Structure):
    _fields_ = [("bn", c_int), ("splits", c_int), ("raster", c_int), ("max_ctas", c_int), ("pair", c_int)]


class IpcError(RuntimeError):
    """A C-ABI call returned a negative code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ipc error {code}: {msg}")
        self.code = code


_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("LICH_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(f"native library {path} is missing: build it with `python -m lich_b200.build`")
    lib = ctypes.CDLL(str(path))
    vp, i, f, ll = c_void_p, c_int, c_float, c_longlong
    sig = {
        "ipc_abi_version": (i, []),
        "ipc_last_error": (c_char_p, []),
        "ipc_launch_count": (c_ulonglong, []),
        "ipc_pred_err": (i, [vp, vp, vp, vp, i, i, i, i, i, i, i, vp]),
        "ipc_pred_err_saved": (i, [vp, vp, vp, vp, i, i, i, i, i, i, vp]),
        "ipc_forward": (i, [vp, vp, vp, i, i, i, i, i, i, i, vp]),
        "ipc_infer_update": (i, [vp, vp, vp, vp, vp, i, i, i, i, f, i, i, i, vp]),
        "ipc_weight_update": (i, [vp, vp, vp, i, i, i, i, f, i, i, i, i, vp]),
        "ipc_weight_delta": (i, [vp, vp, vp, i, i, i, i, f, i, i, i, i, i, vp]),
        "ipc_weight_apply": (i, [vp, vp, ll, i, vp]),
        "ipc_activate": (i, [vp, vp, ll, i, i, vp]),
        "ipc_net_train": (i, [POINTER(IpcNet), POINTER(IpcNetRun), vp]),
        "ipc_net_plan": (i, [POINTER(IpcNet), i, POINTER(c_int), POINTER(c_int)]),
        "ipc_fused_gemm": (i, [i, vp, vp, vp, vp, vp, i, i, i, i, f, i, i, i, i, vp]),
        "ipc_device_status": (i, [POINTER(c_int), i]),
        "ipc_fused_gemm_ws": (i, [i, vp, vp, vp, vp, vp, i, i, i, i, f, i, i, i, i, vp, c_size_t, vp]),
        "ipc_weight_update_noalloc": (i, [i, vp, vp, vp, i, i, i, i, f, i, i, i, i, vp]),
        "ipc_selftest_barrier_timeout": (i, [vp, i, vp]),
        "ipc_set_max_ctas": (i, [i]),
        "ipc_fused_gemm_ws_bytes": (i, [i, i, i, i, i, i, i, i, POINTER(c_size_t)]),
        "ipc_fused_gemm_tuned": (i, [i, vp, vp, vp, vp, vp, i, i, i, i, f, i, i, i, i, vp, c_size_t,
                                     POINTER(IpcGemmTune), vp]),
        "ipc_weight_update_opt": (i, [vp, vp, vp, i, i, i, i, POINTER(IpcOptim), i, i, i, i, vp, c_size_t, vp]),
        "ipc_count_correct": (i, [vp, i, i, vp, vp, i, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != IPC_OK:
        msg = load().ipc_last_error().decode(errors="replace")
        if rc == IPC_ERR_ARG:
            raise ValueError(f"ipc error {rc}: {msg}")
        raise IpcError(rc, msg)


def stream_handle(device: torch.device | None = None) -> int:
    """The current torch CUDA stream as a raw cudaStream_t value."""
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: "torch.Tensor | int | None") -> int | None:
    """A tensor's device address; an int is taken as an address already (a multicast pointer)."""
    if t is None or isinstance(t, int):
        return t
    return t.data_ptr()


def act_code(name: str) -> int:
    try:
        return ACT_CODES[str(name).lower()]
    except KeyError as exc:
        raise ValueError(f"Unsupported activation {name!r}") from exc


def dtype_code(dtype) -> int:
    if isinstance(dtype, str):
        if dtype not in DTYPE_NAMES:
            raise ValueError(f"Unsupported dtype {dtype!r}")
        dtype = DTYPE_NAMES[dtype]
    try:
        return DTYPE_CODES[dtype]
    except KeyError as exc:
        raise ValueError(f"Unsupported dtype {dtype!r}") from exc


def torch_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, str):
        if dtype not in DTYPE_NAMES:
            raise ValueError(f"Unsupported dtype {dtype!r}")
        return DTYPE_NAMES[dtype]
    return dtype


def tc_eligible(mode: int, M: int, K: int, B: int, dtype) -> bool:
    """Whether ``ipc_fused_gemm`` (IPC_ALGO_AUTO, stored operand, no workspace) takes the tcgen05 kernel
    for this shape: the rule of ``tc_eligible`` in csrc/ipc_tc.cu (16-bit operands, every extent a
    multiple of 8, at least 64 x 128 x 64 and 128 x 256 x 256 multiply-adds)."""
    if torch_dtype(dtype) not in (torch.float16, torch.bfloat16):
        return False
    if M % 8 or K % 8 or B % 8:
        return False
    Mg, Ng, Kg = (M, K, B) if mode in (MODE_WEIGHT, MODE_WDELTA) else (M, B, K)
    return Mg >= 64 and Ng >= 128 and Kg >= 64 and Mg * Ng * Kg >= 128 * 256 * 256


def net_plan(dims, B: int, nets: int = 1, cluster: int = 0) -> tuple[int, int] | None:
    """(cluster, shared-memory bytes) the persistent kernel would use, or None if it cannot run.

    A pure function of its arguments on a given device kind: remembered per process (the trainer asks
    before every launch)."""
    key = (tuple(int(d) for d in dims), int(B), int(nets), int(cluster))
    hit = _NET_PLANS.get(key, _MISS)
    if hit is not _MISS:
        return hit
    res = _net_plan(key[0], *key[1:])
    _NET_PLANS[key] = res
    return res


_NET_PLANS: dict = {}
_MISS = object()


def _net_plan(dims, B: int, nets: int, cluster: int) -> tuple[int, int] | None:
    desc = IpcNet()
    desc.L = len(dims) - 1
    if not 1 <= desc.L <= NET_MAX_LAYERS:
        return None
    for l, d in enumerate(dims):
        desc.dims[l] = int(d)
    desc.B, desc.nets = int(B), int(nets)
    c, sm = c_int(0), c_int(0)
    rc = load().ipc_net_plan(ctypes.byref(desc), int(cluster), ctypes.byref(c), ctypes.byref(sm))
    return (c.value, sm.value) if rc == IPC_OK else None


def fused_gemm(mode: int, a, b, out, aux=None, aux2=None, *, M: int, K: int, B: int, groups: int = 1,
               scale: float = 0.0, flags: int = 0, act: str = "identity", dtype=torch.float16, algo: str = "auto",
               device=None, workspace=None, tune: IpcGemmTune | None = None) -> None:
    """``ipc_fused_gemm`` on the current stream (operand roles per mode: include/ipc_b200.h); with a
    workspace ``ipc_fused_gemm_ws``, with tuning overrides ``ipc_fused_gemm_tuned``."""
    if tune is not None:
        nbytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(load().ipc_fused_gemm_tuned(int(mode), ptr(a), ptr(b), ptr(out), ptr(aux), ptr(aux2), int(M), int(K),
                                          int(B), int(groups), float(scale), int(flags), act_code(act),
                                          dtype_code(dtype), ALGO_CODES[algo], ptr(workspace), nbytes,
                                          ctypes.byref(tune), stream_handle(device)))
    elif workspace is None:
        check(load().ipc_fused_gemm(int(mode), ptr(a), ptr(b), ptr(out), ptr(aux), ptr(aux2), int(M), int(K), int(B),
                                    int(groups), float(scale), int(flags), act_code(act), dtype_code(dtype),
                                    ALGO_CODES[algo], stream_handle(device)))
    else:  # fp32 scratch for split-K partial tiles (``ipc_fused_gemm_ws``)
        nbytes = workspace.numel() * workspace.element_size()
        check(load().ipc_fused_gemm_ws(int(mode), ptr(a), ptr(b), ptr(out), ptr(aux), ptr(aux2), int(M), int(K),
                                       int(B), int(groups), float(scale), int(flags), act_code(act),
                                       dtype_code(dtype), ALGO_CODES[algo], ptr(workspace), nbytes,
                                       stream_handle(device)))


def workspace_bytes(mode: int, *, M: int, K: int, B: int, groups: int = 1, flags: int = 0, dtype=torch.float16,
                    algo: str = "auto") -> int:
    """Workspace ``fused_gemm(..., workspace=)`` uses for this call (``ipc_fused_gemm_ws_bytes``)."""
    n = c_size_t(0)
    check(load().ipc_fused_gemm_ws_bytes(int(mode), int(M), int(K), int(B), int(groups), int(flags),
                                         dtype_code(dtype), ALGO_CODES[algo], ctypes.byref(n)))
    return int(n.value)


def weight_update_opt(w, e, x_up, *, M: int, K: int, B: int, groups: int = 1, kind: str, lr: float,
                      momentum: float = 0.0, weight_decay: float = 0.0, betas=(0.9, 0.999), eps: float = 1e-8,
                      step: int = 1, m=None, v=None, recompute: bool = False, act: str = "identity",
                      dtype=torch.float16, algo: str = "auto", workspace=None, device=None) -> None:
    """``ipc_weight_update_opt`` on the current stream: an SGD / AdamW step on W from ``E @ f(X)^T``."""
    o = IpcOptim()
    o.kind = OPT_KINDS[kind]
    o.lr, o.momentum, o.weight_decay = float(lr), float(momentum), float(weight_decay)
    o.beta1, o.beta2, o.eps, o.step = float(betas[0]), float(betas[1]), float(eps), int(step)
    o.m, o.v = ptr(m), ptr(v)
    nbytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(load().ipc_weight_update_opt(ptr(w), ptr(e), ptr(x_up), int(M), int(K), int(B), int(groups),
                                       ctypes.byref(o), int(bool(recompute)), act_code(act), dtype_code(dtype),
                                       ALGO_CODES[algo], ptr(workspace), nbytes, stream_handle(device)))


def device_status(clear: bool = True) -> int:
    """First device-side error code recorded by a bounded wait (0 if none); synchronises."""
    v = c_int(0)
    check(load().ipc_device_status(ctypes.byref(v), int(clear)))
    return v.value


def set_max_ctas(max_ctas: int) -> None:
    """Cap the CTAs of persistent tensor-core GEMMs (0 = one per SM); see ``ipc_set_max_ctas``."""
    check(load().ipc_set_max_ctas(int(max_ctas)))


def launch_count() -> int:
    return int(load().ipc_launch_count())
