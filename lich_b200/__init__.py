"""lich_b200 -- B200 (sm_100a) implementation of the iPC step of laghzen/Lich.

The operator and trainer modules keep the reference's ``ipc_tilelang`` names:

    from lich_b200.tilelang_kernels import KernelConfig, build_prediction_error, ...
    from lich_b200.trainer import IPCConfig, TileLangIPC, prepare_batch

``install_ipc_tilelang_alias()`` registers this package under the name
``ipc_tilelang`` so code written against the reference imports it unchanged.
The native library (``lich_b200/_lib/libipc_b200.so``, C ABI in
``include/ipc_b200.h``) is built with ``python -m lich_b200.build``.
"""
from __future__ import annotations

import importlib
import sys

__all__ = ["install_ipc_tilelang_alias"]

_ALIASED = ("activations", "tilelang_kernels", "layer_batching", "trainer", "cuda_graph",
            "weight_update_specialization", "tuning")


def install_ipc_tilelang_alias() -> None:
    """Make ``import ipc_tilelang.<module>`` resolve to this package's modules."""
    pkg = sys.modules[__name__]
    sys.modules.setdefault("ipc_tilelang", pkg)
    for name in _ALIASED:
        mod = importlib.import_module(f"{__name__}.{name}")
        sys.modules.setdefault(f"ipc_tilelang.{name}", mod)
