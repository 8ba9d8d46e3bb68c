"""CPU tests: the C-ABI library loads and exports every declared symbol; host-side logic.

No kernel is launched here (there is no GPU in the build container).
"""
import json
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _declared_functions():
    text = (ROOT / "include" / "ipc_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ipc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from lich_b200 import _native as N
    lib = N.load()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ipc_b200.h but not exported"
    assert set(N.EXPORTED) == set(declared)
    assert lib.ipc_abi_version() == 4


def test_abi_rejects_bad_arguments_without_a_gpu():
    from lich_b200 import _native as N
    lib = N.load()
    # bad activation / dtype / groups are argument errors, reported before any device access
    assert lib.ipc_pred_err(None, None, None, None, 4, 4, 4, 1, 99, 1, 0, None) == N.IPC_ERR_ARG
    assert b"activation" in lib.ipc_last_error()
    assert lib.ipc_pred_err(None, None, None, None, 4, 4, 4, 1, 1, 7, 0, None) == N.IPC_ERR_ARG
    assert lib.ipc_weight_update(None, None, None, 4, 4, 4, 0, 1e-4, 1, 1, 1, 0, None) == N.IPC_ERR_ARG
    assert lib.ipc_net_train(None, None, None) == N.IPC_ERR_ARG


def test_kernel_config_positional_compat():
    from lich_b200.tilelang_kernels import KernelConfig
    cfg = KernelConfig(64, 128, 16, 128, 2, True, 8, False)  # scripts/smoke.py:20 of the reference
    assert cfg.block_m == 64 and cfg.backend == "auto"


def test_builders_validate_like_the_reference():
    from lich_b200 import tilelang_kernels as K
    from lich_b200 import layer_batching as LB
    cfg = K.KernelConfig()
    with pytest.raises(ValueError):
        K.build_prediction_error(4, 4, 4, "swish", "float16", cfg)
    with pytest.raises(ValueError):
        K.build_weight_update(4, 4, 4, "tanh", "int8", cfg, 1e-4)
    with pytest.raises(ValueError):
        LB.build_prediction_error_batched(64, 64, 128, 1, "relu", "float16", cfg)
    with pytest.raises(ValueError):
        LB.build_inference_update_batched(64, 32, 128, 2, "relu", "float16", cfg, 0.5)
    k = K.build_prediction_error(4, 4, 4, "tanh", "float16", cfg)
    assert K.build_prediction_error(4, 4, 4, "tanh", "float16", cfg) is k  # lru-cached like the reference
    x = torch.zeros(4, 4, dtype=torch.float16)
    with pytest.raises(ValueError):
        k(x, x, x, x)  # CPU tensors are rejected before any launch
    assert "prediction_error" in k.get_kernel_source()


# find_internal_square_groups expectations, recorded from the reference's own function
# (src/ipc_tilelang/layer_batching.py:46-86) on these inputs.
GROUPS_EXPECTED = [
    ((10, 64, 64, 64, 784), 2, [(1, 2, 64)]),
    ((10, 64, 64, 64, 64, 64, 64, 784), 2, [(1, 2, 64), (4, 5, 64)]),
    ((10, 64, 64, 64, 64, 64, 64, 784), 5, [(1, 5, 64)]),
    ((10, 64, 64, 64, 64, 784), 3, [(1, 3, 64)]),
    ((784, 64, 64, 10), 2, []),
    ((10, 64, 64, 784), 2, []),
    ((10, 64, 64, 64, 64, 784), 1, []),
]


@pytest.mark.parametrize("dims,cap,expected", GROUPS_EXPECTED)
def test_find_internal_square_groups(dims, cap, expected):
    from lich_b200.layer_batching import find_internal_square_groups
    got = [(g.start, g.end, g.width) for g in find_internal_square_groups(dims, max_group_count=cap)]
    assert got == expected


def test_tuning_table_roundtrip(tmp_path):
    from lich_b200.tilelang_kernels import KernelConfig
    from lich_b200.tuning import TuningEntry, TuningKey, TuningTable
    t = TuningTable.from_entries([TuningEntry(TuningKey("prediction", 64, 64, 128, "tanh", "float16"),
                                              KernelConfig(backend="simt"), 0.001, False)])
    p = tmp_path / "t.json"
    t.to_json(p, device="NVIDIA B200", capability=(10, 0))
    payload = json.loads(p.read_text())
    assert payload["schema_version"] == 1 and payload["search_space"] == "sm100a-v1"
    t2 = TuningTable.from_json(p)
    assert t2.lookup(kind="prediction", M=64, K=64, B=128, activation="tanh", dtype="float16").backend == "simt"
    assert t2.lookup(kind="weight", M=64, K=64, B=128, activation="tanh", dtype="float16") is None


def test_small_b_policy_reads_reference_schema(tmp_path):
    from lich_b200.weight_update_specialization import SmallBWeightPolicy
    p = tmp_path / "policy.json"
    p.write_text(json.dumps({"version": 4, "entries": [
        {"M": 64, "K": 784, "B": 4, "count": 1, "activation": "relu", "dtype": "float16", "backend": "outer"},
        {"M": 64, "K": 64, "B": 4, "backend": "bogus"}, "junk"]}))
    pol = SmallBWeightPolicy(p)
    assert pol.backend(M=64, K=784, B=4, activation="relu", dtype=torch.float16) == "outer"
    assert pol.backend(M=64, K=64, B=4, activation="relu", dtype=torch.float16) == "gemm"


def test_ipc_tilelang_alias():
    import sys
    import lich_b200
    lich_b200.install_ipc_tilelang_alias()
    import ipc_tilelang.trainer as t  # noqa: F401
    assert sys.modules["ipc_tilelang.trainer"].__name__ == "lich_b200.trainer"


def test_synthetic_generators_are_seeded():
    from lich_b200 import synthetic as S
    a = S.fan_in_normal((10, 64, 784), seed=3)
    b = S.fan_in_normal((10, 64, 784), seed=3)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    assert abs(a[1].std().item() - (1 / 784) ** 0.5) < 0.1 * (1 / 784) ** 0.5
    pool = S.batch_pool(784, 10, 16, count=2, seed=4)
    x, y = pool[0]
    assert x.min() >= 0 and x.max() <= 1 and torch.equal(y.sum(0), torch.ones(16))
