"""GPU test of lich_b200.profiling.operator_times: per-operator event timing of a running step."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_operator_times_counts_the_step_launches():
    from lich_b200 import _native as N
    from lich_b200 import profiling as P
    from lich_b200.trainer import IPCConfig, TileLangIPC
    dims, B, T = (104, 512, 512, 1024), 512, 3
    m = TileLangIPC(IPCConfig(dims=dims, activation="tanh", dtype=torch.bfloat16), device=DEV)
    x = torch.rand(dims[-1], B, device=DEV).to(torch.bfloat16)
    y = torch.zeros(dims[0], B, device=DEV, dtype=torch.bfloat16)
    y[0] = 1
    orig = N.fused_gemm
    res = P.operator_times(lambda: m.train_step(x, y, T=T), steps=3, warmup=1)
    assert N.fused_gemm is orig  # unwrapped again
    assert res["step_ms"] > 0 and 0 < res["gemm_ms"] <= res["step_ms"] * 1.05
    per_op = {}
    for r in res["rows"]:
        assert r["median_ms"] > 0 and r["tflops"] > 0
        per_op[r["op"]] = per_op.get(r["op"], 0) + r["per_step"] * r["groups"]
    L = len(dims) - 1
    # every layer's P and every hidden state's I at least once per iteration, one W per layer
    assert per_op["P"] % L == 0 and per_op["P"] >= T * L, per_op
    assert per_op["I"] % (L - 1) == 0 and per_op["I"] >= T * (L - 1), per_op
    assert per_op["W"] == L, per_op
