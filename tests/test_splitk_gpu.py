"""GPU parity of the split-K weight update (``ipc_fused_gemm_ws``).

A weight update W += alpha E A^T reduces over the batch.  When the output has
few 128-row tiles and the batch is long, the tcgen05 kernel splits the batch
over the SMs, writes fp32 partial tiles into the caller's workspace and a
second pass sums them in split order.  Checked here: WEIGHT and WDELTA against
the CPU oracle (``<= 1e-2`` 16-bit gate, ``<= 1e-3`` fp32 delta), tails in
M / N / batch, grouped launches, a workspace too small for the full split
count, bit-identical repeat runs, agreement with the unsplit kernel, the
accumulate flag, and the host checks on the workspace pointer.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
DTYPES = [torch.float16, torch.bfloat16]
SHAPES = [(64, 64, 65536), (256, 256, 16384), (136, 200, 8200), (16, 512, 4096), (128, 128, 1024)]


def _N():
    from lich_b200 import _native as N
    return N


def _r(shape, seed, scale, dt):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dt)


def _operands(M, K, B, dt, groups=1, seed=0):
    lead = (groups,) if groups > 1 else ()
    e = _r(lead + (M, B), seed, 0.5, dt)
    a = _r(lead + (K, B), seed + 1, 1.0, dt)
    w = _r(lead + (M, K), seed + 2, 0.05, dt)
    return e, a, w


def _ws(nbytes):
    return torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=DEV)


def _call(mode, e, a, out, M, K, B, dt, groups=1, ws=None, flags=0, alpha=1e-3, algo="tcgen05"):
    N = _N()
    de, da = e.to(DEV), a.to(DEV)
    N.fused_gemm(mode, de, da, out, M=M, K=K, B=B, groups=groups, scale=alpha, flags=flags, dtype=dt, algo=algo,
                 workspace=ws)
    torch.cuda.synchronize()
    assert N.device_status() == 0
    return out.cpu()


def _ref_w(w, e, a, dt, alpha, groups):
    if groups == 1:
        return O.weight_update_op(w, e, a, act="identity", alpha=alpha, sdt=dt, recompute_activation=False)
    return torch.stack([O.weight_update_op(w[g], e[g], a[g], act="identity", alpha=alpha, sdt=dt,
                                           recompute_activation=False) for g in range(groups)])


def _ref_wd(e, a, dt, alpha, groups):
    if groups == 1:
        return O.weight_delta_op(e, a, act="identity", alpha=alpha, sdt=dt, recompute_activation=False)
    return torch.stack([O.weight_delta_op(e[g], a[g], act="identity", alpha=alpha, sdt=dt,
                                          recompute_activation=False) for g in range(groups)])


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_split_weight_update_matches_oracle(shape, dt):
    N = _N()
    M, K, B = shape
    e, a, w = _operands(M, K, B, dt)
    got = _call(N.MODE_WEIGHT, e, a, w.to(DEV), M, K, B, dt, ws=_ws(64 << 20))
    assert O.rel_inf(got, _ref_w(w, e, a, dt, 1e-3, 1)) <= 1e-2


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_split_weight_delta_matches_oracle(shape, dt):
    N = _N()
    M, K, B = shape
    e, a, _ = _operands(M, K, B, dt, seed=3)
    dw = torch.zeros(M, K, dtype=torch.float32, device=DEV)
    got = _call(N.MODE_WDELTA, e, a, dw, M, K, B, dt, ws=_ws(64 << 20))
    assert O.rel_inf(got, _ref_wd(e, a, dt, 1e-3, 1)) <= 1e-3


@pytest.mark.parametrize("dt", DTYPES)
def test_split_grouped(dt):
    N = _N()
    M, K, B, G = 128, 192, 8192, 3
    e, a, w = _operands(M, K, B, dt, groups=G, seed=7)
    got = _call(N.MODE_WEIGHT, e, a, w.to(DEV), M, K, B, dt, groups=G, ws=_ws(64 << 20))
    assert O.rel_inf(got, _ref_w(w, e, a, dt, 1e-3, G)) <= 1e-2
    dw = torch.zeros(G, M, K, dtype=torch.float32, device=DEV)
    got = _call(N.MODE_WDELTA, e, a, dw, M, K, B, dt, groups=G, ws=_ws(64 << 20))
    assert O.rel_inf(got, _ref_wd(e, a, dt, 1e-3, G)) <= 1e-3


def test_small_workspace_caps_the_split_count():
    """Room for two partial tiles only: still exact, still deterministic."""
    N = _N()
    M, K, B, dt = 64, 64, 65536, torch.bfloat16
    e, a, _ = _operands(M, K, B, dt, seed=11)
    ref = _ref_wd(e, a, dt, 1e-3, 1)
    outs = []
    for nbytes in (2 * M * K * 4, 3 * M * K * 4 - 4, M * K * 4):  # 2, 2 and 1 (no split) partials
        dw = torch.zeros(M, K, dtype=torch.float32, device=DEV)
        outs.append(_call(N.MODE_WDELTA, e, a, dw, M, K, B, dt, ws=_ws(nbytes)))
        assert O.rel_inf(outs[-1], ref) <= 1e-3
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("dt", DTYPES)
def test_split_is_deterministic_and_agrees_with_unsplit(dt):
    N = _N()
    M, K, B = 256, 256, 32768
    e, a, _ = _operands(M, K, B, dt, seed=13)
    runs = []
    for _ in range(2):
        dw = torch.zeros(M, K, dtype=torch.float32, device=DEV)
        runs.append(_call(N.MODE_WDELTA, e, a, dw, M, K, B, dt, ws=_ws(64 << 20)))
    assert torch.equal(runs[0], runs[1])
    dw = torch.zeros(M, K, dtype=torch.float32, device=DEV)
    unsplit = _call(N.MODE_WDELTA, e, a, dw, M, K, B, dt, ws=None)
    # two fp32 summation orders over 32768 products each: they differ by rounding only
    assert O.rel_inf(runs[0], unsplit) <= 1e-4


def test_split_accumulate_adds_into_delta():
    N = _N()
    M, K, B, dt = 128, 64, 16384, torch.float16
    e, a, _ = _operands(M, K, B, dt, seed=17)
    base = _r((M, K), 19, 0.01, torch.float32)
    got = _call(N.MODE_WDELTA, e, a, base.to(DEV), M, K, B, dt, ws=_ws(64 << 20), flags=N.FLAG_ACCUMULATE)
    assert O.rel_inf(got, base.double() + _ref_wd(e, a, dt, 1e-3, 1)) <= 1e-3


def test_auto_uses_split_for_long_batches():
    """IPC_ALGO_AUTO with a workspace picks the tensor-core split path for a narrow, long update."""
    N = _N()
    M, K, B, dt = 32, 48, 16384, torch.bfloat16
    e, a, w = _operands(M, K, B, dt, seed=23)
    n0 = N.launch_count()
    got = _call(N.MODE_WEIGHT, e, a, w.to(DEV), M, K, B, dt, ws=_ws(16 << 20), algo="auto")
    assert N.launch_count() - n0 == 2  # GEMM + reduce
    assert O.rel_inf(got, _ref_w(w, e, a, dt, 1e-3, 1)) <= 1e-2


def test_workspace_pointer_checks():
    N = _N()
    M, K, B, dt = 64, 64, 4096, torch.float16
    e = torch.zeros(M, B, dtype=dt, device=DEV)
    a = torch.zeros(K, B, dtype=dt, device=DEV)
    dw = torch.zeros(M, K, dtype=torch.float32, device=DEV)
    ws = _ws(1 << 20)
    with pytest.raises(ValueError):  # not 16-byte aligned
        N.fused_gemm(N.MODE_WDELTA, e, a, dw, M=M, K=K, B=B, scale=1.0, dtype=dt, algo="tcgen05", workspace=ws[1:])
    lib = N.load()
    rc = lib.ipc_fused_gemm_ws(N.MODE_WDELTA, N.ptr(e), N.ptr(a), N.ptr(dw), None, None, M, K, B, 1, 1.0, 0,
                               N.act_code("identity"), N.dtype_code(dt), N.ALGO_CODES["tcgen05"], None, 1024, None)
    assert rc == N.IPC_ERR_ARG
