"""GPU parity of the fused operators against the CPU oracle (oracle/ipc_oracle.py).

Every call goes through the C ABI (via the ``lich_b200.tilelang_kernels``
adapters).  The oracle applies the same storage-dtype rounding points as the
reference kernels and accumulates in float64, so the tolerances below only
absorb fp32 accumulation order and one-ulp rounding flips:

* fp32 storage: ``max|got - ref| / max|ref| <= 1e-5`` (the north-star fp32 gate);
* fp16 / bf16 storage: ``<= 1e-2`` (the north-star 16-bit gate).
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
TOL = {"float32": 1e-5, "float16": 1e-2, "bfloat16": 1e-2}
ACTS = ["relu", "tanh", "sigmoid", "silu", "gelu", "identity"]
DEV = torch.device("cuda", 0)


def _k():
    from lich_b200 import tilelang_kernels as K
    return K


def _inputs(M, K, B, dt, seed, groups=1):
    g = torch.Generator().manual_seed(seed)
    lead = (groups,) if groups > 1 else ()
    r = lambda *s, scale=1.0: (torch.randn(*lead, *s, generator=g) * scale).to(dt)  # noqa: E731
    return {"x_up": r(K, B), "w": r(M, K, scale=K ** -0.5), "x_lo": r(M, B), "e": r(M, B, scale=0.5),
            "w_low": r(K, M, scale=M ** -0.5), "e_low": r(K, B, scale=0.5), "w_u": r(M, K, scale=0.05)}


def _cuda(t):
    return t.to(DEV).contiguous()


SHAPES = [(64, 64, 128), (10, 64, 128), (64, 784, 128), (37, 53, 19), (64, 64, 1), (1, 1, 1), (256, 1000, 96),
          (128, 128, 256)]


@pytest.mark.parametrize("dtname", list(DTYPES))
@pytest.mark.parametrize("act", ACTS)
def test_prediction_error_all_acts(dtname, act):
    _prediction_error(64, 784, 128, dtname, act)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtname", list(DTYPES))
def test_prediction_error_shapes(shape, dtname):
    _prediction_error(*shape, dtname, "tanh")


def _prediction_error(M, K, B, dtname, act):
    dt = DTYPES[dtname]
    t = _inputs(M, K, B, dt, seed=M * 7 + K + B)
    e = torch.empty((M, B), dtype=dt, device=DEV)
    kern = _k().build_prediction_error(M, K, B, act, dtname, _k().KernelConfig())
    kern(_cuda(t["x_up"]), _cuda(t["w"]), _cuda(t["x_lo"]), e)
    ref = O.pred_err_op(t["x_up"], t["w"], t["x_lo"], act=act, sdt=dt)
    assert O.rel_inf(e.cpu(), ref) <= TOL[dtname]


@pytest.mark.parametrize("dtname", list(DTYPES))
@pytest.mark.parametrize("act", ACTS)
@pytest.mark.parametrize("save", [False, True])
def test_inference_update(dtname, act, save):
    for (M, K, B) in [(64, 64, 128), (64, 10, 128), (784, 64, 32), (33, 17, 9)]:
        dt = DTYPES[dtname]
        t = _inputs(M, K, B, dt, seed=M + 3 * K + B)
        x = _cuda(t["x_lo"])
        a = torch.empty_like(x) if save else None
        kern = _k().build_inference_update(M, K, B, act, dtname, _k().KernelConfig(), 0.5, save)
        args = (x, _cuda(t["e"]), _cuda(t["w_low"]), _cuda(t["e_low"])) + ((a,) if save else ())
        kern(*args)
        x_ref, a_ref = O.infer_update_op(t["x_lo"], t["e"], t["w_low"], t["e_low"], act=act, gamma=0.5, sdt=dt,
                                         save_activation=save)
        assert O.rel_inf(x.cpu(), x_ref) <= TOL[dtname], (M, K, B)
        if save:
            assert O.rel_inf(a.cpu(), a_ref) <= TOL[dtname], (M, K, B)


@pytest.mark.parametrize("dtname", list(DTYPES))
@pytest.mark.parametrize("act", ["relu", "tanh", "gelu"])
@pytest.mark.parametrize("recompute", [True, False])
@pytest.mark.parametrize("backend", ["auto", "simt", "outer"])
def test_weight_update(dtname, act, recompute, backend):
    for (M, K, B) in [(64, 64, 128), (10, 64, 128), (64, 784, 16), (1024, 1024, 4), (30, 70, 1), (64, 64, 300)]:
        dt = DTYPES[dtname]
        t = _inputs(M, K, B, dt, seed=5 * M + K + B)
        alpha = 0.05
        w = _cuda(t["w_u"])
        src = t["x_up"] if recompute else O.act_forward(act, t["x_up"].double()).to(dt)
        cfg = _k().KernelConfig(backend=backend)
        _k().build_weight_update(M, K, B, act, dtname, cfg, alpha, recompute)(w, _cuda(t["e"]), _cuda(src))
        ref = O.weight_update_op(t["w_u"], t["e"], src, act=act, alpha=alpha, sdt=dt, recompute_activation=recompute)
        assert O.rel_inf(w.cpu(), ref) <= TOL[dtname], (M, K, B)


@pytest.mark.parametrize("dtname", list(DTYPES))
@pytest.mark.parametrize("backend", [0, 1, 3])
def test_weight_delta_fp32_and_apply(dtname, backend):
    """dW in fp32 (the data-parallel path): compared in fp32 so bf16 rounding of W cannot hide it."""
    from lich_b200 import _native as N
    lib = N.load()
    dt = DTYPES[dtname]
    for (M, K, B) in [(64, 64, 128), (10, 784, 8), (200, 100, 40)]:
        t = _inputs(M, K, B, dt, seed=M + K)
        alpha = 1e-4
        e, x = _cuda(t["e"]), _cuda(t["x_up"])
        dw = torch.full((M, K), 7.0, dtype=torch.float32, device=DEV)
        N.check(lib.ipc_weight_delta(dw.data_ptr(), e.data_ptr(), x.data_ptr(), M, K, B, 1, alpha, 1, 0,
                                     N.act_code("tanh"), N.dtype_code(dt), backend, N.stream_handle()))
        ref = O.weight_delta_op(t["e"], t["x_up"], act="tanh", alpha=alpha, sdt=dt)
        assert O.rel_inf(dw.cpu(), ref) <= 1e-5 if dtname == "float32" else O.rel_inf(dw.cpu(), ref) <= 1e-3
        # accumulate mode adds
        N.check(lib.ipc_weight_delta(dw.data_ptr(), e.data_ptr(), x.data_ptr(), M, K, B, 1, alpha, 1, 1,
                                     N.act_code("tanh"), N.dtype_code(dt), backend, N.stream_handle()))
        assert O.rel_inf(dw.cpu(), 2 * ref) <= 1e-3
        w = _cuda(t["w_u"])
        N.check(lib.ipc_weight_apply(w.data_ptr(), dw.data_ptr(), M * K, N.dtype_code(dt), N.stream_handle()))
        assert O.rel_inf(w.cpu(), (t["w_u"].double() + dw.cpu().double()).to(dt)) <= TOL[dtname]


@pytest.mark.parametrize("dtname", list(DTYPES))
def test_grouped_equals_singleton_bitwise(dtname):
    """The layer-batched launch must give exactly the per-layer results (max_w = max_x = max_e = 0)."""
    from lich_b200 import layer_batching as LB
    K_ = _k()
    dt = DTYPES[dtname]
    G, D, B = 3, 64, 128
    t = _inputs(D, D, B, dt, seed=99, groups=G)
    cfg = K_.KernelConfig()
    e_g = torch.empty((G, D, B), dtype=dt, device=DEV)
    LB.build_prediction_error_batched(D, D, B, G, "tanh", dtname, cfg)(_cuda(t["x_up"]), _cuda(t["w"]),
                                                                       _cuda(t["x_lo"]), e_g)
    x_g = _cuda(t["x_lo"])
    LB.build_inference_update_batched(D, D, B, G, "tanh", dtname, cfg, 0.5)(x_g, _cuda(t["e"]), _cuda(t["w_low"]),
                                                                           _cuda(t["e_low"]))
    w_g = _cuda(t["w_u"])
    LB.build_weight_update_batched(D, D, B, G, "tanh", dtname, cfg, 0.01)(w_g, _cuda(t["e"]), _cuda(t["x_up"]))
    for g in range(G):
        e1 = torch.empty((D, B), dtype=dt, device=DEV)
        K_.build_prediction_error(D, D, B, "tanh", dtname, cfg)(_cuda(t["x_up"][g]), _cuda(t["w"][g]),
                                                                _cuda(t["x_lo"][g]), e1)
        assert torch.equal(e1, e_g[g])
        x1 = _cuda(t["x_lo"][g])
        K_.build_inference_update(D, D, B, "tanh", dtname, cfg, 0.5)(x1, _cuda(t["e"][g]), _cuda(t["w_low"][g]),
                                                                    _cuda(t["e_low"][g]))
        assert torch.equal(x1, x_g[g])
        w1 = _cuda(t["w_u"][g])
        K_.build_weight_update(D, D, B, "tanh", dtname, cfg, 0.01)(w1, _cuda(t["e"][g]), _cuda(t["x_up"][g]))
        assert torch.equal(w1, w_g[g])


def test_reference_smoke_shapes_fp16_relu():
    """The reference's own smoke test (scripts/smoke.py:21-66), shapes, scales and tolerances."""
    K_ = _k()
    cfg = K_.KernelConfig(64, 128, 16, 128, 2, True, 8, False)
    torch.manual_seed(0)
    a = dict(M=64, K=64, B=128)
    x_up = torch.randn((a["K"], a["B"]), device=DEV, dtype=torch.float16)
    w = torch.randn((a["M"], a["K"]), device=DEV, dtype=torch.float16) * 0.05
    x_lo = torch.randn((a["M"], a["B"]), device=DEV, dtype=torch.float16)
    e = torch.empty_like(x_lo)
    K_.build_prediction_error(a["M"], a["K"], a["B"], "relu", "float16", cfg)(x_up, w, x_lo, e)
    ref_e = x_lo - w @ torch.relu(x_up)
    torch.testing.assert_close(e, ref_e, rtol=2e-2, atol=2e-2)
    x = x_lo.clone()
    e_low = torch.randn_like(x_up)
    infer_w = torch.randn((a["K"], a["M"]), device=DEV, dtype=torch.float16) * 0.05
    K_.build_inference_update(a["M"], a["K"], a["B"], "relu", "float16", cfg, 0.5)(x, e, infer_w, e_low)
    ref_x = x_lo + 0.5 * (-ref_e + (x_lo > 0).to(torch.float16) * (infer_w.T @ e_low))
    torch.testing.assert_close(x, ref_x, rtol=3e-2, atol=3e-2)
    w2 = w.clone()
    alpha = 1e-4
    K_.build_weight_update(a["M"], a["K"], a["B"], "relu", "float16", cfg, alpha, True)(w2, e, x_up)
    ref_w = w + alpha * e.float() @ torch.relu(x_up).float().T
    torch.testing.assert_close(w2.float(), ref_w, rtol=2e-2, atol=2e-2)
    m2, k2, b2 = 10, 64, 128
    xu2 = torch.randn((k2, b2), device=DEV, dtype=torch.float16)
    wsmall = torch.randn((m2, k2), device=DEV, dtype=torch.float16) * 0.05
    xsmall = torch.randn((m2, b2), device=DEV, dtype=torch.float16)
    esmall = torch.empty_like(xsmall)
    K_.build_prediction_error(m2, k2, b2, "relu", "float16", cfg)(xu2, wsmall, xsmall, esmall)
    torch.testing.assert_close(esmall, xsmall - wsmall @ torch.relu(xu2), rtol=3e-2, atol=3e-2)
    w_saved = w.clone()
    K_.build_weight_update(a["M"], a["K"], a["B"], "relu", "float16", cfg, alpha, False)(w_saved, e,
                                                                                        torch.relu(x_up).contiguous())
    torch.testing.assert_close(w_saved.float(), ref_w, rtol=2e-2, atol=2e-2)


def test_outer_sign_matches_gemm_and_oracle():
    """Small-B updater adds +alpha (the oracle's sign), unlike the reference's eager path."""
    from lich_b200.weight_update_specialization import SmallBWeightUpdater
    K_ = _k()
    M, K, B = 64, 784, 4
    t = _inputs(M, K, B, torch.float16, seed=1)
    up = SmallBWeightUpdater(alpha=0.05).make_singleton(M=M, K=K, B=B, activation="relu", dtype=torch.float16)
    w1 = _cuda(t["w_u"])
    up(w1, _cuda(t["e"]), _cuda(t["x_up"]))
    w2 = _cuda(t["w_u"])
    K_.build_weight_update(M, K, B, "relu", "float16", K_.KernelConfig(backend="simt"), 0.05)(w2, _cuda(t["e"]),
                                                                                            _cuda(t["x_up"]))
    ref = O.weight_update_op(t["w_u"], t["e"], t["x_up"], act="relu", alpha=0.05, sdt=torch.float16)
    assert O.rel_inf(w1.cpu(), ref) <= 1e-2 and O.rel_inf(w2.cpu(), ref) <= 1e-2
    delta = (w1.float() - _cuda(t["w_u"]).float()).abs().max().item()
    assert delta > 0


def test_edge_cases():
    K_ = _k()
    cfg = K_.KernelConfig()
    # B = 0: nothing to do, no error
    z = torch.empty((64, 0), dtype=torch.float16, device=DEV)
    K_.build_prediction_error(64, 64, 0, "tanh", "float16", cfg)(torch.empty((64, 0), dtype=torch.float16, device=DEV),
                                                                 torch.zeros((64, 64), dtype=torch.float16, device=DEV),
                                                                 z, z)
    w = torch.randn((8, 8), device=DEV, dtype=torch.float16)
    w0 = w.clone()
    K_.build_weight_update(8, 8, 0, "tanh", "float16", cfg, 0.1)(w, torch.empty((8, 0), dtype=torch.float16, device=DEV),
                                                                 torch.empty((8, 0), dtype=torch.float16, device=DEV))
    assert torch.equal(w, w0)
    # K = 0: E = X_lo exactly
    x_lo = torch.randn((5, 7), device=DEV, dtype=torch.float16)
    e = torch.empty_like(x_lo)
    K_.build_prediction_error(5, 0, 7, "tanh", "float16", cfg)(torch.empty((0, 7), dtype=torch.float16, device=DEV),
                                                               torch.empty((5, 0), dtype=torch.float16, device=DEV),
                                                               x_lo, e)
    assert torch.equal(e, x_lo)
    # wrong shape / dtype / layout -> ValueError before launch
    kern = K_.build_prediction_error(64, 64, 128, "tanh", "float16", cfg)
    good = torch.zeros((64, 128), dtype=torch.float16, device=DEV)
    with pytest.raises(ValueError):
        kern(good, torch.zeros((64, 64), dtype=torch.float16, device=DEV), good, torch.zeros((64, 127),
                                                                                            dtype=torch.float16,
                                                                                            device=DEV))
    with pytest.raises(ValueError):
        kern(good.float(), torch.zeros((64, 64), dtype=torch.float16, device=DEV), good, good)
    with pytest.raises(ValueError):
        kern(torch.zeros((128, 64), dtype=torch.float16, device=DEV).T, torch.zeros((64, 64), dtype=torch.float16,
                                                                                     device=DEV), good, good)


def test_forward_matches_oracle():
    K_ = _k()
    for dtname in DTYPES:
        dt = DTYPES[dtname]
        t = _inputs(64, 784, 128, dt, seed=3)
        out = torch.empty((64, 128), dtype=dt, device=DEV)
        K_.build_forward(64, 784, 128, "tanh", dtname)(_cuda(t["x_up"]), _cuda(t["w"]), out)
        a = O.act_forward("tanh", t["x_up"].double()).to(dt).double()
        ref = (t["w"].double() @ a).to(dt)
        assert O.rel_inf(out.cpu(), ref) <= TOL[dtname]
