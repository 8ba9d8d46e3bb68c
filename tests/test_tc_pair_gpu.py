"""GPU parity of the tcgen05 kernel's CTA-pair form (``ipc_gemm_tune_t.pair = 2``: 256 x 256 tiles,
``tcgen05.mma.cta_group::2`` issued by the even CTA of a two-CTA cluster, each CTA holding 128 rows of
A and 128 columns of B, the odd CTA's TMA loads completing on the leader's stage barriers).

Every mode against the CPU oracle (storage rounding, float64 accumulation) at the 16-bit gate 1e-2
(fp32 weight delta 1e-3), on shapes with row and column tails (M not a multiple of 256, B or K not a
multiple of 256), grouped launches, and the agreement with the single-CTA kernel.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SHAPES = [(256, 256, 256), (384, 512, 264), (1000, 1000, 520), (512, 4096, 256), (136, 256, 512), (2048, 768, 1024)]


def _tune():
    from lich_b200.tilelang_kernels import KernelConfig
    return KernelConfig(tc_pair=2).tune()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("mode_name", ["PRED", "FORWARD", "INFER", "WEIGHT", "WDELTA"])
def test_pair_modes_match_oracle(mode_name, shape, dt):
    from lich_b200 import _native as N
    from tests.test_tc_gpu import _r, _ref
    mode = getattr(N, f"MODE_{mode_name}")
    M, K, B = shape
    ins = {}
    if mode == N.MODE_PRED:
        ins = dict(a=_r((M, K), 1, K ** -0.5, dt), b=_r((K, B), 2, 1, dt), aux=_r((M, B), 3, 1, dt),
                   out=torch.zeros((M, B), dtype=dt))
    elif mode == N.MODE_FORWARD:
        ins = dict(a=_r((M, K), 1, K ** -0.5, dt), b=_r((K, B), 2, 1, dt), out=torch.zeros((M, B), dtype=dt),
                   aux2=torch.zeros((M, B), dtype=dt))
    elif mode == N.MODE_INFER:
        ins = dict(a=_r((K, M), 1, M ** -0.5, dt), b=_r((K, B), 2, 0.5, dt), aux=_r((M, B), 3, 0.5, dt),
                   out=_r((M, B), 4, 1, dt), aux2=torch.zeros((M, B), dtype=dt))
    elif mode == N.MODE_WEIGHT:
        ins = dict(a=_r((M, B), 1, 0.5, dt), b=_r((K, B), 2, 1, dt), out=_r((M, K), 3, 0.05, dt))
    else:
        ins = dict(a=_r((M, B), 1, 0.5, dt), b=_r((K, B), 2, 1, dt), out=torch.zeros((M, K), dtype=torch.float32))
    scale = 0.5 if mode == N.MODE_INFER else 0.01
    flags = N.FLAG_AOUT_STORED if mode == N.MODE_INFER else 0
    got = {}
    for name, tune in (("pair", _tune()), ("single", None)):
        dev = {k: v.to(DEV) for k, v in ins.items()}
        N.fused_gemm(mode, dev["a"], dev["b"], dev["out"], dev.get("aux"), dev.get("aux2"), M=M, K=K, B=B,
                     scale=scale, flags=flags, act="tanh", dtype=dt, algo="tcgen05", tune=tune)
        torch.cuda.synchronize()
        assert N.device_status() == 0
        got[name] = {k: v.cpu() for k, v in dev.items()}
    ref, ref_a = _ref(mode, ins, dt, scale)
    tol = 1e-3 if mode == N.MODE_WDELTA else 1e-2
    assert O.rel_inf(got["pair"]["out"], ref) <= tol
    if ref_a is not None:
        assert O.rel_inf(got["pair"]["aux2"], ref_a) <= tol
    # the same products in the same order over K (fp32 dW: the pair may add two batch halves, a + b
    # against the single kernel's one sum, a few fp32 roundings): the pair agrees with the single-CTA kernel
    assert O.rel_inf(got["pair"]["out"], got["single"]["out"]) <= (4e-6 if mode == N.MODE_WDELTA else 1e-2)


@pytest.mark.parametrize("dt", [torch.bfloat16])
def test_pair_grouped_and_builders(dt):
    """Grouped launches and a builder whose KernelConfig asks for pairs (f on B stored once first)."""
    from lich_b200 import _native as N
    from lich_b200.tilelang_kernels import KernelConfig, build_prediction_error, build_weight_update
    from tests.test_tc_gpu import _batched_ref, _r
    G, M, K, B = 3, 512, 256, 512
    ins = dict(a=_r((G, M, K), 5, K ** -0.5, dt), b=_r((G, K, B), 6, 1, dt), aux=_r((G, M, B), 7, 1, dt),
               out=torch.zeros((G, M, B), dtype=dt))
    dev = {k: v.to(DEV) for k, v in ins.items()}
    N.fused_gemm(N.MODE_PRED, dev["a"], dev["b"], dev["out"], dev["aux"], M=M, K=K, B=B, groups=G, dtype=dt,
                 algo="tcgen05", tune=_tune())
    ref, _ = _batched_ref(N.MODE_PRED, ins, dt, 0.0, G)
    assert O.rel_inf(dev["out"].cpu(), ref) <= 1e-2
    kc = KernelConfig(tc_pair=2)
    x_up, w, x_lo = _r((1024, 768), 8, 1, dt), _r((1024, 1024), 9, 1024 ** -0.5, dt), _r((1024, 768), 10, 1, dt)
    e = torch.empty((1024, 768), device=DEV, dtype=dt)
    build_prediction_error(1024, 1024, 768, "tanh", "bfloat16", kc)(x_up.to(DEV), w.to(DEV), x_lo.to(DEV), e)
    assert O.rel_inf(e.cpu(), O.pred_err_op(x_up, w, x_lo, act="tanh", sdt=dt)) <= 1e-2
    wt = w.to(DEV).clone()
    ee = _r((1024, 768), 11, 0.5, dt)
    build_weight_update(1024, 1024, 768, "tanh", "bfloat16", kc, 1e-2, True)(wt, ee.to(DEV), x_up.to(DEV))
    ref = O.weight_update_op(w, ee, x_up, act="tanh", alpha=1e-2, sdt=dt, recompute_activation=True)
    assert O.rel_inf(wt.cpu(), ref) <= 1e-2
    torch.cuda.synchronize()
    assert N.device_status() == 0


def test_pair_weight_delta_halves_deterministic():
    """fp32 dW on CTA pairs in two batch halves added into zeros (atomics): bitwise the same on every
    run, within 1e-3 of the oracle on sampled rows, and within 4e-6 (fp32 rounding of a + b against one
    sum) of the unsplit pair kernel."""
    from lich_b200 import _native as N
    from lich_b200.tilelang_kernels import KernelConfig
    M, K, B, dt, scale = 2560, 2560, 2048, torch.bfloat16, 1e-3  # 100 pair tiles: 2 waves, 3 half-waves
    e, a = _r2((M, B), 21, 0.5, dt), _r2((K, B), 22, 1.0, dt)
    ed, ad = e.to(DEV), a.to(DEV)
    outs = []
    for tune in (KernelConfig(tc_pair=2).tune(), KernelConfig(tc_pair=2).tune(), KernelConfig(tc_pair=2, tc_splits=1).tune()):
        out = torch.full((M, K), 7.0, device=DEV)  # stale contents must not leak into the result
        N.fused_gemm(N.MODE_WDELTA, ed, ad, out, M=M, K=K, B=B, scale=scale, dtype=dt, algo="tcgen05", tune=tune)
        torch.cuda.synchronize()
        assert N.device_status() == 0
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1])
    rows = torch.cat([torch.arange(0, 128), torch.arange(M - 128, M)])
    ref = scale * (e[rows].double() @ a.double().T)
    assert O.rel_inf(outs[0][rows], ref) <= 1e-3
    assert O.rel_inf(outs[0], outs[2]) <= 4e-6


def _r2(shape, seed, scale, dt):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dt)
