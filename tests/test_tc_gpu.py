"""GPU parity of the tcgen05 / TMEM / TMA kernel (``ipc_fused_gemm`` with IPC_ALGO_TCGEN05).

Every mode against the CPU oracle (storage rounding of the reference kernels,
float64 accumulation), bound ``max|got - ref| / max|ref| <= 1e-2`` (the 16-bit
gate); the fp32 weight delta ``<= 1e-3``.  Also: tails in M / N / K (TMA zero
fill + TMA store clipping + epilogue masks), grouped launches, agreement with
the mma.sync kernel (two storage rounding steps), the staged I epilogue without
an A_out operand, operands that start mid-vector (routed to the generic kernel),
and a clean device status word (no bounded wait expired).
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
DTYPES = [torch.float16, torch.bfloat16]
SHAPES = [(128, 64, 128), (256, 512, 512), (1000, 1000, 264), (384, 200, 136), (128, 4096, 256), (64, 256, 264),
          (72, 128, 136)]


def _N():
    from lich_b200 import _native as N
    return N


def _r(shape, seed, scale=1.0, dt=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dt)


def _run(mode, M, K, B, dt, algo, groups=1, act="tanh", flags=0, seed=0):
    """Run one mode; returns CPU inputs and outputs."""
    N = _N()
    lead = (groups,) if groups > 1 else ()
    ins = {}
    if mode == N.MODE_PRED:
        ins = dict(a=_r(lead + (M, K), seed, K ** -0.5, dt), b=_r(lead + (K, B), seed + 1, 1, dt),
                   aux=_r(lead + (M, B), seed + 2, 1, dt), out=torch.zeros(lead + (M, B), dtype=dt))
    elif mode == N.MODE_FORWARD:
        ins = dict(a=_r(lead + (M, K), seed, K ** -0.5, dt), b=_r(lead + (K, B), seed + 1, 1, dt),
                   out=torch.zeros(lead + (M, B), dtype=dt), aux2=torch.zeros(lead + (M, B), dtype=dt))
    elif mode == N.MODE_INFER:
        ins = dict(a=_r(lead + (K, M), seed, M ** -0.5, dt), b=_r(lead + (K, B), seed + 1, 0.5, dt),
                   aux=_r(lead + (M, B), seed + 2, 0.5, dt), out=_r(lead + (M, B), seed + 3, 1, dt),
                   aux2=torch.zeros(lead + (M, B), dtype=dt))
    elif mode == N.MODE_WEIGHT:
        ins = dict(a=_r(lead + (M, B), seed, 0.5, dt), b=_r(lead + (K, B), seed + 1, 1, dt),
                   out=_r(lead + (M, K), seed + 2, 0.05, dt))
    else:
        ins = dict(a=_r(lead + (M, B), seed, 0.5, dt), b=_r(lead + (K, B), seed + 1, 1, dt),
                   out=torch.zeros(lead + (M, K), dtype=torch.float32))
    dev = {k: v.to(DEV) for k, v in ins.items()}
    scale = 0.5 if mode == N.MODE_INFER else 0.01
    N.fused_gemm(mode, dev["a"], dev["b"], dev["out"], dev.get("aux"), dev.get("aux2"), M=M, K=K, B=B,
                 groups=groups, scale=scale, flags=flags, act=act, dtype=dt, algo=algo)
    torch.cuda.synchronize()
    assert N.device_status() == 0
    return ins, {k: v.cpu() for k, v in dev.items()}, scale


def _ref(mode, ins, dt, scale, act="tanh", stored=True):
    N = _N()
    if mode == N.MODE_PRED:
        return O.pred_err_op(ins["b"], ins["a"], ins["aux"], act="identity", sdt=dt), None
    if mode == N.MODE_FORWARD:
        out = (ins["a"].double() @ ins["b"].double()).to(dt)
        return out, O.act_forward(act, out.double()).to(dt)
    if mode == N.MODE_INFER:
        x_new, _ = O.infer_update_op(ins["out"], ins["aux"], ins["a"], ins["b"], act=act, gamma=scale, sdt=dt)
        return x_new, O.act_forward(act, x_new.double()).to(dt)
    if mode == N.MODE_WEIGHT:
        return O.weight_update_op(ins["out"], ins["a"], ins["b"], act="identity", alpha=scale, sdt=dt,
                                  recompute_activation=False), None
    return O.weight_delta_op(ins["a"], ins["b"], act="identity", alpha=scale, sdt=dt, recompute_activation=False), None


def _batched_ref(mode, ins, dt, scale, groups):
    if groups == 1:
        return _ref(mode, ins, dt, scale)
    outs, a2 = [], []
    for g in range(groups):
        o, a = _ref(mode, {k: v[g] for k, v in ins.items()}, dt, scale)
        outs.append(o)
        a2.append(a)
    return torch.stack(outs), (None if a2[0] is None else torch.stack(a2))


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("mode_name", ["PRED", "FORWARD", "INFER", "WEIGHT", "WDELTA"])
def test_tcgen05_modes_match_oracle(mode_name, shape, dt):
    N = _N()
    mode = getattr(N, f"MODE_{mode_name}")
    M, K, B = shape
    flags = N.FLAG_AOUT_STORED if mode == N.MODE_INFER else 0
    ins, got, scale = _run(mode, M, K, B, dt, "tcgen05", flags=flags)
    ref, ref_a = _ref(mode, ins, dt, scale)
    tol = 1e-3 if mode == N.MODE_WDELTA else 1e-2
    assert O.rel_inf(got["out"], ref) <= tol
    if ref_a is not None:
        assert O.rel_inf(got["aux2"], ref_a) <= tol


@pytest.mark.parametrize("dt", DTYPES)
def test_tcgen05_grouped(dt):
    N = _N()
    for mode in (N.MODE_PRED, N.MODE_INFER, N.MODE_WEIGHT):
        flags = N.FLAG_AOUT_STORED if mode == N.MODE_INFER else 0
        ins, got, scale = _run(mode, 256, 256, 256, dt, "tcgen05", groups=3, flags=flags, seed=5)
        ref, _ = _batched_ref(mode, ins, dt, scale, 3)
        assert O.rel_inf(got["out"], ref) <= 1e-2


@pytest.mark.parametrize("dt", DTYPES)
def test_tcgen05_agrees_with_mma_sync(dt):
    """Same operands through both tensor-core paths."""
    N = _N()
    for mode in (N.MODE_PRED, N.MODE_INFER, N.MODE_WEIGHT, N.MODE_WDELTA):
        flags = N.FLAG_AOUT_STORED if mode == N.MODE_INFER else 0
        _, a, _ = _run(mode, 512, 768, 384, dt, "tcgen05", flags=flags, seed=9)
        _, b, _ = _run(mode, 512, 768, 384, dt, "simt", flags=flags, seed=9)
        # different summation orders, and the tensor-core epilogue evaluates f / f' with the MUFU
        # forms (the mma.sync kernel with tanhf): stored outputs may differ by a storage rounding step
        assert O.rel_inf(a["out"], b["out"]) <= (8e-3 if dt == torch.bfloat16 else 2e-3)


def test_tcgen05_rejects_activated_operand_and_bad_strides():
    """f on the B operand is never applied inside the tensor-core GEMM; odd inner sizes break TMA strides."""
    N = _N()
    x = torch.zeros(256, 256, dtype=torch.float16, device=DEV)
    with pytest.raises(N.IpcError):
        N.fused_gemm(N.MODE_PRED, x, x, x, x, M=256, K=256, B=256, flags=N.FLAG_ACTIVATE_B, act="tanh",
                     algo="tcgen05")
    y = torch.zeros(250, 250, dtype=torch.float16, device=DEV)
    with pytest.raises(N.IpcError):
        N.fused_gemm(N.MODE_PRED, y, y, y, y, M=250, K=250, B=250, algo="tcgen05")
    # auto falls back to the generic kernel for the same request
    N.fused_gemm(N.MODE_PRED, x, x, x, x, M=256, K=256, B=256, flags=N.FLAG_ACTIVATE_B, act="tanh")
    torch.cuda.synchronize()


@pytest.mark.parametrize("mode_name", ["PRED", "INFER", "WEIGHT"])
def test_misaligned_views_take_the_generic_kernel(mode_name):
    """Operands that start 8 bytes into an allocation cannot be TMA-mapped: auto routes them to the
    generic kernel, which gives the oracle's answer."""
    N = _N()
    mode = getattr(N, f"MODE_{mode_name}")
    M = K = B = 256
    dt = torch.float16
    ins, _, scale = _run(mode, M, K, B, dt, "tcgen05", seed=21)
    dev = {}
    for k, v in ins.items():
        buf = torch.zeros(v.numel() + 4, dtype=v.dtype, device=DEV)
        view = buf[4:].view(v.shape)
        view.copy_(v.to(DEV))
        assert view.data_ptr() % 16 == 8
        dev[k] = view
    N.fused_gemm(mode, dev["a"], dev["b"], dev["out"], dev.get("aux"), dev.get("aux2"), M=M, K=K, B=B,
                 scale=scale, flags=N.FLAG_AOUT_STORED if mode == N.MODE_INFER else 0, act="tanh", dtype=dt)
    torch.cuda.synchronize()
    assert N.device_status() == 0
    ref, ref_a = _ref(mode, ins, dt, scale)
    assert O.rel_inf(dev["out"].cpu(), ref) <= 1e-2
    if ref_a is not None:
        assert O.rel_inf(dev["aux2"].cpu(), ref_a) <= 1e-2


@pytest.mark.parametrize("dt", DTYPES)
def test_infer_without_activation_output(dt):
    """The staged I epilogue with no A_out operand writes X only."""
    N = _N()
    M, K, B = 384, 1024, 264
    ins = dict(a=_r((K, M), 31, M ** -0.5, dt), b=_r((K, B), 32, 0.5, dt), aux=_r((M, B), 33, 0.5, dt),
               out=_r((M, B), 34, 1, dt))
    dev = {k: v.to(DEV) for k, v in ins.items()}
    N.fused_gemm(N.MODE_INFER, dev["a"], dev["b"], dev["out"], dev["aux"], None, M=M, K=K, B=B, scale=0.5,
                 act="tanh", dtype=dt, algo="tcgen05")
    torch.cuda.synchronize()
    assert N.device_status() == 0
    ref, _ = _ref(N.MODE_INFER, ins, dt, 0.5)
    assert O.rel_inf(dev["out"].cpu(), ref) <= 1e-2
    assert torch.equal(dev["aux"].cpu(), ins["aux"])  # E is read, never written


def test_cta_cap_keeps_results():
    """A GEMM launched with fewer persistent CTAs than SMs (ipc_set_max_ctas) gives the same answer."""
    N = _N()
    try:
        for cap in (16, 1):
            N.set_max_ctas(cap)
            for mode in (N.MODE_PRED, N.MODE_WDELTA):
                ins, got, scale = _run(mode, 512, 768, 384, torch.float16, "tcgen05", seed=41)
                ref, _ = _ref(mode, ins, torch.float16, scale)
                assert O.rel_inf(got["out"], ref) <= (1e-3 if mode == N.MODE_WDELTA else 1e-2), (cap, mode)
    finally:
        N.set_max_ctas(0)
    with pytest.raises(ValueError):  # IPC_ERR_ARG
        N.set_max_ctas(-1)
