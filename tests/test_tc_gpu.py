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


def _dtname(dt):
    return "float16" if dt == torch.float16 else "bfloat16"


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", [(256, 512, 512), (1000, 1000, 264), (128, 4096, 256), (64, 512, 264)])
def test_builders_with_f_on_b_run_on_tensor_cores(shape, dt):
    """The reference-facing builders with f applied to their B operand (prediction error, forward, weight
    update in recompute mode) on tensor-core shapes: f(B) is stored once in the operator's workspace and
    the tcgen05 GEMM runs on it -- two launches (three with a split-K reduce) -- with the oracle's
    recompute-mode answer, and bit-identical to ipc_activate followed by the stored-operand GEMM."""
    from lich_b200.tilelang_kernels import KernelConfig, build_forward, build_prediction_error, build_weight_update
    N = _N()
    M, K, B = shape
    kc = KernelConfig()
    x_up, w, x_lo = _r((K, B), 51, 1, dt), _r((M, K), 52, K ** -0.5, dt), _r((M, B), 53, 1, dt)
    e_lo = _r((M, B), 54, 0.5, dt)
    d = {k: v.to(DEV) for k, v in dict(x_up=x_up, w=w, x_lo=x_lo, e_lo=e_lo).items()}
    a_up = torch.empty_like(d["x_up"])
    N.check(N.load().ipc_activate(a_up.data_ptr(), d["x_up"].data_ptr(), a_up.numel(), N.act_code("tanh"),
                                  N.dtype_code(dt), N.stream_handle(DEV)))
    # prediction error
    e = torch.empty_like(d["x_lo"])
    op = build_prediction_error(M, K, B, "tanh", _dtname(dt), kc)
    op(d["x_up"], d["w"], d["x_lo"], e)  # first call allocates the workspace
    n0 = N.launch_count()
    op(d["x_up"], d["w"], d["x_lo"], e)
    assert N.launch_count() - n0 == 2
    e2 = torch.empty_like(e)
    N.fused_gemm(N.MODE_PRED, d["w"], a_up, e2, d["x_lo"], M=M, K=K, B=B, dtype=dt, algo="tcgen05")
    assert torch.equal(e, e2)
    assert O.rel_inf(e.cpu(), O.pred_err_op(x_up, w, x_lo, act="tanh", sdt=dt)) <= 1e-2
    # forward
    out = torch.empty_like(d["x_lo"])
    build_forward(M, K, B, "tanh", _dtname(dt), kc)(d["x_up"], d["w"], out)
    ref = (w.double() @ O.act_forward("tanh", x_up.double()).to(dt).double()).to(dt)
    assert O.rel_inf(out.cpu(), ref) <= 1e-2
    # weight update, recompute mode
    wt = d["w"].clone()
    wop = build_weight_update(M, K, B, "tanh", _dtname(dt), kc, 1e-2, True)
    n0 = N.launch_count()
    wop(wt, d["e_lo"], d["x_up"])
    assert N.launch_count() - n0 in (2, 3)
    w2 = d["w"].clone()
    ws = torch.empty(N.SPLITK_WORKSPACE_BYTES // 4, device=DEV, dtype=torch.float32)
    N.fused_gemm(N.MODE_WEIGHT, d["e_lo"], a_up, w2, M=M, K=K, B=B, scale=1e-2, dtype=dt, algo="tcgen05",
                 workspace=ws)
    assert torch.equal(wt, w2)
    ref = O.weight_update_op(w, e_lo, x_up, act="tanh", alpha=1e-2, sdt=dt, recompute_activation=True)
    assert O.rel_inf(wt.cpu(), ref) <= 1e-2
    torch.cuda.synchronize()
    assert N.device_status() == 0


def test_workspace_query():
    """ipc_fused_gemm_ws_bytes: the stored activation (rounded to 256 B) on tensor-core shapes with f on B,
    plus the split-K partials for a weight update; nothing for shapes the generic kernels take."""
    N = _N()
    act = N.FLAG_ACTIVATE_B
    assert N.workspace_bytes(N.MODE_PRED, M=512, K=512, B=512, flags=act) == 512 * 512 * 2
    assert N.workspace_bytes(N.MODE_PRED, M=512, K=512, B=512, flags=0) == 0
    assert N.workspace_bytes(N.MODE_PRED, M=16, K=64, B=64, flags=act) == 0
    assert N.workspace_bytes(N.MODE_WEIGHT, M=512, K=512, B=4096, flags=act) == 512 * 4096 * 2 + (16 << 20)
    assert N.workspace_bytes(N.MODE_WEIGHT, M=512, K=512, B=4096, flags=0) == 16 << 20
    assert N.workspace_bytes(N.MODE_WEIGHT, M=512, K=512, B=8, flags=act) == 0  # outer-product kernel
    assert N.workspace_bytes(N.MODE_PRED, M=512, K=512, B=512, flags=act, dtype=torch.float32) == 0


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("act", ["relu", "tanh", "sigmoid", "silu", "gelu", "identity"])
def test_activate_matches_oracle(act, dt):
    """ipc_activate: A = cast(f(X)) elementwise (16-bit: 16-byte vectors and a scalar tail; also a view
    that starts mid-vector, which takes the scalar kernel)."""
    N = _N()
    for n, off in ((1 << 20, 0), (8 * 1000 + 5, 0), (4099, 3)):
        x = (torch.randn(n + off, generator=torch.Generator().manual_seed(n)) * 2).to(dt)
        xd = x.to(DEV)[off:]
        a = torch.empty(n + off, dtype=dt, device=DEV)[off:]
        N.check(N.load().ipc_activate(a.data_ptr(), xd.data_ptr(), n, N.act_code(act), N.dtype_code(dt),
                                      N.stream_handle(DEV)))
        ref = O.act_forward(act, x[off:].double()).to(dt)
        assert O.rel_inf(a.cpu(), ref) <= (1e-5 if dt == torch.float32 else 1e-2), (n, off)
