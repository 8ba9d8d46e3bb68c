"""GPU tests of the fused optimizer weight update (``ipc_weight_update_opt``, IPCConfig.optimizer).

Against the oracle's restatement of torch.optim.SGD / AdamW (``oracle.optim_step``, itself checked
step for step against torch.optim on the CPU) with the gradient of the energy g = -E f(x)^T:
W within 1e-2 (16-bit storage; the gate of the 16-bit path), the fp32 state within 1e-2, on every
path the update takes: the tcgen05 epilogue, its split-K reduce pass, the small-batch outer-product
kernel and the workspace fallback (fp32 product, then the step).
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

OPTS = {"adamw": dict(kind="adamw", lr=1e-3, weight_decay=0.05, betas=(0.9, 0.99), eps=1e-8),
        "sgd_momentum": dict(kind="sgd", lr=1e-3, momentum=0.9, weight_decay=0.01)}


def _step_ref(w, e, x, state, opt, dt, recompute):
    a = O.act_forward("tanh", x.double()).to(dt).double() if recompute else x.double()
    g = -(e.double() @ a.T)
    return O.optim_step(w, g, state, **opt)


@pytest.mark.parametrize("opt_name", list(OPTS))
@pytest.mark.parametrize("shape,dt", [((512, 768, 512), torch.bfloat16),    # tcgen05 epilogue
                                      ((256, 512, 16384), torch.bfloat16),  # tcgen05 split-K reduce
                                      ((384, 1000, 8), torch.float16),      # outer-product kernel
                                      ((10, 64, 96), torch.bfloat16),       # workspace fallback
                                      ((40, 24, 33), torch.float32)])       # fp32: workspace fallback
@pytest.mark.parametrize("recompute", [False, True])
def test_weight_update_opt_matches_oracle(opt_name, shape, dt, recompute):
    from lich_b200 import _native as N
    M, K, B = shape
    opt = OPTS[opt_name]
    g = torch.Generator().manual_seed(M + K + B)
    w = (torch.rand(M, K, generator=g) - 0.5).to(dt)
    e = (torch.randn(M, B, generator=g) * 0.5).to(dt)
    x = torch.randn(K, B, generator=g).to(dt)
    wd, ed, xd = w.to(DEV), e.to(DEV), x.to(DEV)
    m = torch.zeros(M, K, device=DEV)
    v = torch.zeros(M, K, device=DEV) if opt["kind"] == "adamw" else None
    ws = torch.empty(max(M * K, (K * B * 2 + 255) // 256 * 64 + N.SPLITK_WORKSPACE_BYTES // 4), device=DEV)
    state, ref = {}, w.double()
    for step in (1, 2):
        N.weight_update_opt(wd, ed, xd, M=M, K=K, B=B, step=step, m=m, v=v, recompute=recompute, act="tanh",
                            dtype=dt, workspace=ws, **opt)
        ref = _step_ref(ref.to(dt).double(), e, x, state, opt, dt, recompute)
    torch.cuda.synchronize()
    assert N.device_status() == 0
    assert O.rel_inf(wd.cpu(), ref) <= 1e-2
    assert O.rel_inf(m.cpu(), state["m"]) <= 1e-2
    if v is not None:
        assert O.rel_inf(v.cpu(), state["v"]) <= 1e-2


def test_weight_update_opt_errors():
    from lich_b200 import _native as N
    w = torch.zeros(64, 64, device=DEV, dtype=torch.bfloat16)
    e = torch.zeros(64, 128, device=DEV, dtype=torch.bfloat16)
    x = torch.zeros(64, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # AdamW without its second moment
        N.weight_update_opt(w, e, x, M=64, K=64, B=128, kind="adamw", lr=1e-3, m=torch.zeros(64, 64, device=DEV),
                            dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # step 0
        N.weight_update_opt(w, e, x, M=64, K=64, B=128, kind="adamw", lr=1e-3, step=0,
                            m=torch.zeros(64, 64, device=DEV), v=torch.zeros(64, 64, device=DEV),
                            dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # a shape the fused kernels do not serve needs the workspace
        N.weight_update_opt(w[:10], e[:10], x, M=10, K=64, B=128, kind="sgd", lr=1e-3, dtype=torch.bfloat16)


@pytest.mark.parametrize("dims,B,dt", [((104, 512, 512, 1024), 512, torch.bfloat16),
                                       ((10, 64, 64, 784), 8, torch.float16)])
def test_trainer_adamw_two_steps(dims, B, dt):
    """TileLangIPC(optimizer="adamw"): two training steps (T = 4) against the oracle with the kernels'
    storage rounding (oracle.train_step_opt_storage): the states are stored in 16 bits, and AdamW's
    normalised step turns their rounding into differences the fp32 oracle does not share."""
    from lich_b200 import synthetic as S
    from lich_b200.trainer import IPCConfig, TileLangIPC
    opt = dict(kind="adamw", lr=1e-3, weight_decay=0.01, betas=(0.9, 0.999), eps=1e-8)
    m = TileLangIPC(IPCConfig(dims=dims, alpha=opt["lr"], activation="tanh", dtype=dt, optimizer="adamw",
                              weight_decay=0.01), device=DEV)
    assert m.fused_optimizer and not m.net_kernel_eligible(B)
    w0 = [w * 4 for w in S.fan_in_normal(dims, seed=3)]
    for dst, src in zip(m.w, w0):
        dst.copy_(src.to(DEV, dt))
    pool = S.batch_pool(dims[-1], dims[0], B, count=2, seed=4)
    wq = [w.to(dt) for w in w0]
    states = [{} for _ in wq]
    for xb, yb in pool:
        m.train_step(xb.to(DEV, dt), yb.to(DEV, dt), T=4)
        x, wq, e = O.train_step_opt_storage(xb, yb, wq, states, act="tanh", gamma=0.5, T=4, sdt=dt, **opt)
    torch.cuda.synchronize()
    for l in range(len(wq)):
        assert O.rel_inf(m.w[l].cpu(), wq[l]) <= 1e-2, ("w", l)
        if states[l].get("m") is not None and states[l]["m"].abs().max() > 0:
            # the first moment is a (decayed) gradient: at B = 8 a sum of 8 products, where one-ulp
            # differences of the fp16 states (MUFU f in the state-update epilogue against the oracle's
            # tanhf) do not average out
            assert O.rel_inf(m._opt_state[l][0].cpu(), states[l]["m"]) <= (2e-2 if B >= 128 else 5e-2), ("m", l)
    sd = m.state_dict()
    assert sd["optimizer"]["steps"] == 2
    m2 = TileLangIPC(IPCConfig(dims=dims, alpha=opt["lr"], activation="tanh", dtype=dt, optimizer="adamw",
                               weight_decay=0.01), device=DEV)
    m2.load_state_dict(sd)
    assert m2._opt_steps == 2 and torch.equal(m2._opt_state[0][1], m._opt_state[0][1])
