"""GPU edge cases of the newer paths: limits, empty requests, extreme aspect ratios.

* The wide small-batch step kernel at its largest width (4096: the whole thin operand of a unit
  staged in shared memory) and with a 10-row top layer, against the fp32 oracle (fp16, 1e-2).
* The persistent cluster kernel at its layer limit (IPC_NET_MAX_LAYERS = 8), against the oracle.
* The split-K weight delta with a 16 x 16 output and a 262144-column batch (the most splits).
* Empty requests through the newer entry points: zero-size operands launch nothing and change
  nothing; a zero-step ipc_net_train launches nothing.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _N():
    from lich_b200 import _native as N
    return N


def _one_step(dims, B, dtype, alpha=0.02, T=4, seed=0):
    from lich_b200 import synthetic as S
    from lich_b200.trainer import IPCConfig, TileLangIPC
    w0 = S.fan_in_normal(dims, seed=seed)
    (x, y), = S.batch_pool(dims[-1], dims[0], B, count=1, seed=seed + 1)
    m = TileLangIPC(IPCConfig(dims=tuple(dims), alpha=alpha, gamma=0.5, activation="tanh", dtype=dtype), device=DEV)
    for dst, src in zip(m.w, w0):
        dst.copy_(src.to(DEV, dtype))
    m.train_step(x.to(DEV, dtype), y.to(DEV, dtype), T=T)
    torch.cuda.synchronize()
    wq = [t.to(dtype).float() for t in w0]
    xr, wr, _, _ = O.train([(x.to(dtype).float(), y.to(dtype).float())], wq, act="tanh", alpha=alpha, gamma=0.5,
                           T=T, steps=1)
    return m, xr, wr


def test_wide_kernel_at_its_largest_width():
    N = _N()
    dims, B = (10, 4096, 256), 8
    plan = N.net_plan(dims, B, 1, 0)
    assert plan is not None and plan[0] == 0  # the wide small-batch kernel
    m, x, w = _one_step(dims, B, torch.float16)
    assert N.device_status() == 0
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)


def test_wide_kernel_refuses_wider_than_its_limit():
    N = _N()
    assert N.net_plan((10, 4104, 256), 8, 1, 0) is None


def test_cluster_kernel_at_the_layer_limit():
    N = _N()
    dims, B = (10,) + (64,) * 7 + (784,), 128
    assert len(dims) - 1 == N.NET_MAX_LAYERS
    plan = N.net_plan(dims, B, 1, 0)
    assert plan is not None and plan[0] > 0  # the cluster kernel
    m, x, w = _one_step(dims, B, torch.float16, alpha=1e-3)
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)


def test_split_k_with_a_very_long_batch():
    N = _N()
    M, K, B, dt = 16, 16, 262144, torch.bfloat16
    g = torch.Generator().manual_seed(5)
    e = (0.5 * torch.randn(M, B, generator=g)).to(dt)
    a = torch.randn(K, B, generator=g).to(dt)
    dw = torch.zeros(M, K, dtype=torch.float32, device=DEV)
    ws = torch.empty(N.SPLITK_WORKSPACE_BYTES // 4, dtype=torch.float32, device=DEV)
    n0 = N.launch_count()
    N.fused_gemm(N.MODE_WDELTA, e.to(DEV), a.to(DEV), dw, M=M, K=K, B=B, scale=1e-3, dtype=dt, workspace=ws)
    torch.cuda.synchronize()
    assert N.launch_count() - n0 == 2  # split GEMM + reduce
    ref = O.weight_delta_op(e, a, act="identity", alpha=1e-3, sdt=dt, recompute_activation=False)
    assert O.rel_inf(dw.cpu(), ref) <= 1e-3


def test_empty_requests_launch_nothing():
    N = _N()
    lib = N.load()
    dt = torch.float16
    w = torch.randn(8, 8, device=DEV).to(dt)
    w_before = w.clone()
    z = torch.zeros(8, 0, dtype=dt, device=DEV)
    ws = torch.empty(1024, dtype=torch.float32, device=DEV)
    n0 = N.launch_count()
    # B = 0: the weight update adds nothing
    N.fused_gemm(N.MODE_WEIGHT, z, z, w, M=8, K=8, B=0, scale=1.0, dtype=dt, workspace=ws)
    assert lib.ipc_weight_update_noalloc(N.MODE_WEIGHT, N.ptr(z), N.ptr(z), N.ptr(w), 8, 8, 0, 1, 1.0, 0,
                                         N.act_code("identity"), N.dtype_code(dt), 0, N.stream_handle(DEV)) == 0
    # M = 0: nothing to produce
    N.fused_gemm(N.MODE_PRED, w, z, z, z, M=0, K=8, B=0, dtype=dt)
    torch.cuda.synchronize()
    assert torch.equal(w, w_before)
    # a zero-step persistent launch
    from lich_b200.trainer import IPCConfig, TileLangIPC
    m = TileLangIPC(IPCConfig(dims=(10, 64, 64, 784), dtype=dt), device=DEV)
    px = torch.zeros((1, 784, 128), dtype=dt, device=DEV)
    py = torch.zeros((1, 10, 128), dtype=dt, device=DEV)
    m.train_pool(px, py, steps=0, T=4)
    torch.cuda.synchronize()
    assert N.launch_count() == n0
