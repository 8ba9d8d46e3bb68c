"""GPU tests of the wide small-batch step kernel (``ipc_net_train`` for B <= 16 and wide layers).

* configs[3] small-batch shape (dims (10, 1024 x 4, 784), T = 8) at B = 1, 4, 16, bf16 and fp16:
  one training step against the storage-rounded oracle (1e-2 on x and W) and the fp32 oracle
  (1e-2 in fp16; 2.5e-2 in bf16, where the storage-rounded oracle itself is 1.1-1.8e-2 from
  fp32 after 8 iterations).
* The same step through the operator path (``use_net_kernel=False``: small-batch P / I /
  forward kernels and the outer-product update) agrees within 1e-2.
* dW of the weight phase from random hidden states (O(1) errors) against the fp32 oracle, 2e-2.
* Several steps over a device pool, per-step energy against the oracle's energy metric.
* Shapes the cluster kernel does not take: B = 4 at hidden 64, odd widths (tails in every
  dimension), a one-layer network; with the weights resident in shared memory (each CTA's rows and
  columns, every shape above) and without (4096-wide rows; more units than CTAs).
* Failure detection: the barrier-timeout self-test makes one CTA's grid-barrier wait expire
  (a CTA that never arrives), the status reads IPC_ERR_TIMEOUT, and the context keeps working.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
C4A = (10, 1024, 1024, 1024, 1024, 784)


def _model(dims, dtype, alpha, use_net=True, act="tanh"):
    from lich_b200.trainer import IPCConfig, TileLangIPC
    cfg = IPCConfig(dims=tuple(dims), alpha=alpha, gamma=0.5, activation=act, dtype=dtype, use_net_kernel=use_net)
    return TileLangIPC(cfg, device=DEV, seed=0)


def _inputs(dims, B, seed, count=1):
    from lich_b200 import synthetic as S
    return S.fan_in_normal(dims, seed=seed), S.batch_pool(dims[-1], dims[0], B, count=count, seed=seed + 1)


def _q(w, pool, dtype):
    return ([t.to(dtype).float() for t in w], [(x.to(dtype).float(), y.to(dtype).float()) for x, y in pool])


def _step(m, w0, pool, dtype, T):
    for dst, src in zip(m.w, w0):
        dst.copy_(src.to(DEV, dtype))
    x, y = pool[0]
    m.train_step(x.to(DEV, dtype), y.to(DEV, dtype), T=T)
    torch.cuda.synchronize()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B", [1, 4, 16])
def test_c4a_step_matches_oracle(B, dtype):
    from lich_b200 import _native as N
    alpha, T = 0.05, 8
    w0, pool = _inputs(C4A, B, seed=10 + B)
    m = _model(C4A, dtype, alpha)
    assert m.net_kernel_eligible(B)
    _step(m, w0, pool, dtype, T)
    assert N.device_status() == 0
    wq, bq = _q(w0, pool, dtype)
    x, w, _, _ = O.train(bq, wq, act="tanh", alpha=alpha, gamma=0.5, T=T, steps=1)
    xs, ws, _ = O.train_storage(bq, wq, act="tanh", alpha=alpha, gamma=0.5, T=T, steps=1, sdt=dtype)
    # Against the fp32 oracle: 1e-2 in fp16.  In bf16 with T = 8 the reference kernels' own rounding
    # (the storage-rounded oracle) is already 1.1-1.8e-2 away from fp32 on x[2] and the hidden W, so
    # the bf16 bound there is 2.5e-2; against the storage-rounded oracle both dtypes meet 1e-2.
    gate32 = 1e-2 if dtype == torch.float16 else 2.5e-2
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= gate32, ("w", l)
        assert O.rel_inf(m.w[l].cpu(), ws[l]) <= 1e-2, ("w storage", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= gate32, ("x", l)
        assert O.rel_inf(m.x[l].cpu(), xs[l]) <= 1e-2, ("x storage", l)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B", [4, 16])
def test_c4a_step_agrees_with_operator_path(B, dtype):
    alpha, T = 0.05, 8
    w0, pool = _inputs(C4A, B, seed=30 + B)
    a = _model(C4A, dtype, alpha, use_net=True)
    b = _model(C4A, dtype, alpha, use_net=False)
    assert a.net_kernel_eligible(B) and not b.net_kernel_eligible(B)
    _step(a, w0, pool, dtype, T)
    _step(b, w0, pool, dtype, T)
    for l in range(len(C4A) - 1):
        assert O.rel_inf(a.w[l].cpu(), b.w[l].cpu()) <= 1e-2, ("w", l)
    for l in range(len(C4A)):
        assert O.rel_inf(a.x[l].cpu(), b.x[l].cpu()) <= 1e-2, ("x", l)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B", [4, 16])
def test_weight_update_from_random_states(B, dtype):
    """dW of the weight phase against the fp32 oracle's ipc_step.

    After a forward sweep the hidden errors are differences of nearly equal states, mostly storage
    rounding noise at width 1024 (two correct 16-bit implementations differ by tens of percent in
    e and so in dW), so dW is checked here from random hidden states, where e and dW are O(1):
    one ``step_initialized`` (P, I, W in one launch) against ``reference.py:42-59``."""
    from lich_b200 import synthetic as S
    alpha = 0.05  # dW ~ 0.1-0.25 of max|W|: the bf16 rounding of W moves it by < 0.5 %
    w0, pool = _inputs(C4A, B, seed=90 + B)
    m = _model(C4A, dtype, alpha)
    for dst, src in zip(m.w, w0):
        dst.copy_(src.to(DEV, dtype))
    x_in, y = pool[0]
    m.initialize_batch(x_in.to(DEV, dtype), y.to(DEV, dtype))
    g = torch.Generator().manual_seed(B)
    for l in range(1, len(C4A) - 1):
        m.x[l].copy_((0.5 * torch.randn(C4A[l], B, generator=g)).to(DEV, dtype))
    x0 = [t.cpu().float() for t in m.x]
    m.step_initialized()
    torch.cuda.synchronize()
    wq = [t.to(dtype).float() for t in w0]
    x, w, _, _ = O.ipc_step(x0, wq, act="tanh", alpha=alpha, gamma=0.5)
    for l in range(len(w)):
        dw_gpu = m.w[l].cpu().double() - wq[l].double()
        assert O.rel_inf(dw_gpu, w[l].double() - wq[l].double()) <= 2e-2, ("dW", l)
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)


def test_pool_steps_and_energy():
    dtype, alpha, T, B, steps = torch.float16, 1e-3, 4, 16, 3
    dims = (10, 512, 512, 784)
    w0, pool = _inputs(dims, B, seed=50, count=2)
    m = _model(dims, dtype, alpha)
    for dst, src in zip(m.w, w0):
        dst.copy_(src.to(DEV, dtype))
    px = torch.stack([p[0] for p in pool]).to(DEV, dtype).contiguous()
    py = torch.stack([p[1] for p in pool]).to(DEV, dtype).contiguous()
    energy = torch.zeros(steps, device=DEV, dtype=torch.float32)
    m.train_pool(px, py, steps=steps, T=T, energy=energy)
    torch.cuda.synchronize()
    wq, bq = _q(w0, pool, dtype)
    wr = [t.clone() for t in wq]
    energies = []
    for s in range(steps):
        x, wr, _, met = O.train(bq, wr, act="tanh", alpha=alpha, gamma=0.5, T=T, steps=1, first_batch=s)
        energies.append(met["energy"])
    for l in range(len(wr)):
        assert O.rel_inf(m.w[l].cpu(), wr[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)
    got = energy.cpu().double()
    ref = torch.tensor(energies, dtype=torch.float64)
    assert ((got - ref).abs() / ref.abs()).max().item() <= 2e-2


# the last two shapes: W rows of 4096 do not fit the resident copies (the kernel reads W from L2),
# and more 32-row units than CTAs (every CTA takes several units per phase)
@pytest.mark.parametrize("dims,B", [((10, 64, 64, 784), 4), ((7, 100, 33, 250), 5), ((12, 300), 16),
                                    ((10, 4096, 784), 4), ((10, 1024, 1024, 2048, 1024, 784), 4)])
def test_shapes_outside_the_cluster_kernel(dims, B):
    dtype, alpha, T = torch.float16, 0.02, 4
    w0, pool = _inputs(dims, B, seed=70 + B)
    m = _model(dims, dtype, alpha)
    assert m.net_kernel_eligible(B)
    _step(m, w0, pool, dtype, T)
    wq, bq = _q(w0, pool, dtype)
    x, w, _, _ = O.train(bq, wq, act="tanh", alpha=alpha, gamma=0.5, T=T, steps=1)
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)


def test_barrier_timeout_is_reported_and_context_survives():
    from lich_b200 import _native as N
    assert N.device_status() == 0
    sync = torch.zeros(N.NET_SYNC_BYTES // 4, device=DEV, dtype=torch.int32)
    N.check(N.load().ipc_selftest_barrier_timeout(sync.data_ptr(), 1000, N.stream_handle(DEV)))
    torch.cuda.synchronize()
    assert N.device_status(clear=True) == N.IPC_ERR_TIMEOUT
    assert N.device_status() == 0
    # the context is intact: a training step still runs and matches the oracle
    test_shapes_outside_the_cluster_kernel((10, 64, 64, 784), 4)
