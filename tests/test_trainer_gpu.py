"""GPU parity of whole training steps (trainer, persistent net kernel) against the oracle.

Gates (north star): fp32 path ``max|got-ref|/max|ref| <= 1e-5`` on every x[l]
and W[l]; fp16 / bf16 storage ``<= 1e-2`` on x and W after T inference
iterations plus one weight update.  The oracle runs in fp32 on the
storage-rounded inputs and weights.
"""
import pytest
import torch

from oracle import ipc_oracle as O
from tests.golden_io import load

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _model(dims, act, dtype, *, alpha=1e-4, gamma=0.5, use_net=True, grid_z=2, recompute=True, cluster=0):
    from lich_b200.trainer import IPCConfig, TileLangIPC
    cfg = IPCConfig(dims=tuple(dims), alpha=alpha, gamma=gamma, activation=act, dtype=dtype,
                    use_grid_z=grid_z >= 2, grid_z_max_layers=grid_z, recompute_activation=recompute,
                    use_net_kernel=use_net, net_cluster=cluster)
    return TileLangIPC(cfg, device=DEV, seed=0)


def _set_w(model, w):
    for dst, src in zip(model.w, w):
        dst.copy_(src.to(DEV, model.cfg.dtype))


def _oracle_inputs(w, batches, dtype):
    """Round W and the batches through the storage dtype, return fp32 CPU copies."""
    wq = [t.to(dtype).float() for t in w]
    bq = [(x.to(dtype).float(), y.to(dtype).float()) for x, y in batches]
    return wq, bq


def test_golden_c1_dims_fp32_operator_path_matches_reference():
    """configs[0] dims, fp32: the GPU path reproduces the reference's own golden outputs."""
    meta, w_in, batches, w_out, x_out = load("c1_dims_b8")
    m = _model(meta["dims"], meta["activation"], torch.float32, alpha=meta["alpha"], gamma=meta["gamma"])
    assert not m.net_kernel_eligible(meta["B"])
    _set_w(m, w_in)
    for s in range(meta["steps"]):
        xb, yb = batches[s % len(batches)]
        m.train_step(xb.to(DEV), yb.to(DEV), T=meta["T"])
    for l in range(len(w_in)):
        assert O.rel_inf(m.w[l].cpu(), w_out[l]) <= 1e-5, l
    for l in range(len(x_out)):
        assert O.rel_inf(m.x[l].cpu(), x_out[l]) <= 1e-5, l


@pytest.mark.parametrize("name", ["small_relu", "small_tanh", "small_sigmoid", "small_silu", "small_gelu"])
def test_golden_small_fp32_matches_reference(name):
    meta, w_in, batches, w_out, x_out = load(name)
    m = _model(meta["dims"], meta["activation"], torch.float32, alpha=meta["alpha"], gamma=meta["gamma"])
    _set_w(m, w_in)
    for s in range(meta["steps"]):
        xb, yb = batches[s % len(batches)]
        m.train_step(xb.to(DEV), yb.to(DEV), T=meta["T"])
    for l in range(len(w_in)):
        assert O.rel_inf(m.w[l].cpu(), w_out[l]) <= 1e-5, l
    for l in range(len(x_out)):
        assert O.rel_inf(m.x[l].cpu(), x_out[l]) <= 1e-5, l


def test_c1_full_fp32_10_steps():
    """(10,64,64,784), tanh, B=128, T=4, 10 training steps, fp32, 1e-5."""
    from lich_b200 import synthetic as S
    dims = (10, 64, 64, 784)
    w0 = S.fan_in_normal(dims, seed=1)
    pool = S.batch_pool(784, 10, 128, count=10, seed=2)
    m = _model(dims, "tanh", torch.float32)
    _set_w(m, w0)
    for s in range(10):
        m.train_step(pool[s][0].to(DEV), pool[s][1].to(DEV), T=4)
    x, w, e, _ = O.train(pool, w0, act="tanh", alpha=1e-4, gamma=0.5, T=4, steps=10)
    for l in range(3):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-5, l
    for l in range(4):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-5, l


def _err_scaled(got, ref, scale):
    """max|got - ref| / max|scale|: errors e = x - W f(x) are judged against the state they came from
    (right after a forward sweep e is pure rounding noise, so max|e| is no yardstick)."""
    return (got.cpu().double() - ref.double()).abs().max().item() / scale.double().abs().max().item()


def _pool_run(depth, act, dtype, steps, alpha=1e-4, seed=0):
    from lich_b200 import synthetic as S
    dims = S.paper_dims(depth)
    w0 = S.fan_in_normal(dims, seed=10 + depth + seed)
    pool = S.batch_pool(784, 10, 128, count=2, seed=20 + depth + seed)
    m = _model(dims, act, dtype, alpha=alpha)
    assert m.net_kernel_eligible(128)
    _set_w(m, w0)
    px = torch.stack([p[0] for p in pool]).to(DEV, dtype).contiguous()
    py = torch.stack([p[1] for p in pool]).to(DEV, dtype).contiguous()
    m.train_pool(px, py, steps=steps, T=4)
    wq, bq = _oracle_inputs(w0, pool, dtype)
    x, w, e, _ = O.train(bq, wq, act=act, alpha=alpha, gamma=0.5, T=4, steps=steps)
    return m, x, w, e


@pytest.mark.parametrize("depth", [3, 4, 6])
@pytest.mark.parametrize("act", ["relu"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_net_kernel_relu_against_storage_oracle(depth, act, dtype):
    """relu' is discontinuous at 0, so an fp16 state one ulp off the fp32 oracle can flip it and move
    that element by gamma*|W^T e|.  The gate for relu is the oracle with the reference kernels' own
    storage rounding (oracle.train_step_storage): W within 1e-2; x and e within 1e-2 on at least 99%
    of elements (the reference's probe criterion, scripts/autotune.py:250-260), 5e-2 everywhere."""
    from lich_b200 import synthetic as S
    dims = S.paper_dims(depth)
    w0 = S.fan_in_normal(dims, seed=10 + depth)
    pool = S.batch_pool(784, 10, 128, count=1, seed=20 + depth)
    m = _model(dims, act, dtype)
    _set_w(m, w0)
    m.train_pool(pool[0][0][None].to(DEV, dtype).contiguous(), pool[0][1][None].to(DEV, dtype).contiguous(),
                 steps=1, T=4)
    x, w, e = O.train_storage(pool, w0, act=act, alpha=1e-4, gamma=0.5, T=4, steps=1, sdt=dtype)
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(1, len(x) - 1):
        d = (m.x[l].cpu().double() - x[l].double()).abs() / x[l].double().abs().max()
        assert (d > 1e-2).double().mean().item() <= 0.01, ("x", l)
        assert d.max().item() <= 5e-2, ("x", l)


@pytest.mark.parametrize("depth", [3, 4, 6])
@pytest.mark.parametrize("act", ["tanh", "sigmoid", "gelu"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_net_kernel_one_training_step_gate(depth, act, dtype):
    """The 16-bit parity gate: configs[1] shape (hidden 64, B=128), T=4 inference iterations + 1 weight
    update through the persistent kernel; x and W within 1e-2 of the fp32 oracle."""
    m, x, w, e = _pool_run(depth, act, dtype, steps=1)
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)
    for l in range(len(w)):
        assert _err_scaled(m.e[l], e[l], x[l]) <= 1e-2, ("e", l)


@pytest.mark.parametrize("depth", [3, 6])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_net_kernel_ten_step_trajectory(depth, dtype):
    """10 training steps inside one launch (weights carried on chip, batch prefetch between steps).
    16-bit rounding compounds over steps, so the bound is 2e-2 (fp16) / 5e-2 (bf16)."""
    m, x, w, e = _pool_run(depth, "tanh", dtype, steps=10, alpha=1e-3)
    tol = 2e-2 if dtype == torch.float16 else 5e-2
    for l in range(len(w)):
        assert torch.isfinite(m.w[l].float()).all()
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= tol, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= tol, ("x", l)


@pytest.mark.parametrize("B", [8, 24, 64, 128, 256])
def test_net_kernel_batch_sizes_and_large_alpha_delta(B):
    """Cluster sizes 1..8 (8/16 columns per CTA); alpha large enough that dW is far above fp16 ulp.
    B = 256 does not fit the persistent kernel's shared memory: the trainer runs the operator path."""
    from lich_b200 import synthetic as S
    dims = (10, 64, 64, 64, 784)
    dtype = torch.float16
    w0 = S.fan_in_normal(dims, seed=B)
    pool = S.batch_pool(784, 10, B, count=1, seed=B + 1)
    alpha = 0.02
    m = _model(dims, "tanh", dtype, alpha=alpha)
    assert m.net_kernel_eligible(B) == (B != 256)
    _set_w(m, w0)
    px = pool[0][0][None].to(DEV, dtype).contiguous()
    py = pool[0][1][None].to(DEV, dtype).contiguous()
    m.train_pool(px, py, steps=1, T=4)
    wq, bq = _oracle_inputs(w0, pool, dtype)
    x, w, e, _ = O.train(bq, wq, act="tanh", alpha=alpha, gamma=0.5, T=4, steps=1)
    for l in range(len(w)):
        dw_gpu = m.w[l].cpu().double() - wq[l].double()
        dw_ref = w[l].double() - wq[l].double()
        assert O.rel_inf(dw_gpu, dw_ref) <= 3e-2, ("dW", l)
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)


def test_net_path_equals_operator_path_step_initialized():
    """Reference step semantics (P, I, W every call): one net-kernel launch vs 3L-1 operator launches."""
    from lich_b200 import synthetic as S
    dims = S.paper_dims(6)
    w0 = S.fan_in_normal(dims, seed=3)
    xb, yb = S.batch_pool(784, 10, 128, count=1, seed=4)[0]
    outs = []
    for use_net in (True, False):
        m = _model(dims, "tanh", torch.float16, alpha=1e-3, use_net=use_net)
        assert m.net_kernel_eligible(128) == use_net
        _set_w(m, w0)
        m.initialize_batch(xb.to(DEV, torch.float16), yb.to(DEV, torch.float16))
        for _ in range(3):
            m.step_initialized()
        outs.append(([w.cpu() for w in m.w], [x.cpu() for x in m.x], [e.cpu() for e in m.e[:-1]]))
    (wn, xn, en), (wo, xo, eo) = outs
    for a, b in zip(wn + xn, wo + xo):
        assert O.rel_inf(a, b) <= 1e-2
    for l, (a, b) in enumerate(zip(en, eo)):
        assert _err_scaled(a, b, xo[l]) <= 1e-2


def test_step_initialized_matches_reference_ipc_step():
    """One reference iPC step (P, I, W) from the same state, fp16 storage (persistent kernel)."""
    from lich_b200 import synthetic as S
    dims = (10, 64, 64, 64, 784)
    w0 = S.fan_in_normal(dims, seed=5)
    xb, yb = S.batch_pool(784, 10, 128, count=1, seed=6)[0]
    m = _model(dims, "sigmoid", torch.float16, alpha=0.01)
    _set_w(m, w0)
    m.initialize_batch(xb.to(DEV, torch.float16), yb.to(DEV, torch.float16))
    x_init = [x.cpu().float() for x in m.x]
    wq = [w.cpu().float() for w in m.w]
    m.step_initialized()
    x_ref, w_ref, e_ref, _ = O.ipc_step(x_init, wq, act="sigmoid", alpha=0.01, gamma=0.5)
    for l in range(len(wq)):
        assert O.rel_inf(m.w[l].cpu(), w_ref[l]) <= 1e-2
        assert _err_scaled(m.e[l], e_ref[l], x_init[l]) <= 1e-2
    for l in range(len(x_ref)):
        assert O.rel_inf(m.x[l].cpu(), x_ref[l]) <= 1e-2


def test_cuda_graph_replay_equals_direct():
    from lich_b200 import synthetic as S
    dims = S.paper_dims(4)
    w0 = S.fan_in_normal(dims, seed=8)
    xb, yb = S.batch_pool(784, 10, 128, count=1, seed=9)[0]
    res = []
    for use_graph in (False, True):
        m = _model(dims, "tanh", torch.float16, alpha=1e-3)
        _set_w(m, w0)
        m.prepare_steady_state(xb.to(DEV, torch.float16), yb.to(DEV, torch.float16), steps=4, use_graph=use_graph)
        m.run_prepared_steady_state(steps=4, repeats=2, use_graph=use_graph)
        res.append([t.cpu() for t in m.w + m.x])
    for a, b in zip(*res):
        assert torch.isfinite(a.float()).all()
        assert torch.equal(a, b)


def test_operator_path_grid_z_and_save_activation():
    """Grouped (grid.z) layers and save-A mode on the operator path, fp16, vs the oracle."""
    from lich_b200 import synthetic as S
    dims = S.paper_dims(6)
    w0 = S.fan_in_normal(dims, seed=12)
    pool = S.batch_pool(784, 10, 96, count=1, seed=13)
    for recompute in (True, False):
        m = _model(dims, "tanh", torch.float16, use_net=False, grid_z=2, recompute=recompute)
        assert len(m._layer_groups) == 2
        _set_w(m, w0)
        m.train_step(pool[0][0].to(DEV, torch.float16), pool[0][1].to(DEV, torch.float16), T=4)
        wq, bq = _oracle_inputs(w0, pool, torch.float16)
        x, w, e, _ = O.train(bq, wq, act="tanh", alpha=1e-4, gamma=0.5, T=4, steps=1)
        for l in range(len(w)):
            assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2
        for l in range(len(x)):
            assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2


def test_predict_and_state_dict():
    from lich_b200 import synthetic as S
    dims = S.paper_dims(3)
    w0 = S.fan_in_normal(dims, seed=14)
    xb, _ = S.batch_pool(784, 10, 32, count=1, seed=15)[0]
    m = _model(dims, "tanh", torch.float32)
    _set_w(m, w0)
    out = m.predict(xb.to(DEV))
    h = xb
    for l in reversed(range(len(w0))):
        h = w0[l] @ torch.tanh(h)
    assert O.rel_inf(out.cpu(), h) <= 1e-5
    sd = m.state_dict()
    m2 = _model(dims, "tanh", torch.float32)
    m2.load_state_dict(sd)
    assert all(torch.equal(a, b) for a, b in zip(m.w, m2.w))


def test_metrics_and_errors():
    from lich_b200 import synthetic as S
    dims = S.paper_dims(3)
    m = _model(dims, "tanh", torch.float16)
    with pytest.raises(RuntimeError):
        m.step_initialized()
    xb, yb = S.batch_pool(784, 10, 128, count=1, seed=1)[0]
    with pytest.raises(ValueError):
        m.initialize_batch(xb[:100].to(DEV, torch.float16), yb.to(DEV, torch.float16))
    r = m.step(xb.to(DEV, torch.float16), yb.to(DEV, torch.float16))
    assert r["max_abs_error"] > 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_wide_operator_path_tensor_cores(dtype):
    """A miniature of the wide configuration (hidden 512, B = 512): the operator path with the
    activation cache, whose GEMMs run on the tcgen05 kernel; one training step vs the fp32 oracle."""
    from lich_b200 import synthetic as S
    dims = (104, 512, 512, 512, 1024)
    w0 = S.fan_in_normal(dims, seed=31)
    pool = S.batch_pool(1024, 104, 512, count=1, seed=32)
    m = _model(dims, "tanh", dtype, alpha=1e-3)
    assert not m.net_kernel_eligible(512)
    _set_w(m, w0)
    m.train_step(pool[0][0].to(DEV, dtype), pool[0][1].to(DEV, dtype), T=4)
    from lich_b200 import _native as N
    assert N.device_status() == 0
    wq, bq = _oracle_inputs(w0, pool, dtype)
    x, w, e, _ = O.train(bq, wq, act="tanh", alpha=1e-3, gamma=0.5, T=4, steps=1)
    for l in range(len(w)):
        assert O.rel_inf(m.w[l].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l].cpu(), x[l]) <= 1e-2, ("x", l)
