"""GPU tests of the host-side API around the kernels: weight init, ``prepare_batch``, the
``BatchPipeline`` input ring, CUDA-graph blocks and the steady-state helpers.

* init: ``TileLangIPC(cfg, seed=s).w`` draws exactly ``oracle.init_weights`` on the same CUDA
  generator (the oracle's init is pinned to the reference's ``init_weights`` by a golden fixture);
* ``prepare_batch``: NCHW images -> ``[784, B]``, labels -> one-hot ``[C, B]`` (reference
  ``trainer.py:836-846``);
* ``BatchPipeline``: the overlapped copies give the same batches, and training on them gives
  bit-identical weights to synchronous ``prepare_batch`` + ``train_step``;
* graphs / steady state: a captured block and a single multi-step launch give bit-identical
  results to the same number of ``step_initialized`` calls.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _cfg(dims, dtype=torch.float16, **kw):
    from lich_b200.trainer import IPCConfig
    return IPCConfig(dims=tuple(dims), activation="tanh", dtype=dtype, **kw)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dims,grid_z", [((10, 64, 64, 784), 2), ((10,) + (64,) * 6 + (784,), 2),
                                         ((10,) + (64,) * 6 + (784,), 5), ((1000, 512, 512, 4096), 2)])
def test_weight_init_matches_reference_init(dims, grid_z, dtype):
    from lich_b200.trainer import TileLangIPC
    for seed in (0, 5):
        m = TileLangIPC(_cfg(dims, dtype, grid_z_max_layers=grid_z), device=DEV, seed=seed)
        ref = O.init_weights(dims, dtype=dtype, device=DEV, seed=seed)
        for l, (a, b) in enumerate(zip(m.w, ref)):
            assert a.shape == b.shape
            assert torch.equal(a, b), (dims, grid_z, seed, l)
        bound = [1.0 / dims[l + 1] ** 0.5 for l in range(len(dims) - 1)]
        assert all(w.float().abs().max().item() <= b * 1.001 for w, b in zip(m.w, bound))


def _mnist_like(B, count, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.rand((B, 1, 28, 28), generator=g), torch.randint(0, 10, (B,), generator=g)) for _ in range(count)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_prepare_batch_layout(dtype):
    from lich_b200.trainer import prepare_batch
    (img, lab), = _mnist_like(96, 1, 3)
    x, y = prepare_batch(img, lab, device=DEV, dtype=dtype, num_classes=10)
    assert x.shape == (784, 96) and y.shape == (10, 96)
    assert x.dtype == dtype and y.dtype == dtype and x.is_contiguous()
    assert torch.equal(x.cpu(), img.reshape(96, -1).T.to(dtype))
    assert torch.equal(y.cpu(), O.one_hot(lab, 10, dtype=dtype))
    with pytest.raises(ValueError):
        prepare_batch(img, lab[:10], device=DEV, dtype=dtype, num_classes=10)


@pytest.mark.parametrize("pinned", [False, True])
def test_batch_pipeline_yields_prepare_batch(pinned):
    from lich_b200.input_pipeline import BatchPipeline
    from lich_b200.trainer import prepare_batch
    data = _mnist_like(64, 7, 4)
    if pinned:
        data = [(a.pin_memory(), b.pin_memory()) for a, b in data]
    pipe = BatchPipeline(iter(data), device=DEV, dtype=torch.float16, num_classes=10, depth=3)
    got = [(x.clone(), y.clone()) for x, y in pipe]
    assert len(got) == len(data)
    for (x, y), (img, lab) in zip(got, data):
        xr, yr = prepare_batch(img, lab, device=DEV, dtype=torch.float16, num_classes=10)
        assert torch.equal(x, xr) and torch.equal(y, yr)
    assert pipe.h2d_bytes == sum(a.numel() * 4 + b.numel() * 8 for a, b in data)


def test_batch_pipeline_training_matches_synchronous_copies():
    """Overlapped H2D (copy stream, two slots) vs synchronous prepare_batch: identical weights."""
    from lich_b200 import synthetic as S
    from lich_b200.input_pipeline import BatchPipeline
    from lich_b200.trainer import TileLangIPC, prepare_batch
    dims = S.paper_dims(3)
    data = _mnist_like(128, 6, 5)
    res = []
    for overlapped in (False, True):
        m = TileLangIPC(_cfg(dims, alpha=1e-2), device=DEV, seed=1)
        if overlapped:
            for x, y in BatchPipeline(iter(data), device=DEV, dtype=torch.float16, num_classes=10):
                m.train_step(x, y, T=4)
        else:
            for img, lab in data:
                m.train_step(*prepare_batch(img, lab, device=DEV, dtype=torch.float16, num_classes=10), T=4)
        torch.cuda.synchronize()
        res.append([w.cpu() for w in m.w])
    for a, b in zip(*res):
        assert torch.equal(a, b)


def test_batch_pipeline_pools_feed_train_pool():
    """steps_per_slot = 4 over prepared pinned batches: each slot is a [4, d, B] pool for train_pool;
    the weights equal training on one device-resident pool of all batches."""
    from lich_b200 import synthetic as S
    from lich_b200.input_pipeline import BatchPipeline
    from lich_b200.trainer import TileLangIPC
    dims = S.paper_dims(6)
    x_h, y_h = S.stacked_pool(784, 10, 128, count=10, nets=1, seed=9, dtype=torch.float16)
    x_h, y_h = x_h[:, 0].contiguous().pin_memory(), y_h[:, 0].contiguous().pin_memory()
    res = []
    for piped in (False, True):
        m = TileLangIPC(_cfg(dims, alpha=1e-2), device=DEV, seed=2)
        if piped:
            pipe = BatchPipeline(((x_h[i], y_h[i]) for i in range(10)), device=DEV, dtype=torch.float16,
                                 num_classes=10, steps_per_slot=4)
            sizes = []
            for px, py in pipe:
                sizes.append(int(px.shape[0]))
                m.train_pool(px, py, steps=int(px.shape[0]), T=4)
            assert sizes == [4, 4, 2]
            # the same batches as pool chunks (one copy per tensor and slot), from pageable memory
            chunks = [(x_h[i:i + 3].clone(), y_h[i:i + 3].clone()) for i in (0, 3, 6)] + [(x_h[9:], y_h[9:])]
            m2 = TileLangIPC(_cfg(dims, alpha=1e-2), device=DEV, seed=2)
            for px, py in BatchPipeline(iter(chunks), device=DEV, dtype=torch.float16, num_classes=10,
                                        steps_per_slot=3):
                m2.train_pool(px, py, steps=int(px.shape[0]), T=4)
            torch.cuda.synchronize()
            assert all(torch.equal(a, b) for a, b in zip(m.w, m2.w))
        else:
            m.train_pool(x_h.to(DEV), y_h.to(DEV), steps=10, T=4)
        torch.cuda.synchronize()
        res.append([w.cpu() for w in m.w])
    for a, b in zip(*res):
        assert torch.equal(a, b)


@pytest.mark.parametrize("use_net", [True, False])
def test_graph_block_equals_step_calls(use_net):
    """A captured block of 3 steps replayed twice == 6 step_initialized calls (net path: one kernel node)."""
    from lich_b200 import synthetic as S
    from lich_b200.cuda_graph import IPCGraphRunner
    from lich_b200.trainer import TileLangIPC
    dims = S.paper_dims(4)
    xb, yb = S.batch_pool(784, 10, 128, count=1, seed=6)[0]
    res = []
    for graph in (False, True):
        m = TileLangIPC(_cfg(dims, alpha=1e-3, use_net_kernel=use_net), device=DEV, seed=3)
        m.initialize_batch(xb.to(DEV, torch.float16), yb.to(DEV, torch.float16))
        if graph:
            r = IPCGraphRunner(m, 3).capture()
            assert r.single_node == use_net
            assert m.steps_done == 0  # capturing trains nothing
            r.replay()
            r.replay()
            assert m.steps_done == 6
            r.release()
            with pytest.raises(RuntimeError):
                r.replay()
        else:
            for _ in range(6):
                m.step_initialized()
        torch.cuda.synchronize()
        res.append([t.cpu() for t in m.w + m.x + m.e[:-1]])
    for a, b in zip(*res):
        assert torch.equal(a, b)


def test_steady_state_single_launch_equals_step_calls():
    """run_prepared_steady_state without a graph runs steps x repeats in one persistent launch."""
    from lich_b200 import _native as N
    from lich_b200 import synthetic as S
    from lich_b200.trainer import TileLangIPC
    dims = S.paper_dims(6)
    xb, yb = S.batch_pool(784, 10, 128, count=1, seed=7)[0]
    res = []
    for one_launch in (False, True):
        m = TileLangIPC(_cfg(dims, alpha=1e-3), device=DEV, seed=4)
        m.prepare_steady_state(xb.to(DEV, torch.float16), yb.to(DEV, torch.float16), steps=5, use_graph=False)
        before = N.launch_count()
        if one_launch:
            m.run_prepared_steady_state(steps=5, repeats=2, use_graph=False)
            assert N.launch_count() - before == 1
        else:
            for _ in range(10):
                m.step_initialized()
        torch.cuda.synchronize()
        res.append([t.cpu() for t in m.w + m.x])
    for a, b in zip(*res):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dims,dtype", [((10, 64, 64, 784), torch.float16), ((10, 64, 64, 784), torch.float32),
                                        ((1000, 512, 512, 1024), torch.bfloat16)])
def test_evaluate_counts_argmax_on_device(dims, dtype):
    """evaluate = predict + argmax over classes (first on ties) + compare, counted on the device."""
    from lich_b200 import synthetic as S
    from lich_b200.trainer import TileLangIPC
    m = TileLangIPC(_cfg(dims, dtype), device=DEV, seed=11)
    B = 300
    (x, y), = S.batch_pool(dims[-1], dims[0], B, count=1, seed=12)
    labels = torch.randint(0, dims[0], (B,), generator=torch.Generator().manual_seed(13))
    xd = x.to(DEV, dtype)
    logits = m.predict(xd)
    ref = int((logits.float().argmax(dim=0).cpu() == labels).sum())
    labels[:50] = logits[:, :50].float().argmax(dim=0).cpu()  # some certain hits
    ref = int((logits.float().argmax(dim=0).cpu() == labels).sum())
    cnt = m.evaluate(xd, labels)
    assert int(cnt.item()) == ref >= 50
    m.evaluate(xd, labels.to(DEV), counter=cnt)  # accumulates
    assert int(cnt.item()) == 2 * ref
    assert m.accuracy(xd, labels) == ref / B
    # ties: the first maximal row wins, as torch.argmax
    from lich_b200 import _native as N
    tie = torch.zeros((4, 8), device=DEV, dtype=torch.float16)
    tie[1:3] = 1.0
    lab = torch.full((8,), 1, dtype=torch.int64, device=DEV)
    c = torch.zeros(1, dtype=torch.int32, device=DEV)
    N.check(N.load().ipc_count_correct(tie.data_ptr(), 4, 8, lab.data_ptr(), c.data_ptr(), N.dtype_code(torch.float16),
                                       N.stream_handle(DEV)))
    assert int(c.item()) == 8


@pytest.mark.parametrize("depth,B", [(3, 128), (6, 96), (4, 8)])
def test_predict_single_launch_matches_layer_chain(depth, B):
    """Hidden-64 networks predict in one persistent-kernel launch (forward sweep + a prediction-error pass
    against a zero target); the answer matches the per-layer forward operators (both storage-round each
    layer) and the fp32 oracle's forward chain, and the model's states are untouched."""
    from lich_b200 import _native as N
    from lich_b200 import synthetic as S
    from lich_b200.trainer import TileLangIPC
    dims = S.paper_dims(depth)
    m = TileLangIPC(_cfg(dims, torch.float16), device=DEV, seed=21)
    (x, y), = S.batch_pool(784, 10, B, count=1, seed=22)
    xd = x.to(DEV, torch.float16)
    m.train_step(xd, y.to(DEV, torch.float16), T=2)
    state = [t.clone() for t in m.x + m.e[:-1]]
    n0 = N.launch_count()
    fused = m.predict(xd)
    assert N.launch_count() - n0 == 1
    assert all(torch.equal(a, b) for a, b in zip(state, m.x + m.e[:-1]))
    m.cfg = type(m.cfg)(**{**m.cfg.__dict__, "use_net_kernel": False})
    chain = m.predict(xd)
    assert O.rel_inf(fused.cpu(), chain.cpu()) <= 1e-2
    h = x.to(torch.float16).float()
    for l in reversed(range(len(dims) - 1)):
        h = m.w[l].float().cpu() @ torch.tanh(h)
    assert O.rel_inf(fused.cpu(), h) <= 2e-2
