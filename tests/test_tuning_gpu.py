"""GPU tests: tuning-table rows, execution / grid.z policies and the sweep change what runs.

* a weight-update row with ``tc_splits = 1`` turns off the split-K pass the heuristic picks (one launch
  fewer), and the answer stays the oracle's;
* ``tc_bn`` / ``tc_raster`` overrides give the oracle's answer too;
* a grid.z policy file regroups the hidden layers of the operator path for that batch;
* an execution-policy kernel row is the config the trainer uses for that shape;
* ``sweep_gemm`` times every candidate, fills the SQLite cache and returns the fastest.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _ops(M, K, B, dt, seed):
    g = torch.Generator().manual_seed(seed)
    return ((torch.randn(M, K, generator=g) * 0.05).to(dt), (torch.randn(M, B, generator=g) * 0.5).to(dt),
            torch.randn(K, B, generator=g).to(dt))


def test_table_row_turns_off_split_k():
    from lich_b200 import _native as N
    from lich_b200.tilelang_kernels import KernelConfig, build_weight_update
    M, K, B, dt = 512, 512, 16384, torch.bfloat16
    w0, e, x = _ops(M, K, B, dt, 1)
    ref = O.weight_update_op(w0, e, x, act="tanh", alpha=1e-3, sdt=dt, recompute_activation=True)
    counts = {}
    for splits in (0, 1, 4):
        op = build_weight_update(M, K, B, "tanh", "bfloat16", KernelConfig(tc_splits=splits), 1e-3, True)
        w = w0.to(DEV)
        op(w.clone(), e.to(DEV), x.to(DEV))  # first call: workspace
        n0 = N.launch_count()
        op(w, e.to(DEV), x.to(DEV))
        counts[splits] = N.launch_count() - n0
        assert O.rel_inf(w.cpu(), ref) <= 1e-2, splits
    assert counts[0] == 3 and counts[4] == 3  # activation, split GEMM, reduce
    assert counts[1] == 2  # activation, GEMM


@pytest.mark.parametrize("bn,raster", [(128, 4), (256, 32), (128, 1)])
def test_tile_and_raster_overrides_keep_results(bn, raster):
    from lich_b200 import _native as N
    from lich_b200.tilelang_kernels import KernelConfig, build_prediction_error
    M, K, B, dt = 1024, 768, 2048, torch.float16
    g = torch.Generator().manual_seed(2)
    w = (torch.randn(M, K, generator=g) * K ** -0.5).to(dt)
    x_lo, x_up = torch.randn(M, B, generator=g).to(dt), torch.randn(K, B, generator=g).to(dt)
    e = torch.empty((M, B), device=DEV, dtype=dt)
    build_prediction_error(M, K, B, "tanh", "float16", KernelConfig(tc_bn=bn, tc_raster=raster))(
        x_up.to(DEV), w.to(DEV), x_lo.to(DEV), e)
    torch.cuda.synchronize()
    assert N.device_status() == 0
    assert O.rel_inf(e.cpu(), O.pred_err_op(x_up, w, x_lo, act="tanh", sdt=dt)) <= 1e-2


def test_trainer_uses_table_rows():
    """A TuningTable row for one layer's weight update reaches the trainer's operator path."""
    from lich_b200 import _native as N
    from lich_b200 import synthetic as S
    from lich_b200.tilelang_kernels import KernelConfig
    from lich_b200.trainer import IPCConfig, TileLangIPC
    from lich_b200.tuning import TuningEntry, TuningKey, TuningTable
    dims, B, dt = (104, 512, 512, 1024), 8192, torch.bfloat16
    w0 = S.fan_in_normal(dims, seed=5)
    (x, y), = S.batch_pool(dims[-1], dims[0], B, count=1, seed=6)
    res, launches = [], []
    for splits in (0, 1):
        rows = [TuningEntry(TuningKey("weight", dims[l], dims[l + 1], B, "tanh", "bfloat16"),
                            KernelConfig(backend="tcgen05", tc_splits=splits)) for l in range(3)]
        m = TileLangIPC(IPCConfig(dims=dims, alpha=1e-3, activation="tanh", dtype=dt,
                                  tuning_table=TuningTable.from_entries(rows)), device=DEV)
        assert m._kernel_config("weight", 512, 512, B).tc_splits == splits
        for dst, src in zip(m.w, w0):
            dst.copy_(src.to(DEV, dt))
        m.train_step(x.to(DEV, dt), y.to(DEV, dt), T=2)  # plan + workspaces
        for dst, src in zip(m.w, w0):
            dst.copy_(src.to(DEV, dt))
        n0 = N.launch_count()
        m.train_step(x.to(DEV, dt), y.to(DEV, dt), T=2)
        launches.append(N.launch_count() - n0)
        res.append([w.float().cpu() for w in m.w])
    assert launches[1] < launches[0]  # split-K reduce passes gone
    for a, b in zip(*res):
        assert O.rel_inf(a, b) <= 1e-2


def test_grid_z_policy_file_regroups(tmp_path):
    from lich_b200 import synthetic as S
    from lich_b200.trainer import IPCConfig, TileLangIPC
    from lich_b200.tuning import policy_key, write_grid_z_policy
    dims, B, dt = S.paper_dims(6), 96, torch.float16
    path = tmp_path / "gridz.json"
    write_grid_z_policy(path, {policy_key(device_name=torch.cuda.get_device_name(DEV),
                                          capability=torch.cuda.get_device_capability(DEV), dims=dims, batch=B,
                                          activation="tanh", dtype=dt): 5})
    w0 = S.fan_in_normal(dims, seed=8)
    (x, y), = S.batch_pool(784, 10, B, count=1, seed=9)
    outs = []
    for policy, cap in ((str(path), 2), (str(tmp_path / "none.json"), 5)):
        m = TileLangIPC(IPCConfig(dims=dims, activation="tanh", dtype=dt, use_net_kernel=False,
                                  grid_z_max_layers=cap, grid_z_policy_path=policy), device=DEV)
        for dst, src in zip(m.w, w0):
            dst.copy_(src.to(DEV, dt))
        m.train_step(x.to(DEV, dt), y.to(DEV, dt), T=4)
        assert m._grid_z_cap == 5 and len(m._layer_groups) == 1 and m._layer_groups[0].count == 5
        outs.append([w.cpu() for w in m.w])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_execution_policy_kernel_row(tmp_path):
    import json

    from lich_b200.trainer import IPCConfig, TileLangIPC
    path = tmp_path / "hier.json"
    path.write_text(json.dumps({"version": 1, "kernel_entries": [
        {"kind": "prediction", "shape": {"M": 512, "K": 1024, "B": 256}, "activation": "tanh",
         "dtype": "bfloat16", "config": {"backend": "simt"}}], "execution_entries": []}))
    m = TileLangIPC(IPCConfig(dims=(104, 512, 1024), activation="tanh", dtype=torch.bfloat16,
                              hierarchical_policy_path=str(path)), device=DEV)
    assert m._kernel_config("prediction", 512, 1024, 256).backend == "simt"
    assert m._kernel_config("prediction", 104, 512, 256).backend == "auto"


def test_sweep_fills_cache(tmp_path):
    from lich_b200 import tuning as T
    with T.MeasurementCache(tmp_path / "m.sqlite") as cache:
        e = T.sweep_gemm("prediction", 512, 512, 1024, dtype=torch.bfloat16, cache=cache, reps=2,
                         flush_bytes=1 << 20)
        assert e.median_ms > 0 and e.config.backend == "tcgen05"
        dev_fp, code_fp = T._fingerprints(DEV)
        prob = T.ProblemKey("prediction", 512, 512, 1024, "tanh", "bfloat16", dev_fp, code_fp)
        rows = list(cache.iter_problem(prob))
        assert len(rows) == len(T.gemm_candidates("prediction", 512, 512, 1024))
        assert all(m.status == "ok" for _, m in rows)
        again = T.sweep_gemm("prediction", 512, 512, 1024, dtype=torch.bfloat16, cache=cache, reps=2)
        assert again.config in T.gemm_candidates("prediction", 512, 512, 1024)
        assert len(list(cache.iter_problem(prob))) == len(rows)  # answered from the cache
