"""Host-side tests of lich_b200.tuning: file formats, lookups, the measurement cache (no GPU).

Formats follow the reference: tuning tables ``src/ipc_tilelang/tuning.py:10-108``, grid.z policies
``gridz_tuning.py:16-73``, execution policies ``hierarchical_policy.py:55-238`` and the SQLite
``measurements`` table ``config.py:174-256``.
"""
import json

from lich_b200 import tuning as T
from lich_b200.tilelang_kernels import KernelConfig


def test_table_round_trip_keeps_tcgen05_knobs(tmp_path):
    cfg = KernelConfig(backend="tcgen05", tc_bn=256, tc_splits=4, tc_raster=8, tc_max_ctas=120)
    e = T.TuningEntry(T.TuningKey("weight", 4096, 4096, 8192, "tanh", "bfloat16"), cfg, 0.5)
    path = tmp_path / "t.json"
    T.TuningTable.from_entries([e]).to_json(path, device="NVIDIA B200", capability=(10, 0))
    payload = json.loads(path.read_text())
    assert payload["schema_version"] == 1 and payload["search_space"] == "sm100a-v1"
    back = T.TuningTable.from_json(path)
    got = back.lookup(kind="weight", M=4096, K=4096, B=8192, activation="tanh", dtype="bfloat16")
    assert got == cfg and got.tune().splits == 4 and got.tune().bn == 256
    assert back.lookup(kind="weight", M=4096, K=4096, B=8192, activation="relu", dtype="bfloat16") is None
    assert T.TuningTable.load(str(path)).entries == back.entries


def test_reference_format_table_loads_with_heuristic_knobs(tmp_path):
    """A table written by the reference (sm_86 TileLang configs) loads; its rows leave the tcgen05 knobs
    at the library's heuristics."""
    row = {"kind": "prediction", "shape": {"M": 64, "K": 64, "B": 128}, "activation": "relu", "dtype": "float16",
           "median_ms": 0.015, "spill_suspected": False,
           "config": {"block_m": 64, "block_n": 128, "block_k": 32, "threads": 128, "num_stages": 2,
                      "swizzle": True, "swizzle_panel": 8, "shared_swizzle": False}}
    path = tmp_path / "ref.json"
    path.write_text(json.dumps({"schema_version": 1, "device": "RTX 3060", "capability": [8, 6], "entries": [row]}))
    t = T.TuningTable.from_json(path)
    kc = t.lookup(kind="prediction", M=64, K=64, B=128, activation="relu", dtype="float16")
    assert kc is not None and kc.block_m == 64 and kc.backend == "auto" and kc.tune() is None


def test_merge_and_signature():
    a = T.TuningEntry(T.TuningKey("prediction", 1, 2, 3, "tanh", "bfloat16"), KernelConfig(tc_bn=128))
    b = T.TuningEntry(T.TuningKey("prediction", 1, 2, 3, "tanh", "bfloat16"), KernelConfig(tc_bn=256))
    c = T.TuningEntry(T.TuningKey("weight", 1, 2, 3, "tanh", "bfloat16"), KernelConfig())
    t1 = T.TuningTable.from_entries([a, c])
    t2 = t1.merged(T.TuningTable.from_entries([b]))
    assert t2.lookup(kind="prediction", M=1, K=2, B=3, activation="tanh", dtype="bfloat16").tc_bn == 256
    assert len(t2.entries) == 2
    assert t1.signature() != t2.signature()
    assert t1.signature() == T.TuningTable.from_entries([c, a]).signature()


def test_grid_z_policy(tmp_path):
    path = tmp_path / "gridz.json"
    key = T.policy_key(device_name="NVIDIA B200", capability=(10, 0), dims=(10, 64, 64, 64, 784), batch=96,
                       activation="tanh", dtype="torch.float16")
    T.write_grid_z_policy(path, {key: 3})
    q = dict(device_name="NVIDIA B200", capability=(10, 0), dims=(10, 64, 64, 64, 784), activation="tanh",
             dtype="float16")
    assert T.lookup_grid_z_cap(path, batch=96, default=2, **q) == 3
    assert T.lookup_grid_z_cap(path, batch=128, default=2, **q) == 2
    assert T.lookup_grid_z_cap(tmp_path / "missing.json", batch=96, default=5, **q) == 5


def test_execution_policy(tmp_path):
    path = tmp_path / "hier.json"
    path.write_text(json.dumps({
        "version": 1,
        "kernel_entries": [{"kind": "inference", "shape": {"M": 512, "K": 512, "B": 512}, "activation": "tanh",
                            "dtype": "bfloat16", "config": {"backend": "simt"}}],
        "execution_entries": [{"dims": [104, 512, 512, 1024], "batch": 512, "activation": "tanh",
                               "dtype": "bfloat16", "kernel_signature": "sm100a-v1",
                               "best": {"grid_z_max_layers": 0, "use_cuda_graph": True}},
                              {"dims": [104, 512, 512, 1024], "batch": 512, "activation": "tanh",
                               "dtype": "bfloat16", "kernel_signature": "someone-elses-table",
                               "best": {"grid_z_max_layers": 7}}]}))
    p = T.ExecutionPolicy(path)
    assert p.exists
    assert p.lookup_kernel(kind="inference", M=512, K=512, B=512, activation="tanh", dtype="bfloat16").backend == "simt"
    key = dict(dims=(104, 512, 512, 1024), batch=512, activation="tanh", dtype="torch.bfloat16")
    assert p.lookup_execution(**key)["best"]["grid_z_max_layers"] == 0
    assert p.selected("use_cuda_graph", False, **key) is True
    assert p.selected("use_cuda_graph", False, **{**key, "batch": 64}) is False
    assert not T.ExecutionPolicy(tmp_path / "none.json").exists


def test_measurement_cache(tmp_path):
    db = tmp_path / "m.sqlite"
    prob = T.ProblemKey("weight", 1024, 1024, 65536, "tanh", "bfloat16", "NVIDIA B200|sm_100|148SM", "abc")
    cfg = KernelConfig(backend="tcgen05", tc_splits=4)
    with T.MeasurementCache(db) as c:
        assert c.get(prob, cfg) is None
        c.put(prob, cfg, T.Measurement("ok", 0.1, True, 5))
        c.put(prob, cfg, T.Measurement("ok", 0.09, True, 5))  # updated in place
        c.put(prob, KernelConfig(backend="tcgen05", tc_splits=8), T.Measurement("error", error_message="x"))
    with T.MeasurementCache(db) as c:
        assert c.get(prob, cfg).latency_ms == 0.09
        rows = list(c.iter_problem(prob))
        assert len(rows) == 2 and {m.status for _, m in rows} == {"ok", "error"}
        other = T.ProblemKey("weight", 1024, 1024, 65536, "tanh", "bfloat16", "RTX 3060|sm_86", "abc",
                             search_space_version="sm86-v2")
        assert c.get(other, cfg) is None
    cols = [r[1] for r in __import__("sqlite3").connect(str(db)).execute("PRAGMA table_info(measurements)")]
    assert cols == ["cache_key", "problem_digest", "problem_json", "config_json", "measurement_json", "updated_at"]


def test_sweep_candidates():
    w = T.gemm_candidates("weight", 1024, 1024, 65536)
    p = T.gemm_candidates("prediction", 4096, 4096, 8192)
    assert len(w) == 1 + 2 * 4 * 6 + 4 and len(p) == 1 + 2 * 4 + 4
    assert all(c.backend == "tcgen05" for c in w + p)
    assert len({c for c in w}) == len(w)


def test_packaged_table_is_sm100a():
    t = T.default_table()
    if t is None:
        return
    assert t.search_space == "sm100a-v1"
    assert all(e.key.kind in T.KINDS for e in t.entries)
    assert all(e.config.tc_bn in (0, 128, 256) for e in t.entries)
