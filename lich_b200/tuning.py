"""Tuning tables, execution policies and the measurement cache, rebuilt for sm_100a.

File formats follow the reference so its tables and policies load here:

* ``TuningTable`` -- per-shape ``KernelConfig`` rows keyed by ``(kind, M, K,
  B, activation, dtype)``, JSON ``schema_version`` 1
  (``src/ipc_tilelang/tuning.py:10-108``).  Tables written here add
  ``"search_space": "sm100a-v1"``; their configs set ``backend`` and the
  tcgen05 launch knobs ``tc_bn`` / ``tc_splits`` / ``tc_raster`` /
  ``tc_max_ctas`` (``ipc_gemm_tune_t``).  Rows of tables measured on other
  GPUs load with those knobs at 0 (the library's heuristics).
* grid.z policy -- ``{"version": 1, "entries": {key: {"grid_z_max_layers":
  n}}}`` with the key a canonical JSON of device name, capability, dims,
  batch, activation and dtype (``src/ipc_tilelang/gridz_tuning.py:16-73``).
* execution policy -- ``hierarchical_policy.json`` with ``kernel_entries``
  (rows like a tuning table's) and ``execution_entries`` whose ``best`` dict
  holds ``grid_z_max_layers`` / ``use_cuda_graph``
  (``src/ipc_tilelang/hierarchical_policy.py:55-238``).  An execution row
  applies when its ``kernel_signature`` is this build's search space or the
  signature of the tuning table in use.
* ``MeasurementCache`` -- a SQLite ``measurements`` table with the
  reference's columns (``src/ipc_tilelang/config.py:174-256``): one row per
  (problem, config), the problem keyed with ``search_space_version``
  ``"sm100a-v1"`` so sm_86 observations never answer for this hardware.

``sweep_gemm`` is the exhaustive search that fills them: every candidate
launch configuration of the tcgen05 kernel for one operator shape, timed with
CUDA events after an L2 flush, each result stored in the cache, the fastest
returned as a ``TuningEntry``.  ``default_table()`` is the table measured on
B200 and shipped with the package (``tables/b200_sm100a.json``).
"""
from __future__ import annotations

import hashlib
import json
import sqlite3
import statistics
import threading
import time
from dataclasses import asdict, dataclass, field, fields
from functools import lru_cache
from pathlib import Path
from typing import Any, Iterable

from .tilelang_kernels import KernelConfig

SCHEMA_VERSION = 1
SEARCH_SPACE = "sm100a-v1"
CACHE_SCHEMA_VERSION = 3
PACKAGED_TABLE = Path(__file__).resolve().parent / "tables" / "b200_sm100a.json"
KINDS = ("prediction", "inference", "weight", "forward")


def _dtype_name(dtype: Any) -> str:
    return str(dtype).split(".")[-1]


def _dims_key(dims) -> str:
    return "x".join(str(int(d)) for d in dims)


def _config_from(row_cfg: dict) -> KernelConfig:
    known = {f.name for f in fields(KernelConfig)}
    return KernelConfig(**{k: v for k, v in row_cfg.items() if k in known})


# ------------------------------------------------------------------ tuning table
@dataclass(frozen=True)
class TuningKey:
    kind: str
    M: int
    K: int
    B: int
    activation: str
    dtype: str


@dataclass(frozen=True)
class TuningEntry:
    key: TuningKey
    config: KernelConfig
    median_ms: float | None = None
    spill_suspected: bool | None = None


@dataclass(frozen=True)
class TuningTable:
    entries: tuple[TuningEntry, ...]
    search_space: str | None = None

    @classmethod
    def from_entries(cls, entries: Iterable[TuningEntry], search_space: str | None = SEARCH_SPACE) -> "TuningTable":
        return cls(tuple(entries), search_space)

    @classmethod
    def from_json(cls, path: str | Path) -> "TuningTable":
        payload = json.loads(Path(path).read_text(encoding="utf-8"))
        if payload.get("schema_version") != SCHEMA_VERSION:
            raise ValueError(f"Unsupported tuning schema: {payload.get('schema_version')!r}; expected {SCHEMA_VERSION}")
        out = []
        for row in payload.get("entries", []):
            shape = row["shape"]
            key = TuningKey(str(row["kind"]), int(shape["M"]), int(shape["K"]), int(shape["B"]),
                            str(row.get("activation", "relu")), str(row.get("dtype", "float16")))
            med = row.get("median_ms")
            out.append(TuningEntry(key, _config_from(row["config"]), None if med is None else float(med),
                                   row.get("spill_suspected")))
        return cls(tuple(out), payload.get("search_space"))

    @classmethod
    def load(cls, source) -> "TuningTable | None":
        """A table, a path to one, or None."""
        if source is None or isinstance(source, TuningTable):
            return source
        return cls.from_json(source)

    def _index(self) -> dict:
        idx = self.__dict__.get("_idx")
        if idx is None:
            idx = {e.key: e.config for e in self.entries}
            object.__setattr__(self, "_idx", idx)
        return idx

    def lookup(self, *, kind: str, M: int, K: int, B: int, activation: str, dtype) -> KernelConfig | None:
        return self._index().get(TuningKey(kind, int(M), int(K), int(B), str(activation), _dtype_name(dtype)))

    def merged(self, other: "TuningTable") -> "TuningTable":
        """This table with ``other``'s rows added (``other`` wins on equal keys)."""
        rows = {e.key: e for e in self.entries}
        rows.update({e.key: e for e in other.entries})
        return TuningTable(tuple(rows.values()), self.search_space or other.search_space)

    def signature(self) -> str:
        """Stable fingerprint of the rows (an execution policy names the kernel table it was measured with)."""
        rows = sorted(json.dumps([asdict(e.key), asdict(e.config)], sort_keys=True, separators=(",", ":"))
                      for e in self.entries)
        raw = "\n".join(rows)
        return hashlib.sha256(raw.encode("utf-8")).hexdigest()[:20]

    def to_json(self, path: str | Path, *, device: str | None = None,
                capability: tuple[int, int] | None = None) -> None:
        rows = [{"kind": e.key.kind, "shape": {"M": e.key.M, "K": e.key.K, "B": e.key.B},
                 "activation": e.key.activation, "dtype": e.key.dtype, "median_ms": e.median_ms,
                 "spill_suspected": e.spill_suspected, "config": asdict(e.config)} for e in self.entries]
        payload = {"schema_version": SCHEMA_VERSION, "search_space": self.search_space or SEARCH_SPACE,
                   "device": device, "capability": list(capability) if capability is not None else None,
                   "entries": rows}
        out = Path(path)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps(payload, indent=1), encoding="utf-8")


@lru_cache(maxsize=1)
def default_table() -> TuningTable | None:
    """The table measured on B200 that ships with the package (None if it is absent)."""
    return TuningTable.from_json(PACKAGED_TABLE) if PACKAGED_TABLE.exists() else None


# --------------------------------------------------------------- grid.z policy
def policy_key(*, device_name: str, capability, dims, batch: int, activation: str, dtype) -> str:
    return json.dumps({"device": device_name, "capability": list(capability), "dims": _dims_key(dims),
                       "batch": int(batch), "activation": activation, "dtype": _dtype_name(dtype)},
                      sort_keys=True, separators=(",", ":"))


def load_grid_z_policy(path: str | Path) -> dict:
    p = Path(path)
    if not p.exists():
        return {"version": 1, "entries": {}}
    obj = json.loads(p.read_text(encoding="utf-8"))
    if not isinstance(obj, dict) or not isinstance(obj.get("entries", {}), dict):
        raise ValueError(f"Invalid grid.z policy file: {p}")
    return obj


def lookup_grid_z_cap(path: str | Path, *, device_name: str, capability, dims, batch: int, activation: str, dtype,
                      default: int = 2) -> int:
    """grid.z layer cap recorded for this device / network / batch, or ``default``."""
    row = load_grid_z_policy(path)["entries"].get(policy_key(device_name=device_name, capability=capability,
                                                             dims=dims, batch=batch, activation=activation,
                                                             dtype=dtype))
    return int(row.get("grid_z_max_layers", default)) if isinstance(row, dict) else int(default)


def write_grid_z_policy(path: str | Path, entries: dict[str, int]) -> None:
    """``entries``: policy_key -> cap; merged into the file at ``path``."""
    obj = load_grid_z_policy(path)
    for k, cap in entries.items():
        obj["entries"][k] = {"grid_z_max_layers": int(cap)}
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_text(json.dumps(obj, indent=1, sort_keys=True), encoding="utf-8")


# ------------------------------------------------------------ execution policy
class ExecutionPolicy:
    """Reader of an execution policy (``hierarchical_policy.json``): kernel rows and per-network choices."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        data = json.loads(self.path.read_text(encoding="utf-8")) if self.path.exists() else {}
        if not isinstance(data, dict):
            raise ValueError(f"Invalid execution policy: {self.path}")
        self.data = data
        self._kernels: dict[TuningKey, KernelConfig] = {}
        for row in data.get("kernel_entries", []):
            try:
                shape = row["shape"]
                key = TuningKey(str(row["kind"]), int(shape["M"]), int(shape["K"]), int(shape["B"]),
                                str(row.get("activation", "relu")), str(row.get("dtype", "float16")))
                self._kernels[key] = _config_from(dict(row["config"]))
            except (KeyError, TypeError, ValueError):
                continue
        self._execution: dict[tuple, dict] = {}
        for row in data.get("execution_entries", []):
            try:
                key = (_dims_key(row["dims"]), int(row["batch"]), str(row.get("activation", "relu")),
                       str(row.get("dtype", "float16")), str(row.get("kernel_signature", "")))
                self._execution[key] = row
            except (KeyError, TypeError, ValueError):
                continue

    @property
    def exists(self) -> bool:
        return self.path.exists()

    def lookup_kernel(self, *, kind: str, M: int, K: int, B: int, activation: str, dtype) -> KernelConfig | None:
        return self._kernels.get(TuningKey(kind, int(M), int(K), int(B), str(activation), _dtype_name(dtype)))

    def lookup_execution(self, *, dims, batch: int, activation: str, dtype,
                         signatures: Iterable[str] = (SEARCH_SPACE,)) -> dict | None:
        for sig in signatures:
            row = self._execution.get((_dims_key(dims), int(batch), str(activation), _dtype_name(dtype), str(sig)))
            if row is not None:
                return row
        return None

    def selected(self, name: str, default, **key):
        row = self.lookup_execution(**key)
        best = (row or {}).get("best") or {}
        return type(default)(best.get(name, default)) if best.get(name) is not None else default


# ---------------------------------------------------------- measurement cache
@dataclass(frozen=True)
class ProblemKey:
    kind: str
    M: int
    K: int
    B: int
    activation: str
    dtype: str
    device_fingerprint: str
    code_fingerprint: str
    search_space_version: str = SEARCH_SPACE

    def payload(self) -> dict:
        return asdict(self)

    def digest(self) -> str:
        return hashlib.sha256(json.dumps(self.payload(), sort_keys=True, separators=(",", ":")).encode()).hexdigest()


@dataclass(frozen=True)
class Measurement:
    status: str                      # "ok" | "error"
    latency_ms: float | None = None
    correctness_ok: bool | None = None
    fidelity: int = 0                # timed repetitions behind latency_ms
    clock_mhz: float | None = None
    error_message: str | None = None
    origin: str = "gpu"
    created_at: float = field(default_factory=time.time)


class MeasurementCache:
    """Every (problem, config) observation in SQLite; a re-run of a sweep reuses what was measured."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self._lock = threading.RLock()
        self._conn = sqlite3.connect(str(self.path), timeout=60.0, check_same_thread=False)
        self._conn.execute("PRAGMA journal_mode=WAL")
        self._conn.execute(
            "CREATE TABLE IF NOT EXISTS measurements (cache_key TEXT PRIMARY KEY, problem_digest TEXT NOT NULL, "
            "problem_json TEXT NOT NULL, config_json TEXT NOT NULL, measurement_json TEXT NOT NULL, "
            "updated_at REAL NOT NULL)")
        self._conn.execute("CREATE INDEX IF NOT EXISTS idx_measurements_problem ON measurements(problem_digest)")
        self._conn.commit()

    @staticmethod
    def _key(problem: ProblemKey, cfg: KernelConfig) -> str:
        cfg_json = json.dumps(asdict(cfg), sort_keys=True, separators=(",", ":"))
        return hashlib.sha256((problem.digest() + "|" + cfg_json).encode()).hexdigest()

    def get(self, problem: ProblemKey, cfg: KernelConfig) -> Measurement | None:
        with self._lock:
            row = self._conn.execute("SELECT measurement_json FROM measurements WHERE cache_key=?",
                                     (self._key(problem, cfg),)).fetchone()
        if row is None:
            return None
        known = {f.name for f in fields(Measurement)}
        return Measurement(**{k: v for k, v in json.loads(row[0]).items() if k in known})

    def put(self, problem: ProblemKey, cfg: KernelConfig, m: Measurement) -> None:
        with self._lock:
            self._conn.execute(
                "INSERT INTO measurements(cache_key, problem_digest, problem_json, config_json, measurement_json, "
                "updated_at) VALUES (?, ?, ?, ?, ?, ?) ON CONFLICT(cache_key) DO UPDATE SET "
                "measurement_json=excluded.measurement_json, updated_at=excluded.updated_at",
                (self._key(problem, cfg), problem.digest(), json.dumps(problem.payload(), sort_keys=True),
                 json.dumps(asdict(cfg), sort_keys=True), json.dumps(asdict(m), sort_keys=True), time.time()))
            self._conn.commit()

    def iter_problem(self, problem: ProblemKey):
        with self._lock:
            rows = self._conn.execute("SELECT config_json, measurement_json FROM measurements WHERE problem_digest=?",
                                      (problem.digest(),)).fetchall()
        known = {f.name for f in fields(Measurement)}
        for c, m in rows:
            yield _config_from(json.loads(c)), Measurement(**{k: v for k, v in json.loads(m).items() if k in known})

    def close(self) -> None:
        with self._lock:
            self._conn.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ----------------------------------------------------------------------- sweep
def gemm_candidates(kind: str, M: int, K: int, B: int) -> list[KernelConfig]:
    """Every launch configuration the sweep tries for one operator shape: the library's heuristic, then
    tile width x raster band (x split-K ranges for the weight update) on the tcgen05 kernel."""
    out = [KernelConfig(backend="tcgen05")]
    splits = (0, 1, 2, 4, 8, 16) if kind == "weight" else (0,)
    for bn in (128, 256):
        for raster in (4, 8, 16, 32):
            for sp in splits:
                out.append(KernelConfig(backend="tcgen05", tc_bn=bn, tc_raster=raster, tc_splits=sp, tc_pair=1))
    for raster in (4, 8, 16, 32):  # CTA pairs (256 x 256 tiles, no split)
        out.append(KernelConfig(backend="tcgen05", tc_bn=256, tc_raster=raster, tc_pair=2))
    return out


def _fingerprints(device) -> tuple[str, str]:
    import torch

    from . import _native as N
    p = torch.cuda.get_device_properties(device)
    dev = f"{p.name}|sm_{p.major}{p.minor}|{p.multi_processor_count}SM"
    code = hashlib.sha256(Path(N.LIB_PATH).read_bytes()).hexdigest()[:16] if Path(N.LIB_PATH).exists() else "none"
    return dev, code


def _operands(kind: str, M: int, K: int, B: int, dtype, device):
    """Seeded operands of one operator in the roles ``ipc_fused_gemm`` gives them (stored activations)."""
    import torch

    from . import _native as N
    g = torch.Generator(device=device).manual_seed(M * 31 + K * 7 + B)
    r = lambda *s, sc=1.0: (torch.randn(s, generator=g, device=device) * sc).to(dtype)  # noqa: E731
    if kind == "prediction":
        return N.MODE_PRED, dict(a=r(M, K, sc=K ** -0.5), b=r(K, B), out=r(M, B), aux=r(M, B)), 0
    if kind == "forward":
        return N.MODE_FORWARD, dict(a=r(M, K, sc=K ** -0.5), b=r(K, B), out=r(M, B), aux2=r(M, B)), 0
    if kind == "inference":
        return N.MODE_INFER, dict(a=r(K, M, sc=M ** -0.5), b=r(K, B), out=r(M, B), aux=r(M, B), aux2=r(M, B)), \
            N.FLAG_AOUT_STORED
    if kind == "weight":
        return N.MODE_WEIGHT, dict(a=r(M, B), b=r(K, B), out=r(M, K, sc=0.02)), 0
    raise ValueError(f"unknown kind {kind!r} (one of {KINDS})")


def sweep_gemm(kind: str, M: int, K: int, B: int, *, activation: str = "tanh", dtype=None, device=None,
               cache: MeasurementCache | None = None, reps: int = 5, flush_bytes: int = 256 << 20) -> TuningEntry:
    """Exhaustive search over ``gemm_candidates`` for one operator shape on the current GPU.

    Each candidate runs once untimed, then ``reps`` times, each after a write of ``flush_bytes`` (larger
    than L2), timed with CUDA events on the launching stream; the median is the candidate's latency.
    Measurements already in ``cache`` for this device and library build are reused; new ones are added.
    Returns the fastest candidate as a table row."""
    import torch

    from . import _native as N
    dtype = dtype or torch.bfloat16
    device = torch.device(device or "cuda")
    mode, ops, flags = _operands(kind, M, K, B, dtype, device)
    ws = torch.empty(N.SPLITK_WORKSPACE_BYTES // 4, device=device, dtype=torch.float32) if kind == "weight" else None
    flush = torch.empty(flush_bytes // 4, device=device, dtype=torch.float32)
    dev_fp, code_fp = _fingerprints(device)
    problem = ProblemKey(kind, M, K, B, activation, _dtype_name(dtype), dev_fp, code_fp)
    scale = 0.5 if kind == "inference" else 1e-6

    def call(cfg):
        N.fused_gemm(mode, ops["a"], ops["b"], ops["out"], ops.get("aux"), ops.get("aux2"), M=M, K=K, B=B,
                     scale=scale, flags=flags, act=activation, dtype=dtype, algo=cfg.backend, device=device,
                     workspace=ws, tune=cfg.tune())

    def timed(cfg, n):
        times = []
        for _ in range(n):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call(cfg)
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    cands = gemm_candidates(kind, M, K, B)
    heuristic = cands[0]
    # bring the GPU to its working clock first (>= ~50 ms busy): a cold first candidate reads slow
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.05:
        call(heuristic)
    torch.cuda.synchronize(device)
    best: tuple[float, KernelConfig] | None = None
    for cfg in cands:
        m = cache.get(problem, cfg) if cache is not None else None
        if m is None:
            try:
                call(cfg)
                m = Measurement("ok", timed(cfg, reps), True, reps)
            except (RuntimeError, ValueError) as exc:  # a configuration the kernel rejects
                m = Measurement("error", error_message=str(exc))
            if cache is not None:
                cache.put(problem, cfg, m)
        if m.status == "ok" and m.latency_ms is not None and (best is None or m.latency_ms < best[0]):
            best = (m.latency_ms, cfg)
    if best is None:
        raise RuntimeError(f"no candidate ran for {kind} {M}x{K}x{B}")
    if best[1] != heuristic:
        # confirm against the heuristic, the two interleaved (the clock moves under the power cap over
        # milliseconds, so separate runs of a few launches differ by more than many real gains): a row
        # only overrides the heuristic for a clear gain (> 3%)
        th, tb = [], []
        for _ in range(2 * reps):
            th.append(timed(heuristic, 1))
            tb.append(timed(best[1], 1))
        th, tb = statistics.median(th), statistics.median(tb)
        best = (th, heuristic) if tb > 0.97 * th else (tb, best[1])
    return TuningEntry(TuningKey(kind, M, K, B, activation, _dtype_name(dtype)), best[1], round(best[0], 5))


def main(argv=None) -> None:
    """python -m lich_b200.tuning --out TABLE.json [--cache CACHE.sqlite] --shapes kind:M:K:B,...

    Sweeps every listed operator shape on cuda:0 and writes (or extends) a tuning table."""
    import argparse

    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--cache", default="")
    ap.add_argument("--shapes", required=True, help="comma-separated kind:M:K:B (kind in %s)" % (KINDS,))
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--activation", default="tanh")
    a = ap.parse_args(argv)
    from . import _native as N
    dt = N.torch_dtype(a.dtype)
    cache = MeasurementCache(a.cache) if a.cache else None
    table = TuningTable.from_json(a.out) if Path(a.out).exists() else TuningTable((), SEARCH_SPACE)
    rows = []
    for spec in a.shapes.split(","):
        kind, M, K, B = spec.split(":")
        e = sweep_gemm(kind, int(M), int(K), int(B), activation=a.activation, dtype=dt, cache=cache)
        print(json.dumps({"kind": kind, "M": int(M), "K": int(K), "B": int(B), "best": asdict(e.config),
                          "ms": e.median_ms}), flush=True)
        rows.append(e)
    table = table.merged(TuningTable(tuple(rows), SEARCH_SPACE))
    p = torch.cuda.get_device_properties(0)
    table.to_json(a.out, device=p.name, capability=(p.major, p.minor))
    if cache is not None:
        cache.close()


if __name__ == "__main__":
    main()
