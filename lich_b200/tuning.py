"""Per-shape kernel tuning table with the reference's JSON schema (``schema_version`` 1).

Same file format as ``src/ipc_tilelang/tuning.py:10-108`` so existing tables
load; rows are keyed by ``(kind, M, K, B, activation, dtype)`` and carry a
``KernelConfig`` (whose ``backend`` field selects the sm_100a algorithm).
Tables written here record ``"search_space": "sm100a-v1"``; tables measured
on other GPUs load but describe other hardware.
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, fields
from pathlib import Path
from typing import Iterable

from .tilelang_kernels import KernelConfig

SCHEMA_VERSION = 1
SEARCH_SPACE = "sm100a-v1"


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

    @classmethod
    def from_entries(cls, entries: Iterable[TuningEntry]) -> "TuningTable":
        return cls(tuple(entries))

    @classmethod
    def from_json(cls, path: str | Path) -> "TuningTable":
        payload = json.loads(Path(path).read_text(encoding="utf-8"))
        if payload.get("schema_version") != SCHEMA_VERSION:
            raise ValueError(f"Unsupported tuning schema: {payload.get('schema_version')!r}; expected {SCHEMA_VERSION}")
        known = {f.name for f in fields(KernelConfig)}
        out = []
        for row in payload.get("entries", []):
            shape = row["shape"]
            cfg = KernelConfig(**{k: v for k, v in row["config"].items() if k in known})
            key = TuningKey(str(row["kind"]), int(shape["M"]), int(shape["K"]), int(shape["B"]),
                            str(row.get("activation", "relu")), str(row.get("dtype", "float16")))
            med = row.get("median_ms")
            out.append(TuningEntry(key, cfg, None if med is None else float(med), row.get("spill_suspected")))
        return cls(tuple(out))

    def lookup(self, *, kind: str, M: int, K: int, B: int, activation: str, dtype: str) -> KernelConfig | None:
        want = TuningKey(kind, int(M), int(K), int(B), activation, dtype)
        for e in self.entries:
            if e.key == want:
                return e.config
        return None

    def to_json(self, path: str | Path, *, device: str | None = None,
                capability: tuple[int, int] | None = None) -> None:
        rows = [{"kind": e.key.kind, "shape": {"M": e.key.M, "K": e.key.K, "B": e.key.B},
                 "activation": e.key.activation, "dtype": e.key.dtype, "median_ms": e.median_ms,
                 "spill_suspected": e.spill_suspected, "config": asdict(e.config)} for e in self.entries]
        payload = {"schema_version": SCHEMA_VERSION, "search_space": SEARCH_SPACE, "device": device,
                   "capability": list(capability) if capability is not None else None, "entries": rows}
        out = Path(path)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps(payload, indent=2), encoding="utf-8")
