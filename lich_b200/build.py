"""Build the native library ``lich_b200/_lib/libipc_b200.so`` for sm_100a.

    python -m lich_b200.build [--verbose] [--ptxas-info]

Each ``csrc/*.cu`` is compiled by nvcc (``-gencode arch=compute_100a,code=sm_100a``)
in parallel, then linked into one shared library with the CUDA runtime
linked statically, so the library depends only on the driver.  The build is
incremental: an object is rebuilt when its source or any ``csrc/*.cuh`` /
``include/*.h`` header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_lib" / "obj"
LIB = PKG / "_lib" / "libipc_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, extra: list[str], verbose: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and ("-Xptxas" in " ".join(extra) or verbose):
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr_t = _headers_mtime()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    todo = []
    for s in srcs:
        o = OBJ / (s.stem + ".o")
        if force or ptxas_info or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_t):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda s: _compile(s, extra, verbose), todo))
    objs = [OBJ / (s.stem + ".o") for s in srcs]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        # --no-undefined: a symbol missing at link time is a build error, not a dlopen failure later
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--no-undefined", "-o", str(tmp),
               *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem per kernel")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force))


if __name__ == "__main__":
    main()
