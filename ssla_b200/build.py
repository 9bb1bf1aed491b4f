"""Build the sm_100a C-ABI library ``ssla_b200/libssla_b200.so`` in-tree with nvcc.

Usage: ``python -m ssla_b200.build [--force]``.  Objects go to ``ssla_b200/_build/``; a
source is recompiled only when it (or any header) is newer than its object.  The CUDA
runtime is linked statically so the library only needs the driver at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libssla_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-I",
    str(ROOT / "include"),
]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(src: Path, obj: Path, hdr_mtime: float) -> bool:
    if not obj.exists():
        return True
    m = obj.stat().st_mtime
    return src.stat().st_mtime > m or hdr_mtime > m


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [NVCC, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = True, extra: list[str] | None = None) -> Path:
    extra = extra or []
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    hdr_mtime = max(hdr_mtime, Path(__file__).stat().st_mtime)
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or _stale(s, o, hdr_mtime):
            jobs.append((s, o))
    if jobs:
        if verbose:
            print(f"[ssla_b200] nvcc sm_100a: {', '.join(s.name for s, _ in jobs)}", flush=True)
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(lambda j: _compile(j[0], j[1], extra), jobs))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"[ssla_b200] linked {LIB}", flush=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
