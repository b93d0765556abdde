"""Ahead-of-time build of the C-ABI library ``tensorium_b200/libtensorium_b200.so``.

Every ``csrc/*.cu`` file is compiled by nvcc for sm_100a only (the reference instead JIT-compiles
one generic .cu string with NVRTC at start-up, source/nncuda.pas:1586-1642) and linked into one
shared library with a plain C ABI (include/tensorium_b200.h).  The library is built in-tree so it
travels with the repository snapshot.

    python -m tensorium_b200.build [--force] [-j N] [-v]
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
OBJ = PKG / "_build"
LIB = PKG / "libtensorium_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: no silent a*b+c contraction; every FMA on the path is an explicit fmaf, so the
# separate roundings of the reference's epilogue arithmetic are kept.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "tensorium_b200.h"]


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool, extra) -> Path:
    obj = OBJ / (src.stem + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout + r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, extra=()) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = _sources()
    if force:
        for o in OBJ.glob("*.o"):
            o.unlink()
    jobs = jobs or min(8, os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, list(extra)), srcs))
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, jobs=a.j, verbose=a.v or a.ptxas_info, extra=extra))


if __name__ == "__main__":
    main()
