"""Build the in-tree CUDA library ``libgdn_b200.so`` for sm_100a with nvcc.

    python -m <package>.build        (or: python <package>/build.py [--verbose-ptxas])

Every ``csrc/*.cu`` file is compiled for ``sm_100a`` (tcgen05 / TMA need the
``a`` target) and linked into one shared library next to this file, where the
ctypes binding loads it.  Object files go to ``_build/`` (git-ignored).
Rebuilds only what changed (source or header newer than its object).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
# the repository keeps the C ABI header in include/; a packaged copy of the library
# (submission.py) carries it inside the package
INCLUDE = REPO / "include" if (REPO / "include" / "gdn_b200.h").exists() else PKG / "include"
BUILD = pathlib.Path(os.environ.get("GDN_B200_BUILD_DIR", str(REPO / "_build")))
LIB = PKG / "libgdn_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUTLASS_CANDIDATES = []  # headers are not needed: tcgen05 / TMA are issued as inline PTX


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def _flags(verbose_ptxas: bool):
    f = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
                "-I", str(CSRC), "--expt-relaxed-constexpr"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _stale(obj: pathlib.Path, src: pathlib.Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False, quiet: bool = False) -> pathlib.Path:
    nvcc = nvcc_path()
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    objs = []
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, src):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [nvcc, "-c", str(src), "-o", str(obj)] + _flags(verbose_ptxas)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = False
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for src, r in ex.map(compile_one, jobs):
            out = (r.stdout + r.stderr).strip()
            if r.returncode != 0:
                failed = True
                print(f"[build] FAILED {src.name}\n{out}", file=sys.stderr)
            elif out and (verbose_ptxas or not quiet):
                print(f"[build] {src.name}\n{out}")
    if failed:
        raise RuntimeError("nvcc compilation failed")
    if jobs or force or not LIB.exists():
        cmd = [nvcc, "-shared", "-o", str(LIB)] + [str(o) for o in objs] + ARCH + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    if not quiet:
        print(f"[build] {LIB} up to date")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(verbose_ptxas=a.verbose_ptxas, force=a.force)
