"""Compile the sm_100a kernels into the in-tree shared library ``libssm_b200.so``.

    python -m metal_kernelops_b200.build [--force] [--verbose]

Every ``csrc/*.cu`` is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into an object
under ``_build/`` (in parallel), then linked into one position-independent
shared library next to this file.  Objects are rebuilt only when their source or
a header changed.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libssm_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _nvcc():
    found = shutil.which("nvcc")
    if found:
        return found
    cand = pathlib.Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found")


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(obj, src, headers):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def _compile(src, obj, verbose):
    cmd = [_nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr}")
    return proc.stderr


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if force or verbose or _stale(obj, src, headers):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(workers) as pool:
            for (src, _), log in zip(jobs, pool.map(lambda j: _compile(*j, verbose), jobs)):
                if verbose and log:
                    print(f"--- {src.name}\n{log}", file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp),
               "-lcudart"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
