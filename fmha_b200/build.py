"""Builds the native parts of fmha_b200 in-tree (no JIT cache):

* ``fmha_b200/libfmha_b200.so`` -- the CUDA C-ABI library (include/fmha.h),
  sm_100a only: the decode_*.cu kernels compiled once per head_dim, plus
  fmha_api.cu and fmha_noalloc.cu;
* ``fmha_b200/bin/fmha_host`` -- the C++ benchmark/validation host linked
  against that library (when its source is present).

Objects go to ``fmha_b200/_build``; each step reruns only when a source or
header is newer than its output. Usage: ``python -m fmha_b200.build``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfmha_b200.so")
HOST_BIN = os.path.join(PKG, "bin", "fmha_host")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                  "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the fmha_b200 CUDA library cannot be built")


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h", ".hpp"))]
    return hs + [os.path.join(ROOT, "include", "fmha.h")]


def _stale(out: str, deps) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _objects():
    objs = []
    for src, d in (("decode_bulk.cu", 128), ("decode_bulk.cu", 256),
                   ("decode_ldg.cu", 128), ("decode_ldg.cu", 256),
                   ("decode_varlen.cu", 128), ("decode_varlen.cu", 256),
                   ("decode_varlen_chunk.cu", 128), ("decode_varlen_chunk.cu", 256)):
        stem = src[:-3]
        objs.append((os.path.join(CSRC, src), os.path.join(BUILD, f"{stem}_d{d}.o"),
                     [f"-DFMHA_HEAD_DIM={d}"]))
    objs.append((os.path.join(CSRC, "fmha_api.cu"), os.path.join(BUILD, "fmha_api.o"), []))
    objs.append((os.path.join(CSRC, "fmha_noalloc.cu"), os.path.join(BUILD, "fmha_noalloc.o"), []))
    return objs


def _compile(job, verbose=False):
    src, out, extra = job
    cmd = [nvcc()] + NVFLAGS + extra + ["-c", src, "-o", out]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build_lib(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = _headers()
    jobs = [j for j in _objects() if force or _stale(j[1], [j[0]] + hdrs)]
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for log in ex.map(lambda j: _compile(j, verbose), jobs):
                if verbose and log:
                    sys.stderr.write(log)
    objs = [j[1] for j in _objects()]
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        subprocess.check_call(cmd)
    return LIB


def build_host(force: bool = False) -> str | None:
    src = os.path.join(CSRC, "fmha_host.cpp")
    if not os.path.exists(src):
        return None
    os.makedirs(os.path.dirname(HOST_BIN), exist_ok=True)
    if force or _stale(HOST_BIN, [src, LIB] + _headers()):
        cmd = [nvcc()] + ARCH + ["-O2", "-std=c++17", "-cudart", "static", "-Xcompiler", "-fopenmp",
               "-I" + os.path.join(ROOT, "include"), src, "-o", HOST_BIN,
               "-L" + PKG, "-lfmha_b200", "-Xlinker", "-rpath=$ORIGIN/..", "-lgomp"]
        subprocess.check_call(cmd)
    return HOST_BIN


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force, verbose)
    build_host(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
