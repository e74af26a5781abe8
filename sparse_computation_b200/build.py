"""Builds libsc_b200.so in-tree for sm_100a (B200) with nvcc.

    python -m sparse_computation_b200.build          # or build() from Python

The library is self-contained (static CUDA runtime) and exports only the C
ABI declared in include/sc_b200.h.  Objects go to _build/ (git-ignored).
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.environ.get("SC_BUILD_DIR", os.path.join(ROOT, "_build"))
LIB = os.environ.get("SC_LIB", os.path.join(PKG, "libsc_b200.so"))
# Extra nvcc flags (e.g. tuning macros such as -DSC_WIDE_MINB=2) for experiments.
EXTRA_NVCC = os.environ.get("SC_NVCC_FLAGS", "").split()

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-pthread", "-Wall", "-Wno-unused-function"]

HOST_SOURCES = ["sc_host.cpp"]
# (source, extra flags, object name): sc_inst.cu is compiled once per
# (kernel_m, wide|narrow); the slowest units are listed first.
CUDA_SOURCES = [("sc_plan.cu", [], "sc_plan.cu.o"), ("sc_dense.cu", [], "sc_dense.cu.o"),
                ("sc_noalloc.cu", [], "sc_noalloc.cu.o")] + [
    ("sc_inst.cu", [f"-DSC_KM={km}", f"-DSC_PART={part}"], f"sc_inst_km{km}_{'wn'[part]}.cu.o")
    for km in (4, 6, 5, 3, 2, 1) for part in (0, 1)]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def _newer(target, deps):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    """Compiles what is missing or stale.  Serialised across processes by a
    lock file, so the ranks of one node started together build once."""
    import fcntl
    os.makedirs(BUILD, exist_ok=True)
    with open(os.path.join(BUILD, ".lock"), "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        try:
            return _build_locked(verbose, force)
        finally:
            fcntl.flock(lk, fcntl.LOCK_UN)


def _build_locked(verbose: bool, force: bool) -> str:
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(INCLUDE, "sc_b200.h"))
    jobs, objs = [], []
    for src in HOST_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or not _newer(o, [s] + headers):
            jobs.append(["g++", *CXXFLAGS, "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o])
    for src, extra, oname in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, oname)
        objs.append(o)
        if force or not _newer(o, [s] + headers):
            jobs.append([NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                         "-Xptxas", "-v" if verbose else "-O3",
                         *extra, *EXTRA_NVCC, "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o])
    with ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for out in ex.map(_run, jobs):
            if verbose and out:
                print(out)
    if force or jobs or not _newer(LIB, objs):
        os.makedirs(os.path.dirname(LIB), exist_ok=True)
        tmp = f"{LIB}.tmp{os.getpid()}"  # renamed into place: a reader never sees a partial file
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", "-Xlinker",
              "--exclude-libs,ALL", *objs, "-o", tmp, "-lpthread"])
        os.replace(tmp, LIB)
    build_apps(force=force)
    return LIB


APPS = {"spmm_demo_gpu": 0, "spmm_small_b_col_demo_gpu": 1, "spmv_demo_gpu": 2}
# Executables beside the package's own library; a library built elsewhere
# (SC_LIB, e.g. a variant with other compile flags) gets its own bin/ beside it.
BIN = os.path.join(PKG, "bin") if os.path.dirname(LIB) == PKG else os.path.join(os.path.dirname(LIB), "bin")


def build_apps(force: bool = False) -> None:
    """The three demo executables (reference command line) in sparse_computation_b200/bin/."""
    os.makedirs(BIN, exist_ok=True)
    src = os.path.join(PKG, "apps", "sc_demo.cu")
    jobs = []
    for name, mode in APPS.items():
        out = os.path.join(BIN, name)
        if force or not _newer(out, [src, LIB, os.path.join(INCLUDE, "sc_b200.h")]):
            jobs.append([NVCC, *ARCH, "-O2", "-std=c++17", f"-DSC_DEMO_MODE={mode}", "-I", INCLUDE, src,
                         "-o", out, "-L", os.path.dirname(LIB), "-l:" + os.path.basename(LIB),
                         "-Xlinker", "-rpath,$ORIGIN/..", "-lcusparse", "-lcublas"])
    with ThreadPoolExecutor(max_workers=3) as ex:
        list(ex.map(_run, jobs))


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
