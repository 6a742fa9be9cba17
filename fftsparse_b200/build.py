"""Compile libfftsparse_b200.so (all CUDA sources under csrc/) for sm_100a.

The library is built in-tree next to this file so that it travels with the
repository; nvcc cross-compiles without a GPU.  A second variant,
libfftsparse_b200_checked.so, is the same sources compiled with
-DFFTS_BOUNDS_CHECK: every data-dependent or ragged-edge kernel index is tested
against its extent, and a failure is recorded (ffts_bounds_report) and the access
skipped instead of faulting.  FFTS_LIBRARY=checked makes the package load it.

    python -m fftsparse_b200.build [--force] [--verbose] [--normal-only]
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libfftsparse_b200.so")
LIB_CHECKED = os.path.join(HERE, "libfftsparse_b200_checked.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]
VARIANTS = {LIB: [], LIB_CHECKED: ["-DFFTS_BOUNDS_CHECK"]}


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(INCLUDE, "fftsparse_b200.h")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(p) <= t for p in _deps())


def _link(lib: str, objs) -> None:
    tmp = lib + ".tmp"
    subprocess.run([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs],
                   check=True)
    os.replace(tmp, lib)


def build(force: bool = False, verbose: bool = False, checked: bool = True) -> str:
    """Build the normal library (and, unless checked=False, the bounds-checked
    one); returns the normal library's path."""
    libs = [LIB] + ([LIB_CHECKED] if checked else [])
    todo = [lib for lib in libs if force or not up_to_date(lib)]
    if not todo:
        return LIB
    jobs = []
    for lib in todo:
        sub = "checked" if lib == LIB_CHECKED else "normal"
        build_dir = os.path.join(HERE, "_build", sub)
        os.makedirs(build_dir, exist_ok=True)
        for src in _sources():
            obj = os.path.join(build_dir, os.path.basename(src) + ".o")
            cmd = [nvcc(), *NVCC_FLAGS, *VARIANTS[lib], "-I", INCLUDE, "-c", src, "-o", obj]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append((lib, obj, cmd))
    workers = max(1, min(len(jobs), os.cpu_count() or 1, 8))
    with cf.ThreadPoolExecutor(workers) as ex:
        for fut in [ex.submit(subprocess.run, cmd, check=True) for _, _, cmd in jobs]:
            fut.result()
    for lib in todo:
        _link(lib, [obj for l, obj, _ in jobs if l == lib])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv,
                checked="--normal-only" not in sys.argv))
