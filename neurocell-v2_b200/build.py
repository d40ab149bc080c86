"""Builds ``neurocell_b200/libneurocell_b200.so`` from ``csrc/*.cu`` with nvcc for sm_100a.

Usage: ``python neurocell-v2_b200/build.py [--force] [--phase-timing]``.  The library is
written in-tree next to the Python package so that it travels with the repository
snapshot.  ``--phase-timing`` builds ``libneurocell_b200_timing.so`` instead: the same
library with the fused kernels' clock64 phase marks (``NC_PHASE_TIMING``), read with
``nc_debug_fftf_phases`` / ``nc_debug_phase_times``; load it with NEUROCELL_B200_LIB.
Object files go to ``_build/`` beside this script.  Rebuilds only when a source, header or
this script is newer than the library.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "neurocell_b200", "libneurocell_b200.so")
LIB_TIMING = os.path.join(HERE, "neurocell_b200", "libneurocell_b200_timing.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build neurocell_b200")
    return cand


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    files.append(os.path.abspath(__file__))
    return files


def needs_build(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(f) > t for f in _deps())


def build(force: bool = False, phase_timing: bool = False, verbose: bool = False) -> str:
    lib = LIB_TIMING if phase_timing else LIB
    if not force and not needs_build(lib):
        return lib
    nvcc = nvcc_path()
    objdir = os.path.join(OBJDIR, "timing") if phase_timing else OBJDIR
    os.makedirs(objdir, exist_ok=True)
    flags = list(NVCC_FLAGS)
    if phase_timing:
        flags += ["-DNC_PHASE_TIMING=1"]
    srcs = _sources()

    def compile_one(src):
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *ARCH, *flags, "-I", INCLUDE, "-I", CSRC, "-rdc=false", "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = lib + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", *objs, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--phase-timing", action="store_true",
                    help="build libneurocell_b200_timing.so with the kernels' phase clocks")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, phase_timing=args.phase_timing, verbose=args.verbose))
