"""Compiles the optimizer-step library for sm_100a (nvcc cross-compiles
without a GPU). The .so is built in-tree so it travels with the working tree."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # soar.cpp_b200/
CSRC = ROOT / "csrc"
LIBDIR = ROOT / "lib"
LIB = LIBDIR / "libsoar_optim.so"
INCLUDE = ROOT.parent / "include"

SOURCES = ["optim_kernels.cu", "optim_capi.cu", "noalloc_sumsq.cu", "zero1.cu",
           "dp_bootstrap.cu"]
HEADERS = ["optim_kernels.cuh", "pipeline.cuh"]
# the bench-only NVLink probe: a library of its own, not part of the C-ABI
PROBE_LIB = LIBDIR / "libsoar_probe.so"
PROBE_SOURCES = ["nvlink_probe.cu"]
PROBE_HEADERS = ["bench_probe.h", "optim_kernels.cuh", "pipeline.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    # every float op in the update is an explicitly rounded intrinsic; keep
    # the compiler from contracting anything else
    "-fmad=false",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
    "-shared",
    "-ldl",   # NCCL is opened with dlopen by the data-parallel bootstrap
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found: the CUDA extension cannot be built")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "soar_optim.h"]
    return any(d.stat().st_mtime > t for d in deps)


SYNTH_SRC = CSRC / "synth.c"
SYNTH_LIB = LIBDIR / "libsoar_synth.so"


def build_synth(force: bool = False) -> Path:
    """Host-only input generator (gcc + OpenMP)."""
    if not force and SYNTH_LIB.exists() and SYNTH_LIB.stat().st_mtime >= SYNTH_SRC.stat().st_mtime:
        return SYNTH_LIB
    LIBDIR.mkdir(exist_ok=True)
    cc = "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else "gcc"
    tmp = SYNTH_LIB.with_suffix(f".so.tmp{os.getpid()}")  # concurrent builders do not collide
    subprocess.run([cc, "-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared", "-ffp-contract=off",
                    "-o", str(tmp), str(SYNTH_SRC), "-lm"], check=True)
    tmp.replace(SYNTH_LIB)
    return SYNTH_LIB


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")  # concurrent builders do not collide
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp),
           *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


def build_probe(force: bool = False, verbose: bool = False) -> Path:
    """The bench-only NVLink probe library (csrc/bench_probe.h)."""
    deps = [CSRC / s for s in PROBE_SOURCES + PROBE_HEADERS]
    if not force and PROBE_LIB.exists() and \
            all(d.stat().st_mtime <= PROBE_LIB.stat().st_mtime for d in deps):
        return PROBE_LIB
    LIBDIR.mkdir(exist_ok=True)
    tmp = PROBE_LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *[str(CSRC / s) for s in PROBE_SOURCES]]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(PROBE_LIB)
    return PROBE_LIB
