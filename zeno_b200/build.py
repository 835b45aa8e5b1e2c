"""Build libzeno.so in-tree (zeno_b200/lib/libzeno.so) with nvcc for sm_100a.

The kernel is compiled with -fmad=false and IEEE division / square root so that every
floating-point operation is the one written in the source (explicit __fmaf_rn calls
are the only fused operations); host model-building code is compiled with
-ffp-contract=off for the same reason.

The library is also copied to <repo>/zig-out/lib/libzeno.so, where the reference's own
Python package and ABI check look for it.  The sources compile in parallel.

Usage: python -m zeno_b200.build [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "lib"
LIB = OUT_DIR / "libzeno.so"
# where the reference's own Python package (python/zeno/_ffi.py _find_library) and its
# tests/check_abi_contract.py look for the library: <repo>/zig-out/lib/libzeno.so
ZIG_OUT_LIB = PKG.parent / "zig-out" / "lib" / "libzeno.so"
OBJ_DIR = PKG / "_build"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc") if (CUDA_HOME / "bin" / "nvcc").exists() else "nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-fmad=false", "-prec-div=true", "-prec-sqrt=true",
                     "-ftz=false", "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-Wall",
             f"-I{CUDA_HOME / 'include'}", f"-I{INCLUDE}"]
CU_SOURCES = ["step_kernel.cu", "fast_step.cu", "noalloc.cu", "math_eval.cu"]
CXX_SOURCES = ["mjcf.cpp", "model.cpp", "fast_model.cpp", "world.cpp", "capi.cpp"]
HEADERS = ["zeno_types.h", "devmath.cuh", "physics.cuh", "model_access.cuh", "stage_clock.cuh", "fast_model.h", "step_kernel.h", "scene.h", "model.h", "world.h"]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(Path(d).stat().st_mtime <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA/C++ source and link libzeno.so; returns the library path."""
    deps = [CSRC / s for s in CU_SOURCES + CXX_SOURCES + HEADERS] + [INCLUDE / "zeno.h", Path(__file__)]
    if not force and _newer(LIB, deps):
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    cxx = shutil.which("g++") or "g++"

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr)

    jobs = [[NVCC, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(CSRC / src), "-o", str(OBJ_DIR / (src + ".o"))]
            for src in CU_SOURCES]
    jobs += [[cxx, *CXX_FLAGS, "-c", str(CSRC / src), "-o", str(OBJ_DIR / (src + ".o"))] for src in CXX_SOURCES]
    objs = [cmd[-1] for cmd in jobs]
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for f in [pool.submit(run, cmd) for cmd in jobs]:
            f.result()
    tmp = LIB.with_suffix(".so.tmp")
    run([NVCC, *ARCH, "-shared", "-o", str(tmp), *objs, "-Xlinker", "--no-undefined"])
    os.replace(tmp, LIB)
    ZIG_OUT_LIB.parent.mkdir(parents=True, exist_ok=True)
    shutil.copyfile(LIB, ZIG_OUT_LIB.with_suffix(".so.tmp"))
    os.replace(ZIG_OUT_LIB.with_suffix(".so.tmp"), ZIG_OUT_LIB)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
