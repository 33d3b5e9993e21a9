"""Builds the in-tree native libraries of kt_gguf_b200.

  lib/libkt_gguf_b200.so   the CUDA library behind include/kt_gguf_b200.h (sm_100a only)
  lib/libkt_gguf_encode.so host-side GGUF encoders for synthetic expert weights

nvcc compiles each .cu file for `-gencode arch=compute_100a,code=sm_100a` in parallel, then
links them into one shared library with the static CUDA runtime. No GPU is needed to build.

Usage: python -m kt_gguf_b200.build [--force] [--verbose]
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
LIB = PKG / "lib"
CUDA_SOURCES = ["capi.cu", "moe_vec.cu", "moe_misc.cu", "moe_gemm.cu", "ep.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _deps(src: Path):
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "kt_gguf_b200.h"]


def _stale(out: Path, inputs) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, flush=True)
    return r


def build_cuda(force=False, verbose=False, extra_flags=()) -> Path:
    LIB.mkdir(exist_ok=True)
    obj_dir = LIB / "obj"
    obj_dir.mkdir(exist_ok=True)
    out = LIB / "libkt_gguf_b200.so"
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
             f"-I{CSRC}", f"-I{INCLUDE}", *ARCH, *extra_flags]
    jobs = []
    for name in CUDA_SOURCES:
        src = CSRC / name
        obj = obj_dir / (name + ".o")
        if force or _stale(obj, _deps(src)):
            jobs.append([nvcc(), *flags, "-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=len(jobs)) as ex:
            list(ex.map(lambda c: _run(c, verbose), jobs))
    objs = [obj_dir / (n + ".o") for n in CUDA_SOURCES]
    if force or jobs or _stale(out, objs):
        _run([nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(out), *map(str, objs),
              "-cudart=static"], verbose)
    return out


def build_encoder(force=False, verbose=False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / "libkt_gguf_encode.so"
    src = CSRC / "gguf_encode.c"
    if force or _stale(out, [src, CSRC / "iq3s_grid.h"]):
        _run(["gcc", "-O2", "-fPIC", "-std=gnu11", "-fopenmp", "-shared", f"-I{CSRC}", "-o", str(out), str(src), "-lm"],
             verbose)
    return out


def build_all(force=False, verbose=False):
    return build_cuda(force, verbose), build_encoder(force, verbose)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    for p in build_all(a.force, a.verbose):
        print(p)


if __name__ == "__main__":
    sys.exit(main())
