"""Builds libmoe_b200.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage: python -m open_rknpu2_lm_infer_b200.build [--force] [--verbose]
Objects go to open_rknpu2_lm_infer_b200/_build/, the library next to this file.
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
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libmoe_b200.so"
INCLUDE = PKG.parent / "include"

SOURCES = ["api.cu", "router.cu", "dispatch.cu", "gemm.cu", "gemv.cu", "gemv_w8.cu", "exchange.cu",
           "noalloc.cu", "norm.cu"]
# the tensor-core rate probe (open_rknpu2_lm_infer_b200/mma_peak.py), a separate library
PEAK_SOURCE = "mma_peak.cu"
PEAK_LIB = PKG / "libmoe_b200_peak.so"
HEADERS = ["common.cuh", "kernels.cuh", "quant.cuh", "route.cuh"]

# -fmad=false: no implicit a*b+c contraction; every fused multiply-add in the
# kernels is an explicit fmaf, so rounding matches the CPU restatement.
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool, ptxas_info: bool) -> str:
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd.insert(-4, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles the CUDA sources for sm_100a and links the shared library."""
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "moe_b200.h"]
    objs, jobs = [], []
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        for s in SOURCES:
            src, obj = CSRC / s, BUILD / (Path(s).stem + ".o")
            objs.append(obj)
            if force or ptxas_info or _stale(obj, [src, *headers, Path(__file__)]):
                jobs.append(ex.submit(_compile, src, obj, verbose, ptxas_info))
        peak_obj = BUILD / (Path(PEAK_SOURCE).stem + ".o")
        if force or ptxas_info or _stale(peak_obj, [CSRC / PEAK_SOURCE, *headers, Path(__file__)]):
            jobs.append(ex.submit(_compile, CSRC / PEAK_SOURCE, peak_obj, verbose, ptxas_info))
        logs = [j.result() for j in jobs]
    if ptxas_info:
        for log in logs:
            sys.stderr.write(log)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               *map(str, objs), "-o", str(LIB), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if force or _stale(PEAK_LIB, [peak_obj]):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", str(peak_obj),
               "-o", str(PEAK_LIB), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/smem use")
    args = ap.parse_args()
    print(build(args.force, args.verbose, args.ptxas_info))
