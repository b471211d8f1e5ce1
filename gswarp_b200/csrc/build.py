"""Build libgsb200.so (sm_100a) from the .cu sources in this directory.

Each translation unit is compiled by nvcc for sm_100a only; units whose
results must match the CPU oracle bit for bit (preprocess, binning,
preprocess backward, KNN) are compiled with -fmad=false.  The shared library
is written in-tree to gswarp_b200/_lib/libgsb200.so so that it travels with
the repository snapshot.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
BUILD_DIR = PKG / "_build"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libgsb200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-ccbin", "g++"]
# Units that must reproduce the oracle's IEEE binary32 arithmetic exactly.
NO_FMA = {"preprocess.cu", "binning.cu", "preprocess_bwd.cu", "knn.cu"}
SOURCES = ["capi.cu", "preprocess.cu", "binning.cu", "render.cu", "preprocess_bwd.cu", "sh_views.cu",
           "ssim.cu", "knn.cu", "optim.cu", "peaks.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _flags(src: str) -> list[str]:
    f = list(COMMON)
    f += ["-fmad=false"] if src in NO_FMA else ["-fmad=true"]
    return f


def _needs_build(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(HERE.glob("*.cuh")) + [PKG.parent / "include" / "gsb200.h"]
    mt = obj.stat().st_mtime
    return any(d.stat().st_mtime > mt for d in deps if d.exists())


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    compiler = nvcc()
    objs = []
    jobs = []
    for s in SOURCES:
        src = HERE / s
        obj = BUILD_DIR / (s + ".o")
        objs.append(obj)
        if _needs_build(obj, src) or ptxas_info:
            cmd = [compiler, *ARCH, *_flags(s), "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((s, cmd))

    def run(job):
        name, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return name, cmd, r

    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for name, cmd, r in ex.map(run, jobs):
                if verbose or ptxas_info or r.returncode != 0:
                    sys.stderr.write(f"[nvcc] {name}\n{r.stdout}{r.stderr}")
                if r.returncode != 0:
                    raise RuntimeError(f"nvcc failed for {name}:\n{' '.join(cmd)}\n{r.stderr}")
    if jobs or not LIB_PATH.exists():
        cmd = [compiler, *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
