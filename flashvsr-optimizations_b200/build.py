"""Build libfvq.so (the C-ABI CUDA library) in-tree for sm_100a.

    python flashvsr-optimizations_b200/build.py [--force] [--verbose]

Each .cu file is compiled separately (nvcc -c, cached by mtime) and linked
into ``libfvq.so`` beside this file.  cudart is linked statically so the
library works inside any process that already has a CUDA context (torch's
included) without depending on which libcudart that process loaded.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "libfvq.so"

SOURCES = ["fvq_quant.cu", "fvq_fp8.cu", "fvq_resize.cu", "fvq_block.cu", "fvq_gemm.cu",
           "fvq_api.cu", "fvq_noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr", "-Xptxas", "-v",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    objs = []
    changed = force or not LIB.exists()
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            cmd = [nvcc(), *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if verbose or res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}")
            (BUILD / (src + ".ptxas.txt")).write_text(res.stderr)
            changed = True
    if changed or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link of libfvq.so failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
