"""Builds libmomij_moe.so in-tree (momij_b200/lib/) for sm_100a with nvcc.

Each .cu under csrc/ is compiled separately (parallel), then linked into one
shared library with the CUDA runtime linked statically, so the library does
not depend on which libcudart the host process has loaded.  Usage:
``python -m momij_b200.build [-j N] [--verbose-ptxas]``.
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
OBJ = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libmomij_moe.so")
SOURCES = ["route.cu", "gemv.cu", "layer.cu", "token.cu", "decode.cu", "block.cu", "prefill.cu", "ep.cu", "ep_host.cu", "misc.cu",
           "api.cu", "noalloc.cu"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _flags(verbose_ptxas: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "-I", os.path.join(ROOT, "include"), "-I", CSRC, "--expt-relaxed-constexpr",
                "-ccbin", "/usr/bin/g++"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: str, verbose_ptxas: bool) -> str:
    out = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    deps.append(os.path.join(ROOT, "include", "momij_moe.h"))
    if (not verbose_ptxas and os.path.exists(out)
            and os.path.getmtime(out) >= max(os.path.getmtime(d) for d in deps)):
        return out
    cmd = [nvcc()] + _flags(verbose_ptxas) + ["-c", path, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return out


def build(jobs: int = 4, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), SOURCES))
    if (not os.path.exists(LIB) or
            os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-ldl",
                                                                  "-ccbin", "/usr/bin/g++"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=4)
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(args.j, args.verbose_ptxas))
