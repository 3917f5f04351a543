"""Builds libdressi_b200.so in-tree with nvcc for sm_100a.

    python -m opendressi_b200.build        # or opendressi_b200.build.build()

-fmad=false is required, not a tuning choice: the rasterizer's triangle-ID,
coverage and distance outputs are bit-exact with the reference CPU code only
when every multiply and add is rounded separately, as on x86-64 SSE. The
default -prec-div / -prec-sqrt / -ftz=false keep IEEE division, square root
and denormals.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdressi_b200.so")
SOURCES = ["capi.cu", "soft_raster.cu", "silhouette.cu", "hard_raster.cu",
           "fit.cu", "noalloc.cu",
           "antialias.cu", "texture.cu", "interp.cu", "regularize.cu",
           "ibl.cu", "pbr.cu", "faces.cu", "paper.cu", "paper_pixel.cu",
           "graph_ops.cpp", "graph_exec.cu", "graph_ad.cu"]
HEADERS = ["common.h", "exact.cuh", "kernels.h", "raster_soft.cuh",
           "graph.h", "graph_exec.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr",
]


# The C5 shading (pbr.cu) and the paper path's per-pixel chain
# (paper_pixel.cu) have a tolerance contract, not a bit-exact one:
# they contract a * b + c into FMAs and use the fast (<= 2 ulp) division, as
# GPU shader compilers do. Every other translation unit keeps the strict
# flags above (the raster and IBL ops are bit-exact with the reference).
FILE_FLAGS = {"pbr.cu": {"-fmad=false": "-fmad=true",
                         "-prec-div=true": "-prec-div=false"},
              "paper_pixel.cu": {"-fmad=false": "-fmad=true",
                                 "-prec-div=true": "-prec-div=false"}}


def flags_for(src: str) -> list[str]:
    sub = FILE_FLAGS.get(src, {})
    # DRESSI_NVCC_DEFINES: extra -D tuning macros of the kernels (for
    # instance "-DDRESSI_WARP_SORT=64"); empty in a normal build
    extra = os.environ.get("DRESSI_NVCC_DEFINES", "").split()
    return [sub.get(f, f) for f in NVCC_FLAGS] + extra


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin",
                        "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "dressi_b200.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False, jobs: int = 8) -> str:
    """Compiles every translation unit and links the shared library."""
    if not force and not _stale():
        return LIB
    obj_dir = os.path.join(HERE, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    objs, procs = [], []
    for src in SOURCES:
        obj = os.path.join(obj_dir, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        cmd = [nvcc(), *flags_for(src), "-c", os.path.join(CSRC, src), "-o",
               obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT)))
        if len(procs) >= jobs:
            _wait(procs.pop(0))
    for p in procs:
        _wait(p)
    link = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
            "-o", LIB, *objs, "-lcudart"]
    out = subprocess.run(link, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("link failed:\n" + out.stdout + out.stderr)
    return LIB


def _wait(item):
    src, p = item
    out, _ = p.communicate()
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{out.decode()}")


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
