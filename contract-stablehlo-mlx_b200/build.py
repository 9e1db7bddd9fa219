"""Build libshlo_cuda.so for sm_100a (nvcc; no GPU needed).

    python contract-stablehlo-mlx_b200/build.py [--verbose-ptxas]

The library is written in-tree (contract-stablehlo-mlx_b200/lib/), so it travels
with the repository snapshot to the GPU host.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
OBJ_DIR = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(LIB_DIR, "libshlo_cuda.so")

# The mul_mat kernel instances sit in six units of their own, compiled in
# parallel with the rest (the longest compiles of the library).
SOURCES = ["mul_mat_tm_split1.cu", "mul_mat_tm_split2.cu", "mul_mat_tm_split4.cu", "mul_mat_tm_split8.cu",
           "mul_mat_tm_split16.cu", "mul_mat_short.cu", "mul_mat_seg.cu",
           "ggml_kernels.cu", "attention.cu", "runtime.cu", "elementwise.cu", "api.cu", "fusion.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    # Exact IEEE binary32: no contraction of a*b+c, correctly rounded / and sqrt,
    # subnormals kept. Fused multiply-adds are written out where ggml uses them.
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    deps.append(os.path.join(HERE, "..", "include", "shlo_cuda.h"))
    if os.path.exists(obj) and all(os.path.getmtime(obj) >= os.path.getmtime(d) for d in deps) and not verbose_ptxas:
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, "-c", path, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed on %s:\n%s\n%s" % (src, r.stdout, r.stderr))
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), SOURCES))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [nvcc(), "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a",
               *objs, "-o", LIB + ".tmp", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="--verbose-ptxas" in sys.argv))
