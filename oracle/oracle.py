"""ctypes binding of the C oracle (oracle/oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module. It is the checker: the CUDA library never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "liboracle.so")

PINNED, STOCK = 0, 1

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile the oracle library (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    c_u32p = ctypes.POINTER(ctypes.c_uint32)
    L.orc_unif.argtypes = [c_u32p, ctypes.c_float, _f32p, ctypes.c_size_t]
    L.orc_mul_mat.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_long, ctypes.c_int, ctypes.c_int]
    L.orc_soft_max.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]
    L.orc_norm.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]
    L.orc_silu.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
    L.orc_gelu_erf.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_int]
    L.orc_erff_range.argtypes = [ctypes.c_uint32, ctypes.c_uint32, _u32p, ctypes.c_int]
    for name in ("orc_ggml_v_expf", "orc_expf_cr", "orc_erff_cr", "orc_f32_sqrt"):
        getattr(L, name).argtypes = [ctypes.c_float]
        getattr(L, name).restype = ctypes.c_float
    L.orc_f64_ew.argtypes = [ctypes.c_int, _u64p, _u64p, _u64p, ctypes.c_size_t]
    L.orc_f64_of_f32_arr.argtypes = [_f32p, _u64p, ctypes.c_size_t]
    L.orc_f32_of_f64_arr.argtypes = [_u64p, _f32p, ctypes.c_size_t]
    L.orc_f32_div_arr.argtypes = [_f32p, _f32p, _f32p, ctypes.c_size_t]
    L.orc_f32_sqrt_arr.argtypes = [_f32p, _f32p, ctypes.c_size_t]
    _lib = L
    return L


def nthreads_default() -> int:
    return max(1, os.cpu_count() or 1)


class Stream:
    """The splitmix32 stream of ref/ggml_ref.c:21-30, seeded per case."""

    def __init__(self, seed: int):
        self.state = ctypes.c_uint32(seed)

    def unif(self, a: float, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().orc_unif(ctypes.byref(self.state), ctypes.c_float(a), out, n)
        return out


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def mul_mat(w, x, K, M, R, N, wbs=0, flavour=PINNED, nthreads=None):
    """y[r*M+m] = ggml_vec_dot_f32(w row (r//N)*wbs + m*K, x row r)."""
    w = _c(w).reshape(-1)
    x = _c(x).reshape(-1)
    y = np.empty(R * M, dtype=np.float32)
    lib().orc_mul_mat(w, x, y, K, M, R, N, wbs, flavour, nthreads or nthreads_default())
    return y


def soft_max(x, ncols, rows, scale=1.0, nthreads=None):
    x = _c(x).reshape(-1)
    y = np.empty_like(x)
    lib().orc_soft_max(x, y, ncols, rows, scale, nthreads or nthreads_default())
    return y


def norm(x, ncols, rows, eps, nthreads=None):
    x = _c(x).reshape(-1)
    y = np.empty_like(x)
    lib().orc_norm(x, y, ncols, rows, eps, nthreads or nthreads_default())
    return y


def silu(x, ncols, rows):
    x = _c(x).reshape(-1)
    y = np.empty_like(x)
    lib().orc_silu(x, y, ncols, rows)
    return y


def gelu_erf(x, nthreads=None):
    x = _c(x).reshape(-1)
    y = np.empty_like(x)
    lib().orc_gelu_erf(x, y, x.size, nthreads or nthreads_default())
    return y


def erff_range(base, count, nthreads=None):
    out = np.empty(count, dtype=np.uint32)
    lib().orc_erff_range(base, count, out, nthreads or nthreads_default())
    return out


def erff_bits(xbits: np.ndarray) -> np.ndarray:
    """Correctly rounded erff of arbitrary bit patterns (uint32 in, uint32 out)."""
    L = lib()
    f = np.ascontiguousarray(xbits, dtype=np.uint32).view(np.float32)
    return np.array([L.orc_erff_cr(float(v)) for v in f], dtype=np.float32).view(np.uint32)


def ggml_v_expf(x: np.ndarray) -> np.ndarray:
    L = lib()
    return np.array([L.orc_ggml_v_expf(float(v)) for v in np.asarray(x, np.float32)], dtype=np.float32)


def f64_ew(op, a, b):
    a = _c(a, np.uint64).reshape(-1)
    b = _c(b, np.uint64).reshape(-1)
    y = np.empty_like(a)
    lib().orc_f64_ew(op, a, b, y, a.size)
    return y


def f64_of_f32(a):
    a = _c(a).reshape(-1)
    y = np.empty(a.size, dtype=np.uint64)
    lib().orc_f64_of_f32_arr(a, y, a.size)
    return y


def f32_of_f64(a):
    a = _c(a, np.uint64).reshape(-1)
    y = np.empty(a.size, dtype=np.float32)
    lib().orc_f32_of_f64_arr(a, y, a.size)
    return y


def f32_div(a, b):
    a = _c(a).reshape(-1)
    b = _c(b).reshape(-1)
    y = np.empty_like(a)
    lib().orc_f32_div_arr(a, b, y, a.size)
    return y


def f32_sqrt(a):
    a = _c(a).reshape(-1)
    y = np.empty_like(a)
    lib().orc_f32_sqrt_arr(a, y, a.size)
    return y
