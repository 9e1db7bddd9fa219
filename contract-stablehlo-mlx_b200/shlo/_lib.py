"""ctypes binding of libshlo_cuda.so (include/shlo_cuda.h)."""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("SHLO_CUDA_LIB", os.path.join(PKG, "lib", "libshlo_cuda.so"))

# Every exported symbol of include/shlo_cuda.h.
SYMBOLS = [
    "shlo_last_error", "shlo_set_device", "shlo_get_device", "shlo_device_count", "shlo_set_flavor",
    "shlo_get_flavor", "shlo_retain", "shlo_release", "shlo_empty", "shlo_of_bytes", "shlo_nbytes",
    "shlo_to_bytes", "shlo_shape", "shlo_dtype", "shlo_unary", "shlo_binary", "shlo_where", "shlo_reshape",
    "shlo_transpose", "shlo_broadcast", "shlo_slice", "shlo_concat", "shlo_astype", "shlo_view", "shlo_take",
    "shlo_max_axis", "shlo_contiguous", "shlo_eval", "shlo_kernel_new", "shlo_kernel_free",
    "shlo_kernel_apply", "shlo_compile", "shlo_fn_free", "shlo_apply", "shlo_libm_erff_range",
    "shlo_count_nonzero", "shlo_current_stream", "shlo_launch_count", "shlo_device_ptr", "shlo_mul_mat_noalloc",
]


class ShloError(RuntimeError):
    """An error status from libshlo_cuda (the message of shlo_last_error)."""


c_arr = ctypes.c_void_p
c_i64p = ctypes.POINTER(ctypes.c_int64)
TRACE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(c_arr), ctypes.c_int,
                            ctypes.POINTER(c_arr), ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                            ctypes.c_void_p, ctypes.c_size_t)
FREE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError("libshlo_cuda.so is not built (%s); run contract-stablehlo-mlx_b200/build.py" % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    i = ctypes.c_int
    L.shlo_last_error.restype = ctypes.c_char_p
    L.shlo_last_error.argtypes = []
    L.shlo_set_device.argtypes = [i]
    L.shlo_get_device.argtypes = [ctypes.POINTER(i)]
    L.shlo_device_count.argtypes = [ctypes.POINTER(i)]
    L.shlo_set_flavor.argtypes = [i]
    L.shlo_get_flavor.argtypes = [ctypes.POINTER(i)]
    L.shlo_retain.argtypes = [c_arr]
    L.shlo_retain.restype = None
    L.shlo_release.argtypes = [c_arr]
    L.shlo_release.restype = None
    L.shlo_empty.argtypes = []
    L.shlo_empty.restype = c_arr
    L.shlo_of_bytes.argtypes = [ctypes.c_void_p, ctypes.c_size_t, c_i64p, i, ctypes.c_uint8, ctypes.POINTER(c_arr)]
    L.shlo_nbytes.argtypes = [c_arr, ctypes.POINTER(ctypes.c_size_t)]
    L.shlo_to_bytes.argtypes = [c_arr, ctypes.c_void_p, ctypes.c_size_t]
    L.shlo_shape.argtypes = [c_arr, c_i64p, ctypes.POINTER(i)]
    L.shlo_dtype.argtypes = [c_arr, ctypes.POINTER(ctypes.c_uint8)]
    L.shlo_unary.argtypes = [ctypes.c_uint32, c_arr, ctypes.POINTER(c_arr)]
    L.shlo_binary.argtypes = [ctypes.c_uint32, c_arr, c_arr, ctypes.POINTER(c_arr)]
    L.shlo_where.argtypes = [c_arr, c_arr, c_arr, ctypes.POINTER(c_arr)]
    L.shlo_reshape.argtypes = [c_arr, c_i64p, i, ctypes.POINTER(c_arr)]
    L.shlo_transpose.argtypes = [c_arr, c_i64p, i, ctypes.POINTER(c_arr)]
    L.shlo_broadcast.argtypes = [c_arr, c_i64p, i, ctypes.POINTER(c_arr)]
    L.shlo_slice.argtypes = [c_arr, c_i64p, c_i64p, c_i64p, i, ctypes.POINTER(c_arr)]
    L.shlo_concat.argtypes = [ctypes.POINTER(c_arr), i, ctypes.c_uint32, ctypes.POINTER(c_arr)]
    L.shlo_astype.argtypes = [c_arr, ctypes.c_uint8, ctypes.POINTER(c_arr)]
    L.shlo_view.argtypes = [c_arr, ctypes.c_uint8, ctypes.POINTER(c_arr)]
    L.shlo_take.argtypes = [c_arr, c_arr, ctypes.c_uint32, ctypes.POINTER(c_arr)]
    L.shlo_max_axis.argtypes = [c_arr, ctypes.c_uint32, ctypes.POINTER(c_arr)]
    L.shlo_contiguous.argtypes = [c_arr, ctypes.POINTER(c_arr)]
    L.shlo_eval.argtypes = [ctypes.POINTER(c_arr), i]
    L.shlo_kernel_new.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), i,
                                  ctypes.POINTER(ctypes.c_char_p), i, ctypes.c_char_p, ctypes.c_char_p,
                                  ctypes.POINTER(ctypes.c_void_p)]
    L.shlo_kernel_free.argtypes = [ctypes.c_void_p]
    L.shlo_kernel_free.restype = None
    L.shlo_kernel_apply.argtypes = [ctypes.c_void_p, ctypes.POINTER(c_arr), i, ctypes.POINTER(c_i64p),
                                    ctypes.POINTER(i), ctypes.POINTER(ctypes.c_uint8), i, c_i64p, c_i64p,
                                    ctypes.POINTER(c_arr)]
    L.shlo_compile.argtypes = [TRACE_FN, ctypes.c_void_p, FREE_FN, i, ctypes.POINTER(ctypes.c_void_p)]
    L.shlo_fn_free.argtypes = [ctypes.c_void_p]
    L.shlo_fn_free.restype = None
    L.shlo_apply.argtypes = [ctypes.c_void_p, ctypes.POINTER(c_arr), i, ctypes.POINTER(c_arr),
                             ctypes.POINTER(i), i]
    L.shlo_libm_erff_range.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p]
    L.shlo_count_nonzero.argtypes = [c_arr, ctypes.POINTER(ctypes.c_uint64)]
    L.shlo_current_stream.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
    L.shlo_launch_count.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
    L.shlo_device_ptr.argtypes = [c_arr, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(i)]
    L.shlo_mul_mat_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_void_p]
    special = {"shlo_last_error", "shlo_empty", "shlo_retain", "shlo_release", "shlo_kernel_free", "shlo_fn_free"}
    for name in SYMBOLS:
        if name not in special:
            getattr(L, name).restype = ctypes.c_int
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != 0:
        raise ShloError(load().shlo_last_error().decode("utf-8", "replace"))
