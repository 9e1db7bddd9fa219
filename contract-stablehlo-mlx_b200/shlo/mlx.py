"""StablehloMlx/Mlx.lean restated over libshlo_cuda: the arrays, ops and kernels.

Each function is one call of the C ABI (include/shlo_cuda.h) -- the same role
as each `@[extern]` declaration of Mlx.lean:16-73. Names follow the Lean
declarations (snake case); errors raise ShloError, as the Lean shim returns an
IO error (c/smlx_shim.c:34-41).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import numpy as np

from ._lib import FREE_FN, TRACE_FN, ShloError, c_arr, check, load

# The library is mapped when this module is imported: a missing or unloadable
# libshlo_cuda.so fails here, never later inside an op.
load()

# mlx_dtype codes (Mlx.lean:30-37)
dtBool, dtU8, dtU16, dtU32, dtU64, dtI8, dtI16, dtI32, dtI64, dtF16, dtF32 = range(11)

NP_OF = {dtBool: np.bool_, dtU8: np.uint8, dtU16: np.uint16, dtU32: np.uint32, dtU64: np.uint64,
         dtI8: np.int8, dtI16: np.int16, dtI32: np.int32, dtI64: np.int64, dtF16: np.float16,
         dtF32: np.float32}
DT_OF = {np.dtype(v): k for k, v in NP_OF.items()}

# unary op codes (Mlx.lean:76-86)
opNeg, opAbs, opSqrt, opFloor, opExp, opErf, opNot, opInvert, opRsqrt, opTanh, opSigmoid = range(11)
# binary op codes (Mlx.lean:87-108)
(opAdd, opSub, opMul, opDiv, opMax, opMin, opAnd, opOr, opXor, opShl, opShr, opEq, opNe, opLt, opLe, opGt,
 opGe, opMatmul, opRem, opLAnd, opLOr) = range(21)


class Arr:
    """One reference to a device array (the Lean external object `Arr`)."""

    __slots__ = ("h",)

    def __init__(self, handle: int):
        self.h = handle

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            try:
                load().shlo_release(h)
            except Exception:
                pass
            self.h = None

    @property
    def shape(self) -> tuple:
        return shape(self)

    @property
    def dtype(self) -> int:
        return dtype(self)


def _i64(xs: Sequence[int]):
    arr = (ctypes.c_int64 * max(len(xs), 1))(*[int(v) for v in xs])
    return arr


def _out(fn, *args) -> Arr:
    o = c_arr()
    check(fn(*args, ctypes.byref(o)))
    return Arr(o.value)


def empty_arr() -> Arr:
    return Arr(load().shlo_empty())


def of_bytes(data: bytes, shape_: Sequence[int], dt: int) -> Arr:
    buf = bytes(data)
    return _out(load().shlo_of_bytes, buf, len(buf), _i64(shape_), len(shape_), dt)


def of_numpy(a: np.ndarray, dt: int | None = None) -> Arr:
    """ofBytes of a numpy array's row-major bytes (its own dtype unless `dt`)."""
    a = np.ascontiguousarray(a)
    if dt is None:
        dt = DT_OF[a.dtype]
    L = load()
    o = c_arr()
    check(L.shlo_of_bytes(a.ctypes.data_as(ctypes.c_void_p), a.nbytes, _i64(a.shape), a.ndim, dt, ctypes.byref(o)))
    return Arr(o.value)


def of_ptr(ptr: int, nbytes: int, shape_: Sequence[int], dt: int) -> Arr:
    """ofBytes from raw host memory (e.g. a pinned buffer)."""
    return _out(load().shlo_of_bytes, ctypes.c_void_p(ptr), nbytes, _i64(shape_), len(shape_), dt)


def to_ptr(a: Arr, ptr: int, cap: int) -> None:
    """toBytes into raw host memory."""
    check(load().shlo_to_bytes(a.h, ctypes.c_void_p(ptr), cap))


def to_bytes(a: Arr) -> bytes:
    L = load()
    n = ctypes.c_size_t()
    check(L.shlo_nbytes(a.h, ctypes.byref(n)))
    buf = ctypes.create_string_buffer(max(n.value, 1))
    check(L.shlo_to_bytes(a.h, buf, n.value))
    return buf.raw[: n.value]


def to_numpy(a: Arr) -> np.ndarray:
    L = load()
    n = ctypes.c_size_t()
    check(L.shlo_nbytes(a.h, ctypes.byref(n)))
    out = np.empty(shape(a), dtype=NP_OF[dtype(a)])
    check(L.shlo_to_bytes(a.h, out.ctypes.data_as(ctypes.c_void_p), out.nbytes))
    return out


def shape(a: Arr) -> tuple:
    s = (ctypes.c_int64 * 16)()
    n = ctypes.c_int()
    check(load().shlo_shape(a.h, s, ctypes.byref(n)))
    return tuple(s[i] for i in range(n.value))


def dtype(a: Arr) -> int:
    d = ctypes.c_uint8()
    check(load().shlo_dtype(a.h, ctypes.byref(d)))
    return d.value


def unary(op: int, a: Arr) -> Arr:
    return _out(load().shlo_unary, op, a.h)


def binary(op: int, a: Arr, b: Arr) -> Arr:
    return _out(load().shlo_binary, op, a.h, b.h)


def where_(c: Arr, a: Arr, b: Arr) -> Arr:
    return _out(load().shlo_where, c.h, a.h, b.h)


def reshape(a: Arr, shape_: Sequence[int]) -> Arr:
    return _out(load().shlo_reshape, a.h, _i64(shape_), len(shape_))


def transpose(a: Arr, perm: Sequence[int]) -> Arr:
    return _out(load().shlo_transpose, a.h, _i64(perm), len(perm))


def broadcast(a: Arr, shape_: Sequence[int]) -> Arr:
    return _out(load().shlo_broadcast, a.h, _i64(shape_), len(shape_))


def slice_(a: Arr, start, stop, step) -> Arr:
    return _out(load().shlo_slice, a.h, _i64(start), _i64(stop), _i64(step), len(start))


def concat(xs: Sequence[Arr], axis: int) -> Arr:
    hs = (c_arr * len(xs))(*[x.h for x in xs])
    return _out(load().shlo_concat, hs, len(xs), axis)


def astype(a: Arr, dt: int) -> Arr:
    return _out(load().shlo_astype, a.h, dt)


def view(a: Arr, dt: int) -> Arr:
    return _out(load().shlo_view, a.h, dt)


def take(a: Arr, idx: Arr, axis: int) -> Arr:
    return _out(load().shlo_take, a.h, idx.h, axis)


def max_axis(a: Arr, axis: int) -> Arr:
    return _out(load().shlo_max_axis, a.h, axis)


def contiguous(a: Arr) -> Arr:
    return _out(load().shlo_contiguous, a.h)


def eval_(xs: Sequence[Arr]) -> None:
    hs = (c_arr * max(len(xs), 1))(*[x.h for x in xs])
    check(load().shlo_eval(hs, len(xs)))


class Kernel:
    """The Lean external object `Kernel` (Mlx.lean:18-21)."""

    __slots__ = ("h", "name")

    def __init__(self, h, name):
        self.h = h
        self.name = name

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            try:
                load().shlo_kernel_free(h)
            except Exception:
                pass
            self.h = None


def kernel_new(name: str, inputs: Sequence[str], outputs: Sequence[str], source: str, header: str) -> Kernel:
    L = load()
    ins = (ctypes.c_char_p * max(len(inputs), 1))(*[s.encode() for s in inputs])
    outs = (ctypes.c_char_p * max(len(outputs), 1))(*[s.encode() for s in outputs])
    h = ctypes.c_void_p()
    check(L.shlo_kernel_new(name.encode(), ins, len(inputs), outs, len(outputs), source.encode(), header.encode(),
                            ctypes.byref(h)))
    return Kernel(h.value, name)


def kernel_apply(k: Kernel, inputs: Sequence[Arr], out_shapes: Sequence[Sequence[int]], out_dtypes: bytes,
                 grid: Sequence[int], threadgroup: Sequence[int]) -> list:
    L = load()
    hs = (c_arr * len(inputs))(*[a.h for a in inputs])
    shape_arrs = [_i64(s) for s in out_shapes]
    shp = (ctypes.POINTER(ctypes.c_int64) * len(out_shapes))(
        *[ctypes.cast(s, ctypes.POINTER(ctypes.c_int64)) for s in shape_arrs])
    nd = (ctypes.c_int * len(out_shapes))(*[len(s) for s in out_shapes])
    dts = (ctypes.c_uint8 * len(out_shapes))(*list(out_dtypes))
    outs = (c_arr * len(out_shapes))()
    check(L.shlo_kernel_apply(k.h, hs, len(inputs), shp, nd, dts, len(out_shapes), _i64(grid), _i64(threadgroup),
                              outs))
    return [Arr(outs[i]) for i in range(len(out_shapes))]


class Fn:
    """A traced function (Mlx.lean:23-26): compile wraps a Python callable
    `f(list[Arr]) -> list[Arr]` the way smlx_compile wraps a Lean closure."""

    def __init__(self, f: Callable, enable: bool):
        self._f = f
        self._err = None

        def tramp(payload, ins, nin, outs, nout, max_out, err, err_cap):
            try:
                args = []
                for i in range(nin):
                    load().shlo_retain(ins[i])
                    args.append(Arr(ins[i]))
                res = f(args)
                if len(res) > max_out:
                    raise ShloError("%d outputs, room for %d" % (len(res), max_out))
                for i, r in enumerate(res):
                    load().shlo_retain(r.h)
                    outs[i] = r.h
                nout[0] = len(res)
                return 0
            except Exception as e:  # the trace error travels back as the message
                msg = ("%s: %s" % (type(e).__name__, e)).encode()[: max(int(err_cap) - 1, 0)]
                ctypes.memmove(err, msg + b"\0", len(msg) + 1)
                return 1

        self._tramp = TRACE_FN(tramp)
        self._free = FREE_FN(lambda p: None)
        h = ctypes.c_void_p()
        check(load().shlo_compile(self._tramp, None, self._free, 1 if enable else 0, ctypes.byref(h)))
        self.h = h.value

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            try:
                load().shlo_fn_free(h)
            except Exception:
                pass
            self.h = None


def compile_(f: Callable, enable: bool) -> Fn:
    return Fn(f, enable)


def apply(fn: Fn, inputs: Sequence[Arr], max_outputs: int = 64) -> list:
    L = load()
    hs = (c_arr * max(len(inputs), 1))(*[a.h for a in inputs])
    outs = (c_arr * max_outputs)()
    n = ctypes.c_int()
    check(L.shlo_apply(fn.h, hs, len(inputs), outs, ctypes.byref(n), max_outputs))
    return [Arr(outs[i]) for i in range(n.value)]


def libm_erff_range(base: int, count: int) -> bytes:
    out = np.empty(count, dtype=np.uint32)
    check(load().shlo_libm_erff_range(base, count, out.ctypes.data_as(ctypes.c_void_p)))
    return out.tobytes()


def count_nonzero(a: Arr) -> int:
    c = ctypes.c_uint64()
    check(load().shlo_count_nonzero(a.h, ctypes.byref(c)))
    return c.value


def set_device(d: int) -> None:
    check(load().shlo_set_device(d))


def device_count() -> int:
    n = ctypes.c_int()
    check(load().shlo_device_count(ctypes.byref(n)))
    return n.value


def current_stream() -> int:
    """The cudaStream_t (as an integer) the current device's work is queued on."""
    s = ctypes.c_void_p()
    check(load().shlo_current_stream(ctypes.byref(s)))
    return s.value or 0


def launch_count() -> int:
    c = ctypes.c_uint64()
    check(load().shlo_launch_count(ctypes.byref(c)))
    return c.value


def device_ptr(a: Arr) -> tuple:
    """(device address, device) of a row-contiguous array's first element."""
    p, d = ctypes.c_void_p(), ctypes.c_int()
    check(load().shlo_device_ptr(a.h, ctypes.byref(p), ctypes.byref(d)))
    return p.value or 0, d.value


def set_flavor(flavor: str) -> None:
    check(load().shlo_set_flavor({"pinned": 0, "stock": 1}[flavor]))


# ---- byte helpers (Mlx.lean:110-135) ----

def words_to_bytes(ws: Sequence[int]) -> bytes:
    return np.asarray([w & 0xFFFFFFFF for w in ws], dtype="<u4").tobytes()


def u32_arr(ws: Sequence[int]) -> Arr:
    return of_bytes(words_to_bytes(ws), [len(ws)], dtU32)


def words64_to_bytes(ws: Sequence[int]) -> bytes:
    return np.asarray([w & 0xFFFFFFFFFFFFFFFF for w in ws], dtype="<u8").tobytes()


def u64_scalar(w: int) -> Arr:
    return of_bytes(words64_to_bytes([w]), [], dtU64)


def f32_scalar(bits: int) -> Arr:
    return of_bytes(words_to_bytes([bits]), [], dtF32)
