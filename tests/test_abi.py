"""The C-ABI library loads without a GPU and exports every symbol the public
headers declare; its host-only entry points work on the CPU."""
import ctypes
import os
import re

import numpy as np

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    inc = os.path.join(ROOT, "include")
    for h in os.listdir(inc):
        if h.endswith(".h"):
            text = open(os.path.join(inc, h)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            syms |= set(re.findall(r"\b(shlo_\w+)\s*\(", text))
    return syms


def test_library_exports_every_declared_symbol():
    from shlo import _lib
    L = ctypes.CDLL(_lib.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 36
    missing = [s for s in sorted(syms) if not hasattr(L, s)]
    assert not missing, missing
    assert syms <= set(_lib.SYMBOLS) | {s for s in syms if s not in _lib.SYMBOLS and hasattr(L, s)}


def test_no_cuda_device_needed_to_load():
    import shlo  # noqa: F401  (loads the library)
    from shlo import mlx as M
    assert M.libm_erff_range(0x3F800000, 4)


def test_libm_erff_range_matches_oracle():
    """smlx_libm_erff_range's replacement: the host's correctly rounded erff."""
    from shlo import mlx as M
    for base in (0x00000000, 0x3E000000, 0x40700000, 0xBF800000, 0x7F7FFF00):
        got = np.frombuffer(M.libm_erff_range(base, 1 << 14), dtype=np.uint32)
        want = O.erff_range(base, 1 << 14)
        assert np.array_equal(got, want), hex(base)


def test_errors_are_reported_not_raised_as_faults():
    from shlo import mlx as M
    try:
        M.kernel_new("smlx_no_such_kernel", [], ["y"], "", "")
    except M.ShloError as e:
        assert "not carried" in str(e)
    else:
        raise AssertionError("unknown kernel accepted")


def test_traced_function_error_travels_back():
    """A trace error comes back as the apply error (c/smlx_shim.c:337-349), no GPU needed."""
    from shlo import mlx as M

    def f(args):
        raise M.ShloError("composite ggml.x: not carried")
    fn = M.compile_(f, True)
    try:
        M.apply(fn, [M.empty_arr()])
    except M.ShloError as e:
        assert "traced function" in str(e) and "not carried" in str(e)
    else:
        raise AssertionError("error swallowed")
