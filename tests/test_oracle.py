"""The CPU oracle against the reference's own golden vectors (no GPU).

Every ggml_ref case (ref/ggml_ref.c:243-283) is regenerated and its inputs and
oracle outputs are hashed against evidence/ref-{stock,pinned}.sha256.
"""
import hashlib
import math
import struct

import numpy as np
import pytest

from oracle import ggml_cases as G
from oracle import oracle as O


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", G.CASES, ids=[c.name for c in G.CASES])
def test_inputs_match_pins(case, pins):
    ins = case.inputs()
    for i, a in enumerate(ins):
        key = "%s/in%d.f32" % (case.name, i)
        assert sha(a) == pins["pinned"][key] == pins["stock"][key]


@pytest.mark.parametrize("flavour", ["pinned", "stock"])
@pytest.mark.parametrize("case", G.CASES, ids=[c.name for c in G.CASES])
def test_outputs_match_pins(case, flavour, pins):
    fl = O.PINNED if flavour == "pinned" else O.STOCK
    out = G.oracle_output(case, case.inputs(), fl)
    got = sha(out.astype(np.float32))
    want = pins[flavour]["%s/out.f32" % case.name]
    why = G.expected_diverges(case, fl)
    if why:
        assert got != want, "expected divergence did not happen: " + why
    else:
        assert got == want


def f2b(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def b2f(b):
    return struct.unpack("<f", struct.pack("<I", b & 0xFFFFFFFF))[0]


def d2b(x):
    return struct.unpack("<Q", struct.pack("<d", x))[0]


def b2d(b):
    return struct.unpack("<d", struct.pack("<Q", b))[0]


def _specials32():
    s = [0, 0x80000000, 1, 0x80000001, 0x7F7FFFFF, 0xFF7FFFFF, 0x7F800000, 0xFF800000,
         0x7FC00000, 0x7F800001, 0xFFC01234, 0x00800000, 0x007FFFFF, 0x3F800000, 0xBF800000,
         0x40490FDB, 0x3F3504F3, 0x33800000, 0x4B000000]
    rng = np.random.default_rng(5)
    s += [int(v) for v in rng.integers(0, 2**32, 4000, dtype=np.uint64)]
    return s


def _specials64():
    s = [0, 1 << 63, 1, 0x7FEFFFFFFFFFFFFF, 0x7FF0000000000000, 0xFFF0000000000000,
         0x7FF8000000000000, 0x7FF0000000000123, 0xFFF4000000000001, 0x0010000000000000,
         0x000FFFFFFFFFFFFF, 0x3FF0000000000000, 0xBFF8000000000000, 0x4330000000000000,
         0x43E0000000000000, 0xC3E0000000000000, 0x43DFFFFFFFFFFFFF, 0x3FE0000000000000]
    rng = np.random.default_rng(7)
    s += [int(v) for v in rng.integers(0, 2**63, 3000, dtype=np.uint64)]
    s += [int(v) | (1 << 63) for v in rng.integers(0, 2**63, 1000, dtype=np.uint64)]
    # values near one another (cancellation) and near the integer grid
    base = rng.normal(size=500) * 1e3
    s += [d2b(float(v)) for v in base] + [d2b(float(v) * (1 + 1e-15)) for v in base]
    return s


def _ieee_nan_ok(got_bits, x_bits_list):
    return ((got_bits >> 52) & 0x7FF) == 0x7FF and (got_bits & 0xFFFFFFFFFFFFF) != 0


def test_soft_f64_matches_ieee_on_non_nan():
    """Soft binary64 (SoftFloat.lean restated) equals the host FPU's IEEE binary64."""
    s = np.array(_specials64(), dtype=np.uint64)
    rng = np.random.default_rng(3)
    a = s[rng.permutation(s.size)]
    b = s[rng.permutation(s.size)]
    with np.errstate(all="ignore"):
        fa, fb = a.view(np.float64), b.view(np.float64)
        natives = {0: fa + fb, 1: fa - fb, 2: fa * fb, 3: fa / fb, 4: np.floor(fa)}
    for op, want in natives.items():
        got = O.f64_ew(op, a, b)
        wbits = want.view(np.uint64)
        nan = np.isnan(want)
        assert np.array_equal(got[~nan], wbits[~nan]), op
        # NaN results: the first NaN operand quieted, else the default NaN.
        for i in np.nonzero(nan)[0]:
            ai, bi = int(a[i]), int(b[i])
            isn = lambda v: (v & 0x7FFFFFFFFFFFFFFF) > 0x7FF0000000000000
            if isn(ai):
                exp = ai | 0x8000000000000
            elif isn(bi) and op != 4:
                exp = bi | 0x8000000000000
            else:
                exp = 0x7FF8000000000000
            assert int(got[i]) == exp, (op, hex(ai), hex(bi), hex(int(got[i])))


def test_soft_f64_to_i64():
    s = _specials64()
    got = O.f64_ew(5, np.array(s, np.uint64), np.array(s, np.uint64))
    for v, g in zip(s, got):
        x = b2d(v)
        if math.isnan(x):
            want = 0
        elif x >= 2.0**63:
            want = 2**63 - 1
        elif x < -2.0**63:
            want = -2**63
        else:
            want = int(x)  # toward zero
        assert int(g) == want & 0xFFFFFFFFFFFFFFFF, hex(v)


def test_soft_conversions():
    s32 = np.array(_specials32(), dtype=np.uint32)
    wide = O.f64_of_f32(s32.view(np.float32))
    f = s32.view(np.float32)
    for b, w in zip(s32, wide):
        x = b2f(int(b))
        if math.isnan(x):
            assert int(w) == (((int(b) >> 31) << 63) | 0x7FF0000000000000 | ((int(b) & 0x7FFFFF) << 29))
        else:
            assert int(w) == d2b(x)
    s64 = np.array(_specials64(), dtype=np.uint64)
    nar = O.f32_of_f64(s64).view(np.uint32)
    with np.errstate(all="ignore"):
        want = s64.view(np.float64).astype(np.float32).view(np.uint32)
    nan = np.isnan(s64.view(np.float64))
    assert np.array_equal(nar[~nan], want[~nan])
    for v, g in zip(s64[nan], nar[nan]):
        v = int(v)
        assert int(g) == (((v >> 63) << 31) | 0x7FC00000 | ((v & 0xFFFFFFFFFFFFF) >> 29))
    del f


def test_soft_f32_div_sqrt():
    s = np.array(_specials32(), dtype=np.uint32)
    rng = np.random.default_rng(1)
    a, b = s, s[rng.permutation(s.size)]
    with np.errstate(all="ignore"):
        wd = (a.view(np.float32) / b.view(np.float32)).view(np.uint32)
        ws = np.sqrt(a.view(np.float32)).view(np.uint32)
    gd = O.f32_div(a.view(np.float32), b.view(np.float32)).view(np.uint32)
    gs = O.f32_sqrt(a.view(np.float32)).view(np.uint32)
    nd = np.isnan(wd.view(np.float32))
    ns = np.isnan(ws.view(np.float32))
    assert np.array_equal(gd[~nd], wd[~nd])
    assert np.array_equal(gs[~ns], ws[~ns])


def test_cr_erff_against_quad_sample():
    """The oracle's erff equals erf rounded from a 113-bit evaluation (mpmath-free spot check
    by monotonicity and known values) on a sample; exhaustive checks run on the GPU side."""
    L = O.lib()
    assert L.orc_erff_cr(0.0) == 0.0 and math.copysign(1, L.orc_erff_cr(-0.0)) < 0
    assert L.orc_erff_cr(10.0) == 1.0 and L.orc_erff_cr(-10.0) == -1.0
    assert L.orc_erff_cr(float("inf")) == 1.0
    xs = np.linspace(-4, 4, 20001, dtype=np.float32)
    ys = np.array([L.orc_erff_cr(float(v)) for v in xs], dtype=np.float32)
    assert np.all(np.diff(ys) >= 0)
    # within half an ulp of the double-precision erf
    ref = np.array([math.erf(float(v)) for v in xs])
    ulp = np.spacing(np.abs(ys)).astype(np.float64)
    assert np.all(np.abs(ys.astype(np.float64) - ref) <= 0.5 * ulp + 1e-300)
