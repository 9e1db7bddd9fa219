"""Generate erf_poly.cuh: the tables of the binary64 erf on (0, 4).

    python contract-stablehlo-mlx_b200/csrc/gen_erf_poly.py > contract-stablehlo-mlx_b200/csrc/erf_poly.cuh

Pure Python (decimal arithmetic at 80 digits): erf comes from its Maclaurin
series, erf(x) = 2/sqrt(pi) * sum_n (-1)^n x^(2n+1) / (n! (2n+1)), exp from
the decimal module, and pi from Machin's formula. Nothing is taken from a
library's erf.

  * [0, 2^-8): erf(a) = a * g(a^2), g(s) = 2/sqrt(pi) * sum_n (-1)^n s^n / (n! (2n+1)),
    the series truncated at degree G_DEG (s < 2^-16, so the first omitted term
    is below 2^-90 relative).
  * [2^-8, 4): a Taylor expansion about the centre m_k = (2k+1)/512 of the row
    k = floor(256 a) (T_ROWS rows of width 1/256), in ds = 512 (a - m) in [-1, 1]:
        erf(m + d) = erf(m) + C_k * sum_{n=1..6} c_n(m) ds^n,
        c_n(m) = (-1)^(n-1) H_{n-1}(m) * 2^(-9n) / n!
    with C_k = 2/sqrt(pi) * exp(-m^2) (the n-th derivative of erf is
    2/sqrt(pi) (-1)^(n-1) H_{n-1}(x) exp(-x^2), H the Hermite polynomials). The
    table holds erf(m_k) and C_k rounded to binary64. c_1 = 2^-9 and
    c_2 = -2^-27 (2k+1) are exact; c_3 = K1 (2k+1)^2 + K0 is evaluated in binary64;
    c_4, c_5, c_6 (whose terms are below 2^-38) are polynomials in m evaluated in
    binary32 with the coefficients A4 .. C6 below.

The script prints the largest relative error of the two forms (table entries and
constants rounded to binary64, the rest evaluated exactly) against the series at
sample points of every row; the rounding test that uses them allows 2^-49 for
that error together with the binary64 evaluation.
"""
from __future__ import annotations

import math
import sys
from decimal import Decimal, getcontext
from fractions import Fraction

getcontext().prec = 80
G_DEG = 4
T_ROWS = 1024
SAMPLES = 8


def machin_pi() -> Decimal:
    def arctan_inv(n: int) -> Decimal:
        x = Decimal(1) / n
        x2 = x * x
        term, total, k = x, x, 1
        while True:
            term *= -x2
            t = term / (2 * k + 1)
            if abs(t) < Decimal(10) ** -(getcontext().prec + 2):
                return total
            total += t
            k += 1
    return 16 * arctan_inv(5) - 4 * arctan_inv(239)


PI = machin_pi()
TWO_OVER_SQRTPI = 2 / PI.sqrt()


def erf(x: Decimal) -> Decimal:
    x2 = x * x
    term = x  # x^(2n+1) / n!
    total = x
    n = 0
    eps = Decimal(10) ** -(getcontext().prec - 5)
    while True:
        n += 1
        term = term * x2 / n
        t = term / (2 * n + 1)
        total += -t if n % 2 else t
        if t < eps * abs(total):
            return TWO_OVER_SQRTPI * total


def dec(q: Fraction) -> Decimal:
    return Decimal(q.numerator) / Decimal(q.denominator)


def small_poly():
    out = []
    fact = 1
    for n in range(G_DEG + 1):
        if n:
            fact *= n
        v = TWO_OVER_SQRTPI / (fact * (2 * n + 1))
        out.append(float(-v if n % 2 else v))
    return out


def taylor_rows():
    rows = []
    for k in range(T_ROWS):
        m = Decimal(2 * k + 1) / 512
        rows.append((float(erf(m)), float(TWO_OVER_SQRTPI * (-(m * m)).exp())))
    return rows


def f32_nearest(q: Fraction) -> float:
    """q rounded to the nearest binary32 (returned as a Python float)."""
    import struct
    f = struct.unpack("<f", struct.pack("<f", float(q)))[0]
    bits = struct.unpack("<I", struct.pack("<f", f))[0]
    cands = [f] + [struct.unpack("<f", struct.pack("<I", b))[0] for b in (bits - 1, bits + 1)]
    return min(cands, key=lambda c: abs(Fraction(c) - q))


def R(n: int) -> Fraction:
    return Fraction(1, 512 ** n * math.factorial(n))


def consts():
    """The binary64 constants K0, K1 of c_3 and the binary32 coefficients of c_4..c_6."""
    r3 = float(R(3))
    d = {"K1": r3 * 2.0 ** -16, "K0": -2.0 * r3}
    exact = {"A4": -8 * R(4), "B4": 12 * R(4),
             "A5": 16 * R(5), "B5": -48 * R(5), "C5": 12 * R(5),
             "A6": -32 * R(6), "B6": 160 * R(6), "C6": -120 * R(6)}
    f = {k: f32_nearest(v) for k, v in exact.items()}
    return d, f


def taylor_exact(k: int, row, d, f, a: Fraction) -> Fraction:
    """The expansion with the rounded table entries and constants, evaluated exactly."""
    c = 2 * k + 1
    ds = 512 * a - c
    m = Fraction(c, 512)
    m2 = m * m
    F = {key: Fraction(v) for key, v in f.items()}
    c1 = Fraction(1, 512)
    c2 = Fraction(-c, 2 ** 27)
    c3 = Fraction(d["K1"]) * c * c + Fraction(d["K0"])
    c4 = m * (F["A4"] * m2 + F["B4"])
    c5 = (F["A5"] * m2 + F["B5"]) * m2 + F["C5"]
    c6 = m * ((F["A6"] * m2 + F["B6"]) * m2 + F["C6"])
    s = ds * (c1 + ds * (c2 + ds * (c3 + ds * (c4 + ds * (c5 + ds * c6)))))
    return Fraction(row[0]) + Fraction(row[1]) * s


def rel_err(approx: Fraction, true: Decimal) -> float:
    return float(abs(dec(approx) - true) / abs(true))


def max_rel_err_taylor(rows, d, f) -> float:
    worst = 0.0
    for k in range(1, T_ROWS):
        for i in range(SAMPLES + 1):
            a = Fraction(k * SAMPLES + i, 256 * SAMPLES)
            if i == SAMPLES:
                a -= Fraction(1, 2 ** 40)
            worst = max(worst, rel_err(taylor_exact(k, rows[k], d, f, a), erf(dec(a))))
    return worst


def max_rel_err_small(coefs) -> float:
    worst = 0.0
    for i in range(1, SAMPLES + 1):
        a = Fraction(i, 256 * SAMPLES)
        g = Fraction(0)
        for c in reversed(coefs):
            g = g * a * a + Fraction(c)
        worst = max(worst, rel_err(a * g, erf(dec(a))))
    return worst


def main():
    small = small_poly()
    rows = taylor_rows()
    d, f = consts()
    worst = max(max_rel_err_small(small), max_rel_err_taylor(rows, d, f))
    sys.stderr.write("max relative error of the rounded tables: %.3e (2^%.1f)\n" % (worst, math.log2(worst)))
    w = sys.stdout.write
    w("// Generated by gen_erf_poly.py (decimal arithmetic at 80 digits); do not edit.\n")
    w("// binary64 erf on (0, 4): erf(a) = a * g(a^2) on [0, 2^-8); on [2^-8, 4) a Taylor\n")
    w("// expansion about m_k = (2k+1)/512, k = floor(256 a), in ds = 512 (a - m_k):\n")
    w("// erf(m_k) + C_k * ds (c1 + ds (c2 + ds (c3 + ds (c4 + ds (c5 + ds c6))))), with\n")
    w("// erf(m_k) and C_k = 2/sqrt(pi) exp(-m_k^2) from the table.\n")
    w("// Largest relative error of the rounded tables and constants (exact evaluation): %.3e.\n" % worst)
    w("#pragma once\n\n")
    w("#define SHLO_ERF_G_DEG %d\n#define SHLO_ERF_T_ROWS %d\n\n" % (G_DEG, T_ROWS))
    w("#define SHLO_ERF_G_COEFS \\\n  {")
    w(", ".join(float.hex(c) for c in small))
    w("}\n\n")
    w("// c3 = K1 (2k+1)^2 + K0 (binary64).\n")
    for key in ("K1", "K0"):
        w("#define SHLO_ERF_%s %s\n" % (key, float.hex(d[key])))
    w("// c4 = m (A4 m^2 + B4), c5 = (A5 m^2 + B5) m^2 + C5, c6 = m ((A6 m^2 + B6) m^2 + C6) (binary32).\n")
    for key in ("A4", "B4", "A5", "B5", "C5", "A6", "B6", "C6"):
        w("#define SHLO_ERF_%s %sf\n" % (key, float.hex(f[key])))
    w("\n// Row k: {erf(m_k), 2/sqrt(pi) exp(-m_k^2)}, m_k = (2k+1)/512 (row 0 is not read).\n")
    w("#define SHLO_ERF_T_VALUES \\\n  {")
    body = ["    {%s, %s}" % (float.hex(e), float.hex(c)) for e, c in rows]
    w(" \\\n" + ", \\\n".join(body) + " \\\n  }\n")


if __name__ == "__main__":
    main()
