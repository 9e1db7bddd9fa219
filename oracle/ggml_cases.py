"""The 38 one-op ggml cases of ref/ggml_ref.c:243-283 -- TEST INFRASTRUCTURE ONLY.

Each case regenerates its inputs exactly as ggml_ref does (splitmix32 with the
case's seed, ``unif(a)`` per input in order; ref/ggml_ref.c:38-43, 152-239) and
computes the oracle output. Shapes are ggml ``ne`` (fastest first): a tensor
``ne = [n0, n1, n2]`` is row-major data of shape ``[n2, n1, n0]``.

The SHA-256 of every input and output is pinned by the reference
(evidence/ref-{stock,pinned}.sha256, copied to tests/golden/).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import oracle as O

SQRT_2_INV_BITS = 0x3F3504F3


@dataclass
class Case:
    name: str
    op: str
    seed: int
    ins: list            # [(ne, amplitude)], drawn in this order
    extra: dict = field(default_factory=dict)
    out_ne: tuple = ()

    def inputs(self):
        s = O.Stream(self.seed)
        arrs = []
        for ne, a in self.ins:
            n = int(np.prod(ne))
            arrs.append(s.unif(a, n).reshape(tuple(reversed(ne))))
        return arrs


def _mm(name, k, m, r, b, aw, ax):
    return Case(name, "mul_mat", 1, [((k, m, 1), aw), ((k, r, b), ax)], {"K": k, "M": m, "R": r, "B": b},
                (m, r, b))


def _add(name, a0, a1, a2):
    return Case(name, "add", 2, [((a0, a1, a2), 4.0), ((a0, a1, a2), 4.0)], {}, (a0, a1, a2))


def _mul(name, a0, a1, a2):
    return Case(name, "mul", 3, [((a0, a1, a2), 4.0), ((a0, a1, a2), 4.0)], {}, (a0, a1, a2))


def _repeat(name, a0, a1, a2):
    return Case(name, "repeat", 4, [((a0, 1, 1), 1.0)], {"to": (a0, a1, a2)}, (a0, a1, a2))


def _norm(name, a0, a1, a2):
    return Case(name, "norm", 5, [((a0, a1, a2), 3.0)], {"eps_bits": 0x3727C5AC}, (a0, a1, a2))


def _scale(name, a0, a1):
    return Case(name, "scale", 6, [((a0, a1, 1), 40.0)], {}, (a0, a1, 1))


def _soft_max(name, a0, a1, a):
    return Case(name, "soft_max", 7, [((a0, a1, 1), a)], {"scale_bits": 0x3F800000}, (a0, a1, 1))


def _gelu(name, a0, a1, a2):
    return Case(name, "gelu_erf", 8, [((a0, a1, a2), 6.0)], {}, (a0, a1, a2))


def _silu(name, a0, a1, a2):
    return Case(name, "silu", 9, [((a0, a1, a2), 12.0)], {}, (a0, a1, a2))


def _concat(name, dim, a0, a1, a2, b):
    bn = [a0, a1, a2]
    bn[dim] = b
    on = [a0, a1, a2]
    on[dim] += b
    return Case(name, "concat%d" % dim, 10, [((a0, a1, a2), 1.0), (tuple(bn), 1.0)], {"dim": dim}, tuple(on))


def _transpose(name, a0, a1):
    return Case(name, "transpose", 11, [((a0, a1, 1), 1.0)], {}, (a1, a0, 1))


def _view(name, w, seq, hw, off):
    return Case(name, "view", 12, [((w, seq, 1), 1.0)], {"off": off, "hw": hw}, (hw, seq, 1))


CASES = [
    _mm("mul_mat_small", 37, 5, 3, 1, 1.0, 1.0),
    _mm("mul_mat_k2", 2, 7, 1, 3, 1.0, 1.0),
    _add("add_small", 7, 3, 2),
    _mul("mul_small", 7, 3, 2),
    _repeat("repeat_small", 7, 3, 2),
    _norm("norm_small", 37, 3, 1),
    _scale("scale_small", 13, 4),
    _soft_max("soft_max_small", 16, 4, 30.0),
    _soft_max("soft_max_tail", 13, 4, 30.0),
    _gelu("gelu_erf_small", 64, 4, 1),
    _silu("silu_small", 16, 2, 1),
    _silu("silu_tail", 7, 2, 1),
    _concat("concat0_small", 0, 5, 3, 2, 4),
    _concat("concat1_small", 1, 5, 3, 2, 4),
    _concat("concat2_small", 2, 5, 3, 2, 4),
    _transpose("transpose_small", 5, 3),
    _view("view_small", 24, 3, 4, 8),
    _mm("mul_mat_qkv", 1024, 3072, 352, 3, 0.05, 2.0),
    _mm("mul_mat_ffn2", 2048, 1024, 352, 3, 0.05, 2.0),
    _mm("mul_mat_text", 4096, 1024, 50, 3, 0.05, 2.0),
    _mm("mul_mat_heading", 2, 1024, 1, 3, 0.5, 1.0),
    _mm("mul_mat_root_in", 738, 1024, 300, 3, 0.05, 2.0),
    _mm("mul_mat_body_in", 737, 1024, 300, 3, 0.05, 2.0),
    _mm("mul_mat_scores", 128, 352, 352, 1, 2.0, 2.0),
    _mm("mul_mat_value", 352, 128, 352, 1, 0.01, 2.0),
    _add("add_kimodo", 3072, 352, 3),
    _mul("mul_kimodo", 1024, 352, 3),
    _repeat("repeat_kimodo", 1024, 352, 3),
    _norm("norm_kimodo", 1024, 352, 3),
    _scale("scale_kimodo", 352, 352),
    _soft_max("soft_max_kimodo", 352, 352, 30.0),
    _gelu("gelu_erf_kimodo", 2048, 352, 3),
    _silu("silu_kimodo", 1024, 1, 3),
    _concat("concat0_kimodo", 0, 896, 352, 1, 128),
    _concat("concat1_kimodo", 1, 1024, 52, 3, 300),
    _concat("concat2_kimodo", 2, 1024, 352, 2, 1),
    _transpose("transpose_kimodo", 128, 352),
    _view("view_kimodo", 3072, 352, 128, 1024 + 3 * 128),
]

BY_NAME = {c.name: c for c in CASES}


def f32_from_bits(b: int) -> float:
    return float(np.array([b], dtype=np.uint32).view(np.float32)[0])


def scale_value() -> np.float32:
    """ggml_ref.c:193: 1.f / sqrtf(128.0f), both binary32 operations."""
    return np.float32(1.0) / np.sqrt(np.float32(128.0))


def oracle_output(c: Case, ins, flavour=O.PINNED) -> np.ndarray:
    """The ggml-cpu output of case `c`, row-major, float32."""
    if c.op == "mul_mat":
        w, x = ins
        K, M, R, B = c.extra["K"], c.extra["M"], c.extra["R"], c.extra["B"]
        return O.mul_mat(w, x, K, M, R * B, R * B, 0, flavour)
    if c.op == "add":
        return (ins[0] + ins[1]).reshape(-1)
    if c.op == "mul":
        return (ins[0] * ins[1]).reshape(-1)
    if c.op == "repeat":
        a0, a1, a2 = c.extra["to"]
        return np.broadcast_to(ins[0].reshape(1, 1, a0), (a2, a1, a0)).reshape(-1).copy()
    if c.op == "norm":
        x = ins[0]
        n = x.shape[-1]
        return O.norm(x, n, x.size // n, f32_from_bits(c.extra["eps_bits"]))
    if c.op == "scale":
        return (ins[0] * scale_value()).reshape(-1)
    if c.op == "soft_max":
        x = ins[0]
        n = x.shape[-1]
        return O.soft_max(x, n, x.size // n, 1.0)
    if c.op == "gelu_erf":
        return O.gelu_erf(ins[0])
    if c.op == "silu":
        x = ins[0]
        n = x.shape[-1]
        return O.silu(x, n, x.size // n)
    if c.op.startswith("concat"):
        d = c.extra["dim"]
        return np.concatenate([ins[0], ins[1]], axis=2 - d).reshape(-1)
    if c.op == "transpose":
        return ins[0].reshape(ins[0].shape[1], ins[0].shape[2]).T.copy().reshape(-1)
    if c.op == "view":
        x = ins[0]
        off, hw = c.extra["off"], c.extra["hw"]
        return x[0, :, off:off + hw].copy().reshape(-1)
    raise ValueError(c.op)


def expected_diverges(c: Case, flavour) -> str | None:
    """Cases whose ggml-cpu output this oracle does not reproduce, and why."""
    if flavour == O.STOCK and c.name == "gelu_erf_kimodo":
        return "stock links Apple libsystem_m erff, which is not carried (correctly rounded erff differs)"
    return None
