"""The denoiser / encoder-layer workload on the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The same computation as shlo.denoiser's StableHLO module, decomposed exactly
as StablehloMlx/Lower.lean lowers it (dot_general -> transpose/reshape ->
ggml_vec_dot_f32 order, Lower.lean:157-182; the ggml.* composites,
:475-494; add/multiply as single IEEE roundings), with the oracle's ggml
kernels and numpy's binary32 add/multiply. Used by the parity tests and as the
CPU baseline of bench.py.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def _f32(bits: int) -> float:
    return float(np.array([bits], np.uint32).view(np.float32)[0])


def dense(x2d, W, b, nthreads=None):
    R, K = x2d.shape
    M = W.shape[0]
    y = O.mul_mat(W, x2d, K, M, R, R, 0, O.PINNED, nthreads).reshape(R, M)
    return (y + b[None, :]).astype(np.float32)


def layer_norm(h2d, g, b, eps_bits, nthreads=None):
    R, D = h2d.shape
    n = O.norm(h2d, D, R, _f32(eps_bits), nthreads).reshape(R, D)
    return ((n * g[None, :]).astype(np.float32) + b[None, :]).astype(np.float32)


def encoder_layer(h, w, cfg, li, nthreads=None):
    B, S, D = h.shape
    H, Dh, F = cfg.heads, cfg.dh, cfg.ffn
    p = "l%d_" % li
    a = layer_norm(h.reshape(B * S, D), w[p + "g1"], w[p + "b1"], 0x3727C5AC, nthreads)
    qkv = dense(a, w[p + "wqkv"], w["b_" + p + "wqkv"], nthreads).reshape(B, S, 3, H, Dh)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    a2 = np.ascontiguousarray(q.transpose(0, 2, 1, 3)).reshape(B * H * S, Dh)
    b2 = np.ascontiguousarray(k.transpose(0, 2, 1, 3)).reshape(B * H * S, Dh)
    s = O.mul_mat(b2, a2, Dh, S, B * H * S, S, S * Dh, O.PINNED, nthreads)
    pr = O.soft_max(s, S, B * H * S, _f32(cfg.scale_bits()), nthreads)
    bv = np.ascontiguousarray(v.transpose(0, 2, 3, 1)).reshape(B * H * Dh, S)
    o = O.mul_mat(bv, pr.reshape(B * H * S, S), S, Dh, B * H * S, S, Dh * S, O.PINNED, nthreads)
    om = np.ascontiguousarray(o.reshape(B, H, S, Dh).transpose(0, 2, 1, 3)).reshape(B * S, D)
    h = (h.reshape(B * S, D) + dense(om, w[p + "wo"], w["b_" + p + "wo"], nthreads)).astype(np.float32)
    a2n = layer_norm(h, w[p + "g2"], w[p + "b2"], 0x3727C5AC, nthreads)
    f1 = dense(a2n, w[p + "w1"], w["b_" + p + "w1"], nthreads)
    g = O.gelu_erf(f1, nthreads).reshape(B * S, F)
    f2 = dense(g, w[p + "w2"], w["b_" + p + "w2"], nthreads)
    return (h + f2).astype(np.float32).reshape(B, S, D)


def forward(cfg, w, ins, nthreads=None, layers=None):
    """The module's @main on the oracle; `layers` limits the layer count (for a
    bounded CPU sample)."""
    x = ins[0]
    B, S, D = x.shape
    h = x
    if cfg.timestep:
        temb = ins[1]
        t1 = dense(temb, w["wt1"], w["b_wt1"], nthreads)
        t1 = O.silu(t1, D, B).reshape(B, D)
        t2 = dense(t1, w["wt2"], w["b_wt2"], nthreads)
        h = (x + t2[:, None, :]).astype(np.float32)
    for li in range(cfg.layers if layers is None else layers):
        h = encoder_layer(h, w, cfg, li, nthreads)
    return h
