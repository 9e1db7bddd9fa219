"""The motion-denoiser workload as StableHLO: the transformer encoder layer and the
8-layer denoiser of the benchmark configurations, written as the generic-form
modules the executor runs (ggml.* custom calls for norm, soft_max, silu and
gelu_erf, dot_general for every matmul).

Architecture (pre-norm encoder layer, ggml's ops):
    a = norm(h) * g1 + b1                      ggml.norm, eps 0x3727C5AC (1e-5f)
    q, k, v = split(a @ Wqkv^T + bqkv)         heads H of width D/H
    p = soft_max(q k^T, scale 1/sqrt(D/H))     ggml.soft_max (scale attribute)
    h = h + merge(p v) @ Wo^T + bo
    a = norm(h) * g2 + b2
    h = h + gelu_erf(a @ W1^T + c1) @ W2^T + c2
The denoiser adds a timestep embedding -- a host-computed sinusoid (ggml uses
libm sinf/cosf/expf for it, which this backend does not carry) through
silu(t @ Wt1^T + bt1) @ Wt2^T + bt2, broadcast over the sequence -- to the
noisy input, then runs L layers. Weights are N(0, 0.02) (norm gains 1 + N(0,
0.02)), inputs N(0, 1), from a seeded generator: synthetic, random-init.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

EPS_BITS = 0x3727C5AC  # 1e-5f


@dataclass(frozen=True)
class Config:
    layers: int = 8
    seq: int = 256
    d: int = 512
    heads: int = 8
    ffn: int = 2048
    timestep: bool = True

    @property
    def dh(self) -> int:
        return self.d // self.heads

    def scale_bits(self) -> int:
        s = np.float32(1.0) / np.sqrt(np.float32(self.dh))
        return int(np.array([s], np.float32).view(np.uint32)[0])

    def flops_per_sample(self) -> int:
        """2*M*N*K per dot_general (an fma counts 2), all layers; the time MLP included."""
        S, D, F = self.seq, self.d, self.ffn
        per_layer = 2 * S * D * 3 * D + 2 * S * D * D + 2 * 2 * S * S * D + 2 * 2 * S * D * F
        t = 2 * 2 * D * D if self.timestep else 0
        return self.layers * per_layer + t


DENOISER = Config()
ENCODER = Config(layers=1, seq=196, timestep=False)


def T(*dims) -> str:
    return "tensor<" + "".join("%dx" % d for d in dims) + "f32>"


class _W:
    def __init__(self):
        self.lines = []
        self.n = 0

    def op(self, name, args, attrs, in_tys, out_ty):
        v = "%%v%d" % self.n
        self.n += 1
        a = (" {" + attrs + "}") if attrs else ""
        self.lines.append('    %s = "%s"(%s)%s : (%s) -> %s' % (v, name, ", ".join(args), a, ", ".join(in_tys), out_ty))
        return v


def _dense(w: _W, x, xt, wname, M, K, lead):
    """x [lead..., K] @ W[M, K]^T + b[M]."""
    out = T(*lead, M)
    dn = "dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [%d], rhs_contracting_dimensions = [1]>" % len(lead)
    y = w.op("stablehlo.dot_general", [x, "%" + wname], dn, [xt, T(M, K)], out)
    b = w.op("stablehlo.broadcast_in_dim", ["%b_" + wname], "broadcast_dimensions = array<i64: %d>" % len(lead),
             [T(M)], out)
    return w.op("stablehlo.add", [y, b], "", [out, out], out)


def _layer_norm(w: _W, h, ty, g, b, lead, D):
    n = w.op("stablehlo.custom_call", [h], 'call_target_name = "ggml.norm", backend_config = "eps = 0x%08X : f32"'
             % EPS_BITS, [ty], ty)
    gg = w.op("stablehlo.broadcast_in_dim", ["%" + g], "broadcast_dimensions = array<i64: %d>" % len(lead), [T(D)], ty)
    t = w.op("stablehlo.multiply", [n, gg], "", [ty, ty], ty)
    bb = w.op("stablehlo.broadcast_in_dim", ["%" + b], "broadcast_dimensions = array<i64: %d>" % len(lead), [T(D)], ty)
    return w.op("stablehlo.add", [t, bb], "", [ty, ty], ty)


def _encoder_layer(w: _W, h, cfg: Config, B: int, li: int):
    S, D, H, Dh, F = cfg.seq, cfg.d, cfg.heads, cfg.dh, cfg.ffn
    hty = T(B, S, D)
    p = "l%d_" % li
    a = _layer_norm(w, h, hty, p + "g1", p + "b1", (B, S), D)
    qkv = _dense(w, a, hty, p + "wqkv", 3 * D, D, (B, S))
    r5 = w.op("stablehlo.reshape", [qkv], "", [T(B, S, 3 * D)], T(B, S, 3, H, Dh))
    parts = []
    for i in range(3):
        sl = w.op("stablehlo.slice", [r5],
                  "start_indices = array<i64: 0, 0, %d, 0, 0>, limit_indices = array<i64: %d, %d, %d, %d, %d>, "
                  "strides = array<i64: 1, 1, 1, 1, 1>" % (i, B, S, i + 1, H, Dh), [T(B, S, 3, H, Dh)],
                  T(B, S, 1, H, Dh))
        parts.append(w.op("stablehlo.reshape", [sl], "", [T(B, S, 1, H, Dh)], T(B, S, H, Dh)))
    q, k, v = parts
    s = w.op("stablehlo.dot_general", [q, k],
             "dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 2], rhs_batching_dimensions = [0, 2], "
             "lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [3]>",
             [T(B, S, H, Dh), T(B, S, H, Dh)], T(B, H, S, S))
    pr = w.op("stablehlo.custom_call", [s], 'call_target_name = "ggml.soft_max", backend_config = "scale = 0x%08X : f32"'
              % cfg.scale_bits(), [T(B, H, S, S)], T(B, H, S, S))
    o = w.op("stablehlo.dot_general", [pr, v],
             "dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 1], rhs_batching_dimensions = [0, 2], "
             "lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [1]>",
             [T(B, H, S, S), T(B, S, H, Dh)], T(B, H, S, Dh))
    ot = w.op("stablehlo.transpose", [o], "permutation = array<i64: 0, 2, 1, 3>", [T(B, H, S, Dh)], T(B, S, H, Dh))
    om = w.op("stablehlo.reshape", [ot], "", [T(B, S, H, Dh)], hty)
    at = _dense(w, om, hty, p + "wo", D, D, (B, S))
    h = w.op("stablehlo.add", [h, at], "", [hty, hty], hty)
    a2 = _layer_norm(w, h, hty, p + "g2", p + "b2", (B, S), D)
    f1 = _dense(w, a2, hty, p + "w1", F, D, (B, S))
    g = w.op("stablehlo.custom_call", [f1], 'call_target_name = "ggml.gelu_erf", backend_config = ""', [T(B, S, F)],
             T(B, S, F))
    f2 = _dense(w, g, T(B, S, F), p + "w2", D, F, (B, S))
    return w.op("stablehlo.add", [h, f2], "", [hty, hty], hty)


def weight_specs(cfg: Config):
    """(name, shape) of every weight argument, in @main's order after the inputs."""
    D, F = cfg.d, cfg.ffn
    specs = []
    if cfg.timestep:
        specs += [("wt1", (D, D)), ("b_wt1", (D,)), ("wt2", (D, D)), ("b_wt2", (D,))]
    for li in range(cfg.layers):
        p = "l%d_" % li
        specs += [(p + "g1", (D,)), (p + "b1", (D,)), (p + "wqkv", (3 * D, D)), ("b_" + p + "wqkv", (3 * D,)),
                  (p + "wo", (D, D)), ("b_" + p + "wo", (D,)), (p + "g2", (D,)), (p + "b2", (D,)),
                  (p + "w1", (F, D)), ("b_" + p + "w1", (F,)), (p + "w2", (D, F)), ("b_" + p + "w2", (D,))]
    return specs


def module_text(cfg: Config, batch: int) -> str:
    """@main(%x [B,S,D], (%temb [B,D]), weights...) -> [B,S,D]."""
    B, S, D = batch, cfg.seq, cfg.d
    w = _W()
    args = ["%%x: %s" % T(B, S, D)]
    if cfg.timestep:
        args.append("%%temb: %s" % T(B, D))
    args += ["%%%s: %s" % (n, T(*shp)) for n, shp in weight_specs(cfg)]
    h = "%x"
    if cfg.timestep:
        t1 = _dense(w, "%temb", T(B, D), "wt1", D, D, (B,))
        t1s = w.op("stablehlo.custom_call", [t1], 'call_target_name = "ggml.silu", backend_config = ""', [T(B, D)], T(B, D))
        t2 = _dense(w, t1s, T(B, D), "wt2", D, D, (B,))
        tb = w.op("stablehlo.broadcast_in_dim", [t2], "broadcast_dimensions = array<i64: 0, 2>", [T(B, D)], T(B, S, D))
        h = w.op("stablehlo.add", [h, tb], "", [T(B, S, D), T(B, S, D)], T(B, S, D))
    for li in range(cfg.layers):
        h = _encoder_layer(w, h, cfg, B, li)
    head = "module {\n  func.func public @main(%s) -> (%s) {\n" % (", ".join(args), T(B, S, D))
    return head + "\n".join(w.lines) + "\n    func.return %s : %s\n  }\n}\n" % (h, T(B, S, D))


def init_weights(cfg: Config, seed: int = 1) -> dict:
    rng = np.random.default_rng(seed)
    out = {}
    for n, shp in weight_specs(cfg):
        v = rng.standard_normal(shp) * 0.02
        if n.endswith("g1") or n.endswith("g2"):
            v = v + 1.0
        out[n] = v.astype(np.float32)
    return out


def timestep_sinusoid(t: np.ndarray, d: int) -> np.ndarray:
    """The host-computed sinusoidal embedding of the diffusion timestep, [B, d]."""
    half = d // 2
    freq = np.exp(-np.log(10000.0) * np.arange(half) / half)
    ang = t[:, None].astype(np.float64) * freq[None, :]
    return np.concatenate([np.sin(ang), np.cos(ang)], axis=1).astype(np.float32)


def inputs(cfg: Config, batch: int, seed: int = 1):
    rng = np.random.default_rng(seed + 1000)
    x = rng.standard_normal((batch, cfg.seq, cfg.d)).astype(np.float32)
    ins = [x]
    if cfg.timestep:
        ins.append(timestep_sinusoid(rng.integers(0, 1000, batch), cfg.d))
    return ins
