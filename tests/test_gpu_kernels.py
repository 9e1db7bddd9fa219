"""The exact kernels against the oracle on the B200, bit for bit, beyond the
ggml fixture shapes: odd sizes, batches, signed zeros, infinities, NaN
payloads and both ggml builds. Every call goes through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from shlo import mlx as M  # noqa: E402
from shlo import run as Run  # noqa: E402


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32).reshape(-1)


def assert_bits(got, want, what=""):
    g, w = bits(got), bits(want)
    assert g.size == w.size, (what, g.size, w.size)
    bad = np.nonzero(g != w)[0]
    assert bad.size == 0, "%s: %d of %d differ, first at %d: got %08x want %08x" % (
        what, bad.size, g.size, bad[0], g[bad[0]], w[bad[0]])


@pytest.fixture(autouse=True)
def _pinned():
    M.set_flavor("pinned")
    yield
    M.set_flavor("pinned")


MM_SHAPES = [  # K, M, R, N, batched
    (16, 1, 1, 1, False), (17, 3, 5, 5, False), (32, 128, 64, 64, False), (48, 130, 70, 70, False),
    (64, 256, 256, 256, True), (100, 64, 33, 11, True), (196, 196, 392, 196, True), (256, 64, 512, 256, True),
    (352, 128, 352, 352, False), (512, 1536, 300, 300, False), (737, 1024, 40, 40, False), (2048, 512, 129, 129, False),
    (4096, 64, 16, 16, False), (80, 33, 200, 50, True), (64, 40, 700, 700, False), (192, 64, 1300, 650, True),
    # segments that do not span whole stages (the fold after groups of 4 k) in
    # eighths, and a batched narrow-M product in sixteenths
    (389, 200, 96, 96, False), (643, 130, 64, 64, False), (1024, 64, 128, 64, True),
]


@pytest.mark.parametrize("flavor", ["pinned", "stock"])
@pytest.mark.parametrize("path", ["fast", "naive", "seg", "fast-split1", "fast-split2", "fast-split4", "fast-split8",
                                  "fast-split16"])
@pytest.mark.parametrize("K,Mm,R,N,batched", MM_SHAPES)
def test_mul_mat_random(K, Mm, R, N, batched, path, flavor, monkeypatch):
    # the fast path in one CTA a tile, or in two or four (halves, quarters of the fold tree)
    monkeypatch.setenv("SHLO_MUL_MAT_PATH", path.split("-")[0])
    if "-split" in path:
        monkeypatch.setenv("SHLO_MM_SPLIT", path.split("split")[1])
    M.set_flavor(flavor)
    rng = np.random.default_rng(K * 7919 + Mm * 31 + R)
    nb = R // N
    wb = nb if batched else 1
    w = rng.standard_normal((wb, Mm, K)).astype(np.float32)
    x = rng.standard_normal((R, K)).astype(np.float32)
    wbs = Mm * K if batched else 0
    got = M.to_numpy(Run.mul_mat(M.of_numpy(w), M.of_numpy(x), K, Mm, R, N, wbs))
    want = O.mul_mat(w, x, K, Mm, R, N, wbs, O.PINNED if flavor == "pinned" else O.STOCK)
    assert_bits(got, want, "mul_mat K=%d M=%d R=%d N=%d" % (K, Mm, R, N))


@pytest.mark.parametrize("path", ["fast", "naive", "seg"])
def test_mul_mat_signed_zeros_and_specials(path, monkeypatch):
    """Chains that end at -0, products that underflow, infinities: the padded
    segments and the tree must keep every sign and special value."""
    monkeypatch.setenv("SHLO_MUL_MAT_PATH", path)
    rng = np.random.default_rng(3)
    K, Mm, R = 200, 96, 80
    w = rng.standard_normal((Mm, K)).astype(np.float32)
    x = rng.standard_normal((R, K)).astype(np.float32)
    w[rng.random(w.shape) < 0.7] = 0.0
    w[rng.random(w.shape) < 0.2] = -0.0
    x[rng.random(x.shape) < 0.3] = -0.0
    tiny = rng.random(w.shape) < 0.1
    w[tiny] = np.float32(-1e-30)
    x[:, :7] = np.float32(1e-20)
    w[5, :] = np.float32(-1e-30)  # every product of row 5 and input 7 rounds to -0: the output is -0
    x[7, :] = np.float32(1e-30)
    w[9, 3] = np.inf
    x[11, 40] = -np.inf
    got = M.to_numpy(Run.mul_mat(M.of_numpy(w), M.of_numpy(x), K, Mm, R, R, 0))
    want = O.mul_mat(w, x, K, Mm, R, R, 0, O.PINNED)
    assert_bits(got, want, "mul_mat specials")  # invalid products give arm64's default NaN in both
    assert np.count_nonzero(bits(got) == 0x80000000) > 0  # some outputs are -0
    assert np.count_nonzero(np.isnan(got)) > 0


def softmax_config2(seed=0):
    """[512,1024], N(0, sd 2), 5% -inf, row 0 near 88."""
    st = O.Stream(seed)
    n = 512 * 1024
    u1 = (st.unif(1.0, n).astype(np.float64) + 1.0) / 2.0
    u2 = (st.unif(1.0, n).astype(np.float64) + 1.0) / 2.0
    z = np.sqrt(-2.0 * np.log(np.maximum(u1, 1e-300))) * np.cos(2 * np.pi * u2)
    x = (2.0 * z).astype(np.float32).reshape(512, 1024)
    mask = O.Stream(seed + 1).unif(1.0, n).reshape(512, 1024)
    x[(mask + 1.0) / 2.0 < 0.05] = -np.inf
    x[0] = np.float32(88.0) + O.Stream(seed + 2).unif(0.5, 1024)
    for r in range(512):
        if np.all(np.isinf(x[r])):
            x[r, 0] = 0.0
    return x


@pytest.mark.parametrize("shape", [(512, 1024), (4, 16), (7, 4), (100, 256), (3, 4100), (1, 8192), (2000, 196 * 0 + 200)])
def test_soft_max(shape):
    rows, ncols = shape
    if shape == (512, 1024):
        x = softmax_config2()
    else:
        rng = np.random.default_rng(ncols + rows)
        x = (rng.standard_normal((rows, ncols)) * 5).astype(np.float32)
        x[rng.random(x.shape) < 0.05] = -np.inf
        x[:, 0] = 1.0
    for scale in (0x3F800000, 0x3E000000):
        sc = float(np.array([scale], np.uint32).view(np.float32)[0])
        got = M.to_numpy(Run.soft_max(M.of_numpy(x), ncols, rows, scale))
        want = O.soft_max(x, ncols, rows, sc)
        assert_bits(got, want, "soft_max %s scale %08x" % (shape, scale))


@pytest.mark.parametrize("ncols", [256, 1024, 2048, 100])
@pytest.mark.parametrize("amp", [0.05, 1.0, 3.0, 40.0])
def test_soft_max_binade_spans(ncols, amp):
    # small amplitudes keep a row's group sums within a few binades (added in any
    # order), large ones spread them (the serial chain); rows of -inf, zeros,
    # equal values, a NaN and an infinity mixed in
    rng = np.random.default_rng(ncols * 7 + int(amp * 100))
    x = (rng.standard_normal((40, ncols)) * amp).astype(np.float32)
    x[1] = 0.0
    x[2] = np.float32(3.5)
    x[3, rng.integers(0, ncols, 10)] = -np.inf
    x[4, 5] = np.nan
    x[5, 7] = np.inf
    x[6, :] = -np.inf
    x[6, 3] = 0.0
    got = M.to_numpy(Run.soft_max(M.of_numpy(x), ncols, 40, 0x3F800000))
    want = O.soft_max(x, ncols, 40, 1.0)
    assert_bits(got, want, "soft_max spans %d %g" % (ncols, amp))


def test_soft_max_refuses_tail():
    x = M.of_numpy(np.zeros((2, 13), np.float32))
    with pytest.raises(M.ShloError, match="not carried"):
        Run.soft_max(x, 13, 2, 0x3F800000)


@pytest.mark.parametrize("shape", [(1, 1), (3, 37), (5, 4), (33, 512), (70, 1024), (1056, 1024), (2, 1100), (64, 7)])
def test_norm(shape):
    rows, ncols = shape
    rng = np.random.default_rng(rows * 1000 + ncols)
    x = (rng.standard_normal((rows, ncols)) * 3 + 0.5).astype(np.float32)
    got = M.to_numpy(Run.norm(M.of_numpy(x), ncols, rows, 0x3727C5AC))
    want = O.norm(x, ncols, rows, float(np.array([0x3727C5AC], np.uint32).view(np.float32)[0]))
    assert_bits(got, want, "norm %s" % (shape,))


@pytest.mark.parametrize("ncols", [512, 1024, 36])
def test_norm_wide_and_narrow_ranges(ncols):
    # rows whose terms span few binades (the sums may be added in any order),
    # rows just past that span, rows of many binades, zeros and signed zeros,
    # and rows with an infinity or a NaN (the serial chains)
    rng = np.random.default_rng(ncols)
    rows = []
    for kind in range(12):
        r = (rng.standard_normal(ncols) * 2).astype(np.float32)
        if kind == 1:
            r[rng.integers(0, ncols, 3)] = np.float32(1e-6)   # about 20 binades below the rest
        elif kind == 2:
            r[rng.integers(0, ncols, 3)] = np.float32(3e-8)   # past the span: serial
        elif kind == 3:
            r = (rng.standard_normal(ncols) * np.float32(2.0) ** rng.integers(-60, 60, ncols)).astype(np.float32)
        elif kind == 4:
            r[:] = 0.0
            r[::3] = -0.0
        elif kind == 5:
            r[rng.integers(0, ncols)] = np.inf
        elif kind == 6:
            r[rng.integers(0, ncols)] = np.nan
        elif kind == 7:
            r[:] = np.float32(1e-41)  # subnormals
            r[0] = np.float32(1.0)
        elif kind == 8:
            r = np.full(ncols, np.float32(7.25))
        elif kind == 9:
            r[rng.integers(0, ncols, 5)] = np.float32(3e37)
        rows.append(r)
    x = np.stack(rows).astype(np.float32)
    eps = 0x3727C5AC
    got = M.to_numpy(Run.norm(M.of_numpy(x), ncols, x.shape[0], eps))
    want = O.norm(x, ncols, x.shape[0], float(np.array([eps], np.uint32).view(np.float32)[0]))
    assert_bits(got, want, "norm ranges %d" % ncols)


def specials32(n=1 << 16, seed=1):
    rng = np.random.default_rng(seed)
    s = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    extra = np.array([0, 0x80000000, 1, 0x80000001, 0x7F7FFFFF, 0xFF7FFFFF, 0x7F800000, 0xFF800000, 0x7FC00000,
                      0x7F800001, 0xFFC01234, 0x7FA00000, 0x00800000, 0x3F800000, 0xBF800000, 0x42B00000,
                      0xC2B00000, 0x40800000, 0xC0800000], dtype=np.uint32)
    return np.concatenate([s, extra])


def test_silu_and_gelu():
    xb = specials32()
    x = xb.view(np.float32)
    x = x[: (x.size // 4) * 4]
    got = M.to_numpy(Run.silu(M.of_numpy(x), x.size))
    assert_bits(got, O.silu(x, x.size, 1), "silu")
    xg = xb.view(np.float32)
    got = M.to_numpy(Run.gelu_erf(M.of_numpy(xg), xg.size))
    want = O.gelu_erf(xg)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    # gelu_erf spells out the NaN rule: payloads match too; non-NaN bit for bit
    assert_bits(got, want, "gelu_erf")


@pytest.mark.parametrize("tail", [0, 1, 4, 5, 7])
def test_gelu_polynomial_range(tail):
    """gelu_erf where erff runs its polynomials (|x| / sqrt(2) below 4): a
    strided sweep of every binade from 2^-40 to 6.5 on both signs (both
    polynomial forms, the rows' edges, the slow path's rare inputs by chance),
    the FFN's own N(0, 0.45) values, and lengths whose last values take the
    one-float4 and scalar tails; bit for bit against the oracle."""
    lo, hi = 0x2B800000, 0x40D00000
    sweep = np.arange(lo, hi, 97, dtype=np.uint32)
    pos = sweep.view(np.float32)
    rng = np.random.default_rng(11)
    x = np.concatenate([pos, -pos, (rng.standard_normal(1 << 20) * 0.45).astype(np.float32)])
    x = x[: (x.size // 8) * 8 + tail] if tail else x[: (x.size // 8) * 8 - 8]
    got = M.to_numpy(Run.gelu_erf(M.of_numpy(x), x.size))
    assert_bits(got, O.gelu_erf(x), "gelu_erf tail %d" % tail)
    small = x[: 8 + tail]
    assert_bits(M.to_numpy(Run.gelu_erf(M.of_numpy(small), small.size)), O.gelu_erf(small), "gelu_erf small")


def test_gelu_stock_is_refused():
    M.set_flavor("stock")
    with pytest.raises(M.ShloError, match="not carried"):
        Run.gelu_erf(M.of_numpy(np.ones(8, np.float32)), 8)


def test_divide_sqrt_specials():
    a = specials32(1 << 16, 2)
    b = specials32(1 << 16, 3)
    got = M.to_numpy(Run.divide(M.of_numpy(a.view(np.float32)), M.of_numpy(b.view(np.float32)), a.size))
    assert_bits(got, O.f32_div(a.view(np.float32), b.view(np.float32)), "divide")
    got = M.to_numpy(Run.sqrt(M.of_numpy(a.view(np.float32)), a.size))
    assert_bits(got, O.f32_sqrt(a.view(np.float32)), "sqrt")


def specials64(n=1 << 15, seed=4):
    rng = np.random.default_rng(seed)
    s = rng.integers(0, 2**64, n, dtype=np.uint64)
    vals = rng.standard_normal(n // 4) * 10.0 ** rng.integers(-5, 20, n // 4)
    extra = np.array([0, 1 << 63, 1, 0x7FEFFFFFFFFFFFFF, 0x7FF0000000000000, 0xFFF0000000000000, 0x7FF8000000000000,
                      0x7FF0000000000123, 0xFFF4000000000001, 0x000FFFFFFFFFFFFF, 0x43E0000000000000,
                      0xC3E0000000000000, 0x43DFFFFFFFFFFFFF, 0xC3E0000000000001], dtype=np.uint64)
    return np.concatenate([s, vals.view(np.uint64), np.floor(vals).view(np.uint64), extra])


@pytest.mark.parametrize("op", range(6))
def test_f64_ew(op):
    a = specials64(seed=5)
    b = np.roll(specials64(seed=6), 3)
    got = M.to_numpy(Run.f64_ew(op, M.of_numpy(a), M.of_numpy(b), a.size))
    want = O.f64_ew(op, a, b)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:5]


def test_f64_conversions():
    a32 = specials32(1 << 16, 8)
    got = M.to_numpy(Run.f64_of_f32(M.of_numpy(a32.view(np.float32)), a32.size))
    assert np.array_equal(got, O.f64_of_f32(a32.view(np.float32)))
    a64 = specials64(seed=9)
    got = M.to_numpy(Run.f32_of_f64(M.of_numpy(a64), a64.size))
    assert_bits(got, O.f32_of_f64(a64), "f32_of_f64")


@pytest.mark.parametrize("base", [0x00000000, 0x00700000, 0x3F000000, 0x40700000, 0x407C0000, 0x80000000,
                                  0xBF7F0000, 0x7F7F0000, 0x7FFF0000])
def test_erff_map_against_oracle(base):
    n = 1 << 18
    got = M.to_numpy(Run.erff_map(base, n))
    want = O.erff_range(base, n)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, "first at %08x: got %08x want %08x" % (base + bad[0], got[bad[0]], want[bad[0]])


def test_compile_and_apply():
    def f(args):
        return [M.binary(M.opAdd, args[0], args[1]), M.unary(M.opNeg, args[0])]
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    y = np.ones((3, 4), np.float32)
    for enable in (True, False):
        fn = M.compile_(f, enable)
        for _ in range(3):
            o = M.apply(fn, [M.of_numpy(x), M.of_numpy(y)])
            assert np.array_equal(M.to_numpy(o[0]), x + y)
            assert np.array_equal(M.to_numpy(o[1]), -x)


def test_builtins_against_numpy():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((4, 1, 5)).astype(np.float32)
    b = rng.standard_normal((3, 1)).astype(np.float32)
    A, B = M.of_numpy(a), M.of_numpy(b)
    for op, f in ((M.opAdd, np.add), (M.opSub, np.subtract), (M.opMul, np.multiply), (M.opMax, np.maximum),
                  (M.opMin, np.minimum)):
        assert_bits(M.to_numpy(M.binary(op, A, B)), f(a, b).astype(np.float32), "binary %d" % op)
    assert np.array_equal(M.to_numpy(M.binary(M.opLt, A, B)), a < b)
    ia = rng.integers(-50, 50, (6, 7)).astype(np.int32)
    ib = rng.integers(1, 9, (7,)).astype(np.int32)
    IA, IB = M.of_numpy(ia), M.of_numpy(ib)
    assert np.array_equal(M.to_numpy(M.binary(M.opRem, IA, IB)), np.remainder(ia, ib))
    assert np.array_equal(M.to_numpy(M.binary(M.opXor, IA, IB)), ia ^ ib)
    assert np.array_equal(M.to_numpy(M.binary(M.opShl, IA, IB)), ia << ib)
    u = rng.integers(0, 2**63, (5,), dtype=np.uint64)
    U = M.of_numpy(u)
    assert np.array_equal(M.to_numpy(M.binary(M.opShr, U, M.u64_scalar(63))), u >> np.uint64(63))
    t = M.transpose(M.of_numpy(ia), [1, 0])
    assert np.array_equal(M.to_numpy(t), ia.T)
    assert np.array_equal(M.to_numpy(M.reshape(t, [42])), ia.T.reshape(-1))
    s = M.slice_(M.of_numpy(ia), [1, 0], [6, 7], [2, 3])
    assert np.array_equal(M.to_numpy(s), ia[1:6:2, 0:7:3])
    c = M.concat([M.of_numpy(ia), M.of_numpy(ia * 2)], 1)
    assert np.array_equal(M.to_numpy(c), np.concatenate([ia, ia * 2], 1))
    idx = np.array([3, 0, 6, 9, -1], np.int64)
    tk = M.take(M.of_numpy(ia), M.of_numpy(idx), 1)
    assert np.array_equal(M.to_numpy(tk), ia[:, np.clip(np.where(idx < 0, idx + 7, idx), 0, 6)])
    assert np.array_equal(M.to_numpy(M.max_axis(M.of_numpy(ia), 0)), ia.max(0))
    assert M.count_nonzero(M.of_numpy(ia)) == np.count_nonzero(ia)
    assert np.array_equal(M.to_numpy(M.astype(M.of_numpy(a), M.dtI32)), a.astype(np.int32))
    assert np.array_equal(M.to_numpy(M.view(M.of_numpy(a), M.dtU32)), a.view(np.uint32))
    cond = a > 0
    w = M.where_(M.of_numpy(cond), M.of_numpy(a), M.f32_scalar(0))
    assert_bits(M.to_numpy(w), np.where(cond, a, np.float32(0)), "where")
    h = M.astype(M.of_numpy(a), M.dtF16)
    assert np.array_equal(M.to_numpy(h), a.astype(np.float16))
    bc = M.broadcast(M.of_numpy(b), [2, 3, 4])
    assert np.array_equal(M.to_numpy(bc), np.broadcast_to(b, (2, 3, 4)))


@pytest.mark.parametrize("bshape", [(6, 1, 8), (1, 5, 8), (6, 5, 1), (6, 1, 1), (1, 1, 8), (6, 5, 8)])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "max"])
def test_binary_three_axis_layouts(bshape, op):
    """f32 binary ops over [planes, rows, cols] with one operand broadcast along
    any axis or transposed (the 16-byte-access path), on both operand sides,
    against the same op over column-strided copies of the operands (the
    general strided path) bit for bit, and against numpy's IEEE results for
    the correctly rounded ops (MLX's divide is the GPU's approximate division,
    within 2 ulp)."""
    rng = np.random.default_rng(7)
    a = rng.standard_normal((6, 5, 8)).astype(np.float32)
    b = (rng.standard_normal(bshape) + 3.0).astype(np.float32)
    code = {"add": M.opAdd, "sub": M.opSub, "mul": M.opMul, "div": M.opDiv, "max": M.opMax}[op]
    f = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide, "max": np.maximum}[op]

    def strided(x):  # the same values at column stride 2
        w = np.zeros(x.shape[:-1] + (2 * x.shape[-1],), np.float32)
        w[..., ::2] = x
        nd = x.ndim
        return M.slice_(M.of_numpy(w), [0] * nd, list(w.shape), [1] * (nd - 1) + [2])

    at = np.ascontiguousarray(a.transpose(1, 0, 2))
    tv = M.transpose(M.of_numpy(at), [1, 0, 2])  # planes walked at a stride, columns contiguous
    for x, y, xm, ym, what in ((a, b, M.of_numpy(a), M.of_numpy(b), "a,b"), (b, a, M.of_numpy(b), M.of_numpy(a), "b,a"),
                               (a, b, tv, M.of_numpy(b), "at,b")):
        got = M.to_numpy(M.binary(code, xm, ym))
        ref = M.to_numpy(M.binary(code, strided(x), strided(y)))
        assert_bits(got, ref, "%s %s %s vs strided" % (op, what, bshape))
        with np.errstate(all="ignore"):
            want = f(x, y)
        if op == "div":
            assert np.all(np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64)) <= 2)
        else:
            assert_bits(got, want, "%s %s %s" % (op, what, bshape))
