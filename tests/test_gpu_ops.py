"""Every ggml case of Tests/OpTests.lean, on the B200, bit for bit.

For each case the module OpTests.lean builds is run through the replay
harness (shlo.exec -> shlo.lower -> the C ABI), compiled and uncompiled, and
the SHA-256 of the output words is compared with the reference's own pinned
hash (evidence/ref-pinned.sha256; tests/golden/). Then the case's planted wrong
lowering must give different bits or refuse (OpTests.lean:216-221), and the
cases ggml-cpu computes with code this backend does not carry must be refused
with "not carried" (OpTests.lean:196-201).
"""
import hashlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import optests as T  # noqa: E402
from oracle import ggml_cases as G  # noqa: E402
from oracle import oracle as O  # noqa: E402
from shlo import exec as E  # noqa: E402
from shlo import lower as L  # noqa: E402
from shlo import mlx as M  # noqa: E402


def run_module(text, ins, faults, compile):
    try:
        f = E.prepare(E.load(text), faults, compile)
        outs = E.call(f, ins)
        return "ok", M.to_bytes(outs[0])
    except M.ShloError as e:
        return "err", str(e)


def first_diff(got: bytes, want: np.ndarray) -> str:
    g = np.frombuffer(got, dtype=np.uint32)
    w = want.view(np.uint32).reshape(-1)
    if g.size != w.size:
        return "size %d vs %d" % (g.size, w.size)
    bad = np.nonzero(g != w)[0]
    if bad.size == 0:
        return "no word differs from the oracle"
    k = int(bad[0])
    return "%d of %d words differ, first at %d: got %s want %s" % (bad.size, g.size, k, T.hex32(int(g[k])),
                                                                   T.hex32(int(w[k])))


def case_module(oc, c):
    ins_ne = [ne for ne, _ in c.ins]
    if oc.op == "view":
        return T.view_module(ins_ne[0], c.out_ne, oc.view_offset)
    return T.module_for(oc.op, ins_ne, c.out_ne)


@pytest.fixture(scope="module", autouse=True)
def pinned_flavor():
    M.set_flavor("pinned")
    yield
    M.set_flavor("pinned")


@pytest.mark.parametrize("path", ["auto", "naive", "fast"])
@pytest.mark.parametrize("oc", T.cases(), ids=[c.name for c in T.cases()])
def test_case_pinned(oc, path, pins, monkeypatch):
    if path != "auto" and oc.op != "mul_mat":
        pytest.skip("one mul_mat path switch")
    if path != "auto":
        monkeypatch.setenv("SHLO_MUL_MAT_PATH", path)
    c = G.BY_NAME[oc.name]
    inputs = c.inputs()
    ins = [M.of_numpy(a) for a in inputs]
    text = case_module(oc, c)
    want = pins["pinned"]["%s/out.f32" % oc.name]
    if oc.expect_refusal:
        st, msg = run_module(text, ins, L.Faults(), True)
        assert st == "err" and "not carried" in msg, msg
        return
    for compile in (True, False):
        st, got = run_module(text, ins, L.Faults(), compile)
        assert st == "ok", got
        if hashlib.sha256(got).hexdigest() != want:
            pytest.fail("%s [%s]: %s" % (oc.name, "compiled" if compile else "uncompiled",
                                         first_diff(got, G.oracle_output(c, inputs, O.PINNED))))
    if path == "auto":
        fault = oc.fault
        if fault.dotPlain and c.extra["K"] < 16:
            # In the pinned build ggml's tail is a separate multiply and add, so for
            # K < 16 the planted sequential sum (written against the stock build's
            # fmaf tail, Tests/OpTests.lean:121) is ggml's own order: plant the
            # built-in matmul instead.
            fault = L.Faults(dotBuiltin=True)
        st, got = run_module(text, ins, fault, True)
        if st == "ok":
            assert hashlib.sha256(got).hexdigest() != want, "planted fault (%s) not caught" % oc.fault_name


STOCK_CASES = ["mul_mat_small", "mul_mat_k2", "mul_mat_heading", "mul_mat_root_in", "mul_mat_body_in",
               "mul_mat_scores", "soft_max_small", "norm_small", "silu_small", "gelu_erf_small"]


@pytest.mark.parametrize("name", STOCK_CASES)
def test_case_stock(name, pins):
    """The stock build differs from pinned only in the mul_mat tail and erff."""
    oc = [x for x in T.cases() if x.name == name][0]
    c = G.BY_NAME[name]
    ins = [M.of_numpy(a) for a in c.inputs()]
    M.set_flavor("stock")
    try:
        st, got = run_module(case_module(oc, c), ins, L.Faults(), True)
    finally:
        M.set_flavor("pinned")
    if name.startswith("gelu_erf"):
        assert st == "err" and "not carried" in got
        return
    assert st == "ok", got
    assert hashlib.sha256(got).hexdigest() == pins["stock"]["%s/out.f32" % name]


def _lcg(s):
    return (s * 1664525 + 1013904223) & 0xFFFFFFFF


def random_normals(n, seed, max_exp=254):
    """OpTests.lean:229-238."""
    out = np.empty(n, dtype=np.uint32)
    s = seed
    for i in range(n):
        s = _lcg(s)
        a = s
        s = _lcg(s)
        e = 1 + (s >> 8) % max_exp
        out[i] = (a & 0x807FFFFF) | (e << 23)
    return out


@pytest.fixture(scope="module")
def probe_inputs():
    n = 1 << 20
    return random_normals(n, 7, 200), random_normals(n, 11, 200)


def test_builtin_probes(probe_inputs):
    """OpTests.lean:240-270: the exact kernels against host IEEE, and the planted faults."""
    from shlo import run as Run
    a, b = probe_inputs
    n = a.size
    fa, fb = M.of_numpy(a.view(np.float32)), M.of_numpy(b.view(np.float32))
    want_div = (a.view(np.float32) / b.view(np.float32)).view(np.uint32)
    abs_a = (a & 0x7FFFFFFF).view(np.float32)
    want_sqrt = np.sqrt(abs_a).view(np.uint32)
    builtin_div = M.to_numpy(M.binary(M.opDiv, fa, fb)).view(np.uint32)
    exact_div = M.to_numpy(Run.divide(fa, fb, n)).view(np.uint32)
    fabs = M.of_numpy(abs_a)
    exact_sqrt = M.to_numpy(Run.sqrt(fabs, n)).view(np.uint32)
    d1 = int(np.count_nonzero(builtin_div != want_div))
    d2 = int(np.count_nonzero(exact_div != want_div))
    d4 = int(np.count_nonzero(exact_sqrt != want_sqrt))
    assert d2 == 0, "exact_divide kernel: %d of %d differ from IEEE" % (d2, n)
    assert d4 == 0, "exact_sqrt kernel: %d of %d differ from IEEE" % (d4, n)
    assert d1 != 0, "exact_divide planted fault (built-in /) not caught"
    nudged = M.of_numpy(((a & 0x7FFFFFFF) ^ 1).view(np.float32))
    d5 = int(np.count_nonzero(M.to_numpy(Run.sqrt(nudged, n)).view(np.uint32) != want_sqrt))
    assert d5 != 0, "exact_sqrt planted fault (input one ulp off) not caught"
