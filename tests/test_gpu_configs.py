"""The benchmark configurations on their exact inputs, bit for bit against the
oracle, through the executor path (module text -> shlo.exec -> shlo.lower ->
the C ABI), compiled (CUDA-graph replay) and uncompiled.

* Configuration 1: one stablehlo.dot_general f32 [64,256] x [256,128] ->
  [64,128] on inputs uniform in [-1, 1] from splitmix32 seed 0, the lhs drawn
  first (the generator of ref/ggml_ref.c:21-43).
* Configuration 5: the 8-layer motion denoiser at batch 16 and 64, every
  sample compared; at batch 512 (the largest of the sweep) a spread subset of
  samples, which is enough because samples are independent: each sample's
  rows meet only its own rows (attention is per sample) and every other op is
  row-wise, so a sample's output does not depend on the batch it rode in.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from oracle import model_oracle as MO  # noqa: E402
from oracle import oracle as O  # noqa: E402
from shlo import denoiser as D  # noqa: E402
from shlo import exec as E  # noqa: E402
from shlo import mlx as M  # noqa: E402
from shlo import run as Run  # noqa: E402

CONFIG1 = """module {
  func.func public @main(%a: tensor<64x256xf32>, %b: tensor<256x128xf32>) -> (tensor<64x128xf32>) {
    %v0 = "stablehlo.dot_general"(%a, %b) {dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [1], rhs_contracting_dimensions = [0]>} : (tensor<64x256xf32>, tensor<256x128xf32>) -> tensor<64x128xf32>
    func.return %v0 : tensor<64x128xf32>
  }
}
"""


def config1_inputs():
    s = O.Stream(0)
    lhs = s.unif(1.0, 64 * 256).reshape(64, 256)
    rhs = s.unif(1.0, 256 * 128).reshape(256, 128)
    return lhs, rhs


def assert_same(got, want, what):
    g = np.ascontiguousarray(got).view(np.uint32).reshape(-1)
    w = np.ascontiguousarray(want).view(np.uint32).reshape(-1)
    assert g.size == w.size, (what, g.size, w.size)
    bad = np.nonzero(g != w)[0]
    assert bad.size == 0, "%s: %d of %d words differ, first at %d: got %08x want %08x" % (
        what, bad.size, g.size, bad[0], g[bad[0]], w[bad[0]])


@pytest.mark.parametrize("flavor", ["pinned", "stock"])
@pytest.mark.parametrize("compile", [True, False])
def test_config1_dot_general_exact_inputs(flavor, compile):
    M.set_flavor(flavor)
    try:
        lhs, rhs = config1_inputs()
        assert lhs.min() >= -1.0 and lhs.max() <= 1.0 and lhs.std() > 0.5
        fn = E.prepare(E.load(CONFIG1), None, compile)
        args = [M.of_numpy(lhs), M.of_numpy(rhs)]
        want = O.mul_mat(np.ascontiguousarray(rhs.T), lhs, 256, 128, 64, 64, 0,
                         O.PINNED if flavor == "pinned" else O.STOCK).reshape(64, 128)
        for call in range(3):  # the first call records the graph, the later ones replay it
            got = M.to_numpy(E.call(fn, args)[0])
            assert_same(got, want, "config 1 (%s, compile=%s), call %d" % (flavor, compile, call))
        # and the kernel alone, as Run.lean's mulMat issues it
        got = M.to_numpy(Run.mul_mat(M.of_numpy(np.ascontiguousarray(rhs.T)), M.of_numpy(lhs), 256, 128, 64, 64, 0))
        assert_same(got.reshape(64, 128), want, "config 1 kernel")
    finally:
        M.set_flavor("pinned")


def _denoiser(batch, seed=1):
    cfg = D.DENOISER
    M.set_flavor("pinned")
    w = D.init_weights(cfg, seed)
    ins = D.inputs(cfg, batch, seed)
    fn = E.prepare(E.load(D.module_text(cfg, batch)), None, True)
    args = [M.of_numpy(a) for a in ins] + [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    got = M.to_numpy(E.call(fn, args)[0])
    again = M.to_numpy(E.call(fn, args)[0])  # a graph replay gives the same bits
    assert_same(again, got, "denoiser batch %d replay" % batch)
    return cfg, w, ins, got


@pytest.mark.parametrize("batch", [16, 64])
def test_denoiser_every_sample(batch):
    cfg, w, ins, got = _denoiser(batch)
    want = MO.forward(cfg, w, ins)
    for s in range(batch):
        assert_same(got[s], want[s], "denoiser batch %d, sample %d" % (batch, s))


def test_denoiser_batch512_spread_samples():
    cfg, w, ins, got = _denoiser(512)
    rng = np.random.default_rng(512)
    idx = sorted({0, 1, 63, 64, 255, 256, 510, 511} | set(int(i) for i in rng.choice(512, 4, replace=False)))
    want = MO.forward(cfg, w, [a[idx] for a in ins])
    for j, s in enumerate(idx):
        assert_same(got[s], want[j], "denoiser batch 512, sample %d" % s)
