"""The benchmark workloads, bit for bit: one transformer encoder layer (seq 196,
d 512, 8 heads, FFN 2048; batch 1) and the 8-layer motion denoiser (seq 256),
each run as a StableHLO module through the executor path and compared word for
word with the oracle's composition of ggml-order ops."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from oracle import model_oracle as MO  # noqa: E402
from shlo import denoiser as D  # noqa: E402
from shlo import exec as E  # noqa: E402
from shlo import mlx as M  # noqa: E402


def run_model(cfg, batch, compile=True, seed=1):
    w = D.init_weights(cfg, seed)
    ins = D.inputs(cfg, batch, seed)
    l = E.load(D.module_text(cfg, batch))
    fn = E.prepare(l, None, compile)
    args = [M.of_numpy(a) for a in ins] + [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    out = M.to_numpy(E.call(fn, args)[0])
    return out, MO.forward(cfg, w, ins)


def assert_same(got, want):
    g, w = got.view(np.uint32).reshape(-1), want.view(np.uint32).reshape(-1)
    bad = np.nonzero(g != w)[0]
    assert bad.size == 0, "%d of %d words differ, first at %d: got %08x want %08x" % (
        bad.size, g.size, bad[0], g[bad[0]], w[bad[0]])


def test_encoder_layer_config4():
    got, want = run_model(D.ENCODER, 1)
    assert_same(got, want)


def test_denoiser_two_layers_batch2():
    cfg = D.Config(layers=2)
    got, want = run_model(cfg, 2, compile=False, seed=3)
    assert_same(got, want)


def test_denoiser_full_batch1():
    got, want = run_model(D.DENOISER, 1)
    assert_same(got, want)
