"""The executor's fusion planner on module text (no GPU): which op sequences it
fuses, and that it leaves alone every sequence whose intermediates are read
elsewhere, or any run with a planted fault."""
from shlo import denoiser as D
from shlo import exec as E
from shlo import fuse as F
from shlo import lower as L


def test_denoiser_layers_fuse():
    cfg = D.Config(layers=2)
    fn = E.load(D.module_text(cfg, 2)).main
    p = F.plan(fn)
    kinds = [v.kind for v in p.values()]
    # per layer: qkv, out projection (+ residual), ffn1, ffn2 (+ residual), 2 norms; plus 2 timestep dense
    assert kinds.count("dense") == 4 * cfg.layers + 2
    assert kinds.count("norm") == 2 * cfg.layers
    res = [v for v in p.values() if v.kind == "dense" and v.res]
    assert len(res) == 2 * cfg.layers
    assert all(v.flags == F.Run.EP_BIAS | F.Run.EP_RES | F.Run.EP_RES_LHS for v in res)
    skipped = [j for v in p.values() for j in v.skip]
    assert len(skipped) == len(set(skipped))


MOD = """module {
  func.func public @main(%x: tensor<4x8xf32>, %w: tensor<6x8xf32>, %b: tensor<6xf32>) -> (tensor<4x6xf32>, tensor<4x6xf32>) {
    %v0 = "stablehlo.dot_general"(%x, %w) {dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [1], rhs_contracting_dimensions = [1]>} : (tensor<4x8xf32>, tensor<6x8xf32>) -> tensor<4x6xf32>
    %v1 = "stablehlo.broadcast_in_dim"(%b) {broadcast_dimensions = array<i64: 1>} : (tensor<6xf32>) -> tensor<4x6xf32>
    %v2 = "stablehlo.add"(%v1, %v0) : (tensor<4x6xf32>, tensor<4x6xf32>) -> tensor<4x6xf32>
    func.return %v2, %RET : tensor<4x6xf32>, tensor<4x6xf32>
  }
}
"""


def test_bias_on_the_left_and_extra_uses():
    fn = E.load(MOD.replace("%RET", "%v2")).main
    p = F.plan(fn)
    assert list(p) == [0] and p[0].flags == F.Run.EP_BIAS | F.Run.EP_BIAS_LHS and p[0].result == "%v2"
    # the dot's own result returned too: it must exist, so nothing is fused
    assert F.plan(E.load(MOD.replace("%RET", "%v0")).main) == {}
    # the broadcast bias read again: not fused
    assert F.plan(E.load(MOD.replace("%RET", "%v1")).main) == {}


def test_faults_disable_fusion():
    assert not F.any_fault(L.Faults())
    assert F.any_fault(L.Faults(dotPlain=True))
    assert F.any_fault(L.Faults(normGpuOps=True))
