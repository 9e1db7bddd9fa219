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
    # per layer: qkv, out projection (+ residual), ffn1, ffn2 (+ residual), 2 norms, the attention chain;
    # plus 2 timestep dense
    assert kinds.count("dense") == 4 * cfg.layers + 2
    assert kinds.count("norm") == 2 * cfg.layers
    assert kinds.count("attention") == cfg.layers
    att = [v for v in p.values() if v.kind == "attention"]
    assert all(len(v.skip) == 3 and v.scale == cfg.scale_bits() for v in att)
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


def attn_text(B, S, H, W, ret="%t"):
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    q, s_, o = T(B, S, H, W), T(B, H, S, S), T(B, H, S, W)
    rt = {"%t": q, "%s": s_, "%p": s_, "%o": o}[ret]
    return f"""module {{
  func.func public @main(%q: {q}, %k: {q}, %v: {q}) -> ({rt}) {{
    %s = "stablehlo.dot_general"(%q, %k) {{dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 2], rhs_batching_dimensions = [0, 2], lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [3]>}} : ({q}, {q}) -> {s_}
    %p = "stablehlo.custom_call"(%s) {{call_target_name = "ggml.soft_max", backend_config = "scale = 0x3E000000 : f32"}} : ({s_}) -> {s_}
    %o = "stablehlo.dot_general"(%p, %v) {{dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 1], rhs_batching_dimensions = [0, 2], lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [1]>}} : ({s_}, {q}) -> {o}
    %t = "stablehlo.transpose"(%o) {{permutation = array<i64: 0, 2, 1, 3>}} : ({o}) -> {q}
    func.return {ret} : {rt}
  }}
}}
"""


def test_attention_chain():
    p = F.plan(E.load(attn_text(2, 256, 8, 64)).main)
    assert list(p) == [0] and p[0].kind == "attention" and p[0].skip == [1, 2, 3] and p[0].v == "%v"
    assert p[0].scale == 0x3E000000 and p[0].result == "%t"
    assert F.plan(E.load(attn_text(1, 128, 2, 64)).main)[0].kind == "attention"
    # positions or width the kernel does not carry, or an intermediate read elsewhere: not fused
    assert F.plan(E.load(attn_text(2, 196, 8, 64)).main) == {}
    assert F.plan(E.load(attn_text(2, 256, 4, 32)).main) == {}
    for ret in ("%s", "%p", "%o"):
        assert F.plan(E.load(attn_text(2, 256, 8, 64, ret)).main) == {}
    # the encoder (196 positions) keeps its attention unfused
    kinds = [v.kind for v in F.plan(E.load(D.module_text(D.ENCODER, 2)).main).values()]
    assert "attention" not in kinds
