"""The DSL front end, fusion rules, plasma grouping, kernel-signature records
and arena plan of libtkm.so produce the same public TkmGraph as the
reference's own host code (oracle/_ref/libtkm_ref_host.so, built from the
reference sources), byte for byte, on models that exercise every rule."""
import ctypes
import glob
import os

import pytest

from oracle.tkm_abi import Graph, bind, compile_graph

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_HOST = os.path.join(ROOT, "oracle", "_ref", "libtkm_ref_host.so")
from oracle.build_ref import REF  # the reference source tree (TKM_REFERENCE, else beside the repository)

REF_MODELS = os.path.join(REF, "models")

# Graphs written for these tests (same grammar as the reference's models).
DSL = {
    "llama_c1": """
input: 1x128x256
prng: pcg32
flow:
  layer x 2: {
    attn: {
      branch: RMSNorm -> {
        q: FC(256) -> RoPE(theta=10000)
        k: FC(256) -> RoPE(theta=10000)
        v: FC(256)
      } -> GQA(q=4, kv=4, d=64, causal=true) -> FC(256)
      skip: Identity
    } -> Add
    ffn: {
      branch: RMSNorm -> {
        gate: FC(688) -> SiLU
        up: FC(688)
      } -> Mul -> FC(256)
      skip: Identity
    } -> Add
  }
  head: RMSNorm -> FC(1024) -> SoftmaxCE
""",
    "gqa_qknorm_rope_scaled": """
input: 1x64x512
flow:
  blk x 2: {
    a: {
      branch: LN(1e-6) -> {
        q: FC(512) -> QKNorm -> RoPE(theta=500000, scale=8, low_freq_factor=1, high_freq_factor=4, original_context_length=8192)
        k: FC(128) -> QKNorm -> RoPE(theta=500000, scale=8, low_freq_factor=1, high_freq_factor=4, original_context_length=8192)
        v: FC(128)
      } -> GQA(q=8, kv=2, d=64) -> FC(512) -> SoftCap(50.0) -> LayerScale -> Drop(0.1)
      skip: Identity
    } -> Add
    f: {
      branch: RMSNorm -> {
        gate: FC(1024) -> SoftCap(30) -> CosGate -> SiLU
        up  : FC(1024) -> ReLU2
      } -> Mul -> FC(512) -> DyT(0.5) -> Drop(p=0.1, rng=philox)
      skip: Identity
    } -> Add
  }
  head: RMSNorm -> FC(10) -> SoftmaxFocal(gamma=2.5)
""",
    "rules": """
input: 1x1x32
prng: xorshift
flow:
  a: FC(64) -> Scale(2.0) -> Scale(0.25) -> Drop(0.0) -> Scale(1.0) -> GELU
  b: { x: FC(64) -> Softplus, y: FC(64) -> Snake(1.7) } -> Mul -> L2Norm -> Tanh
  c: { p: Mish -> HardSwish, q: Identity } -> Add -> BN -> PReLU -> xATLU
  d: FC(16) -> Softmax -> FC(4) -> SoftmaxMSE
""",
    "twin_custom": """
input: 1x1x8
flow:
  trunk: FC(8) -> Softplus -> FC(8) -> Tanh
  gate: {
    branch: FC(8) -> Softplus -> Scale(0.7)
    skip: FC(8) -> GELU
  } -> Mul -> Softplus -> FC(4) -> SoftmaxCE
""",
    "image_like": """
input: 8x8x4
flow:
  s: Flatten -> FC(32) -> LeakyReLU(0.2) -> ELU -> HardSigmoid -> Sigmoid -> SwishBeta -> Sin(2.0) -> Clamp(3)
  h: FC(10) -> SoftmaxCE
""",
    "residual_of_input": """
input: 1x16x64
flow:
  r: {
    branch: SiLU -> Scale(0.5)
    skip: Identity
  } -> Add
  n: RMSNorm -> FC(8) -> SoftmaxCE
""",
}


def ref_lib():
    if not os.path.exists(REF_HOST):
        pytest.skip("oracle/_ref/libtkm_ref_host.so not built (needs the reference tree)")
    return bind(ctypes.CDLL(REF_HOST))


def our_lib():
    import tokamak_b200
    return bind(tokamak_b200.engine())


def all_cases():
    from tokamak_b200 import configs
    cases = [(k, v) for k, v in DSL.items()]
    # the benchmark configurations, including the single-layer slices that the
    # smoke check and the CPU baseline run (written without the loop macro)
    for name, cfg in (("C1", configs.C1), ("C4", configs.C4)):
        for layers in (1, 2):
            cases.append((f"{name}_layers{layers}", configs.dsl_for(dict(cfg, layers=layers, seq=64))))
    for path in sorted(glob.glob(os.path.join(REF_MODELS, "*.tkm"))):
        cases.append((os.path.basename(path), open(path).read()))
    return cases


@pytest.mark.parametrize("name,dsl", all_cases(), ids=[c[0] for c in all_cases()])
@pytest.mark.parametrize("batch", [1, 4])
def test_graph_matches_reference(name, dsl, batch):
    ref, ours = ref_lib(), our_lib()
    gr = compile_graph(ref, dsl, batch)
    go = compile_graph(ours, dsl, batch)
    assert go.num_nodes == gr.num_nodes > 1
    assert go.num_groups == gr.num_groups
    for i in range(gr.num_nodes):
        a, b = bytes(gr.nodes[i]), bytes(go.nodes[i])
        assert a == b, f"node {i} ({gr.nodes[i].tag}) differs"
    for i in range(gr.num_groups):
        assert bytes(gr.groups[i]) == bytes(go.groups[i]), f"group {i} differs"
    assert bytes(gr) == bytes(go)


def test_registry_matches_reference():
    ref, ours = ref_lib(), our_lib()
    n = ref.tkm_get_spec_count()
    assert ours.tkm_get_spec_count() == n
    for i in range(n):
        a, b = ref.tkm_find_spec_by_index(i).contents, ours.tkm_find_spec_by_index(i).contents
        assert (a.op, a.dsl_name, a.cat, a.res_flags, a.default_fval) == \
            (b.op, b.dsl_name, b.cat, b.res_flags, b.default_fval), a.dsl_name
        # the formula operators evaluate to the same values
        for x in (-1.6, -0.4, 0.0, 0.5, 1.4, 3.0):
            for expr_a, expr_b in ((a.fwd_expr, b.fwd_expr), (a.bwd_expr, b.bwd_expr)):
                if expr_a is None:
                    assert expr_b is None
                    continue
                va, vb = ctypes.c_float(), ctypes.c_float()
                f = a.default_fval or 1.3
                assert ref.tkm_eval_math_expr(expr_a, x, f, ctypes.byref(va)) == 1
                assert ours.tkm_eval_math_expr(expr_b, x, f, ctypes.byref(vb)) == 1
                assert abs(va.value - vb.value) <= 1e-6 * max(1.0, abs(va.value)), (a.dsl_name, x)
    assert ours.tkm_verify_registry() == 0
    cr, co = ctypes.c_int(), ctypes.c_int()
    ref.tkm_get_fusion_rules(ctypes.byref(cr))
    ours.tkm_get_fusion_rules(ctypes.byref(co))
    assert cr.value == co.value == 4


@pytest.mark.parametrize("expr,x,fval", [
    ("x * 2 + 1", 1.5, 0.0), ("-(x - 3) / 4", 2.0, 0.0), ("pow(abs(x), 1.5)", -2.0, 0.0),
    ("max(x, fval) - min(x, fval)", 0.3, 0.7), ("exp(log(x)) + sqrt(x)", 4.0, 0.0),
    ("sin(pi * x) + cos(x) + tanh(x)", 0.25, 0.0), ("ln(2)", 0.0, 0.0), ("1 / 2", 0.0, 0.0),
    ("+-x", 3.0, 0.0),
])
def test_formula_evaluator_matches_reference(expr, x, fval):
    ref, ours = ref_lib(), our_lib()
    va, vb = ctypes.c_float(), ctypes.c_float()
    assert ref.tkm_eval_math_expr(expr.encode(), x, fval, ctypes.byref(va)) == 1
    assert ours.tkm_eval_math_expr(expr.encode(), x, fval, ctypes.byref(vb)) == 1
    assert va.value == vb.value


@pytest.mark.parametrize("expr", ["x +", "foo(x)", "x y", "max(x)", "(x", "exp(x, 2)", ""])
def test_formula_evaluator_rejects(expr):
    ours = our_lib()
    v = ctypes.c_float()
    assert ours.tkm_eval_math_expr(expr.encode(), 1.0, 1.0, ctypes.byref(v)) == 0
    ref = ref_lib()
    assert ref.tkm_eval_math_expr(expr.encode(), 1.0, 1.0, ctypes.byref(v)) == 0


def test_rng_names():
    ours = our_lib()
    for name, val in (("xorshift", 1), ("wang", 2), ("pcg32", 3), ("philox4x32", 4), ("bogus", 2)):
        assert ours.tkm_parse_rng_name(name.encode()) == val
    assert ours.tkm_rng_name(3) == b"pcg32"


def test_errors_leave_an_empty_graph_instead_of_exiting():
    ours = our_lib()
    ours.tkm_last_error.restype = ctypes.c_char_p
    g = Graph()
    ours.tkm_parse_dsl(ctypes.byref(g), b"input: 1x1x8\nflow:\n  a: NoSuchOp -> FC(4)\n", 2)
    assert g.num_nodes == 0
    assert b"NoSuchOp" in ours.tkm_last_error()
    # odd channel count in a plasma group
    g = compile_graph(ours, "input: 1x1x8\nflow:\n  a: FC(5) -> SiLU -> FC(4) -> SoftmaxCE\n", 2)
    assert g.num_nodes == 0 and b"odd channel count" in ours.tkm_last_error()
    # GQA head mismatch
    g = compile_graph(ours, "input: 1x16x64\nflow:\n  a: {q: FC(64), k: FC(64), v: FC(64)} -> GQA(q=2, kv=2, d=48)\n", 1)
    assert g.num_nodes == 0 and b"GQA" in ours.tkm_last_error()
