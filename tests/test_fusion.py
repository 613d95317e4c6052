"""Fusion engine: the reference's six rules and greedy grouping.

The groupings the reference's own FusionEngine produced for every benchmark
graph and every graph of its unit tests are recorded in
tests/golden/fusion_groups.json (tests/golden/make_golden.py)."""
import json
import os

import pytest

from molten.compiler import ZeroCompiler
from molten.fusion import FusionEngine
from molten.ir import DataflowGraph, OpType, TensorShape
from molten_b200 import graphs

TS = TensorShape


def names(g, groups):
    return [[g.ops[i].op_type.name for i in grp.op_ids] for grp in groups]


def test_elementwise_chain_is_one_group():
    g = DataflowGraph("elem_chain")
    x = g.add_input("x", TS([4, 8]))
    y = g.add_input("y", TS([4, 8]))
    g.add_output(g.add_op(OpType.RELU, [g.mul(g.add(x, y), x)]))
    groups = FusionEngine().fuse(g)
    assert len(groups) == 1 and len(groups[0].op_ids) == 3


def test_two_matmuls_never_share_a_group():
    g = DataflowGraph("two")
    x = g.add_input("x", TS([4, 8]))
    w1 = g.add_input("w1", TS([8, 16]))
    w2 = g.add_input("w2", TS([16, 8]))
    g.add_output(g.matmul(g.matmul(x, w1), w2))
    groups = FusionEngine().fuse(g)
    assert len(groups) >= 2
    for grp in groups:
        assert sum(g.ops[i].op_type == OpType.MATMUL for i in grp.op_ids) <= 1


def test_matmul_epilogue_fuses():
    g = DataflowGraph("mm")
    x = g.add_input("x", TS([4, 8]))
    w = g.add_input("w", TS([8, 16]))
    b = g.add_input("bias", TS([16]))
    g.add_output(g.add_op(OpType.RELU, [g.add(g.matmul(x, w), b)]))
    assert len(FusionEngine().fuse(g)) == 1


def test_report_text():
    g = DataflowGraph("rep")
    x = g.add_input("x", TS([4]))
    g.add_output(g.add(x, x))
    eng = FusionEngine()
    rep = eng.report(g, eng.fuse(g))
    assert "Fusion Report for 'rep'" in rep and "Kernel 0: [ADD] (elementwise)" in rep


def test_reduction_dims_rule():
    g = DataflowGraph("red")
    x = g.add_input("x", TS([4, 8]))
    a = g.add_op(OpType.SUM, [x])
    g.ops[a].reduction_dim = -1
    b = g.add_op(OpType.MAX, [a])
    g.ops[b].reduction_dim = 0
    c = g.add_op(OpType.MIN, [a])
    g.ops[c].reduction_dim = -1
    groups = FusionEngine().fuse(g)
    by_op = {i: k for k, grp in enumerate(groups) for i in grp.op_ids}
    assert by_op[a] == by_op[c] != by_op[b]


def test_group_ids_keep_counting_across_calls():
    eng = FusionEngine()
    g = graphs.rmsnorm(4, 8)
    first = eng.fuse(g)[0].group_id
    second = eng.fuse(g)[0].group_id
    assert second == first + 1


@pytest.fixture(scope="module")
def ref_groups(golden_dir):
    with open(os.path.join(golden_dir, "fusion_groups.json")) as f:
        return json.load(f)


def _reference_graphs():
    """The graphs tests/golden/make_golden.py fused with the reference."""
    out = {
        "rmsnorm": graphs.rmsnorm(2048, 5120),
        "rmsnorm_silu_gate": graphs.rmsnorm_silu_gate(8192, 3584),
        "softmax": graphs.softmax((32, 2048, 2048)),
        "softmax_causal": graphs.softmax((32, 2048, 2048), causal=True),
        "chain": graphs.chain(16384, 8192),
        "gemm_bias_gelu": graphs.gemm_bias_gelu(8192, 4096, 14336),
    }
    g = DataflowGraph("elem_chain")
    x = g.add_input("x", TS([4, 8]))
    y = g.add_input("y", TS([4, 8]))
    g.add_output(g.add_op(OpType.RELU, [g.mul(g.add(x, y), x)]))
    out["elem_chain"] = g
    g = DataflowGraph("two_matmul")
    x = g.add_input("x", TS([4, 8]))
    w1 = g.add_input("w1", TS([8, 16]))
    w2 = g.add_input("w2", TS([16, 8]))
    g.add_output(g.matmul(g.matmul(x, w1), w2))
    out["two_matmul"] = g
    g = DataflowGraph("matmul_epilogue")
    x = g.add_input("x", TS([4, 8]))
    w = g.add_input("w", TS([8, 16]))
    b = g.add_input("bias", TS([16]))
    g.add_output(g.add_op(OpType.RELU, [g.add(g.matmul(x, w), b)]))
    out["matmul_epilogue"] = g
    g = DataflowGraph("transformer_block")
    x = g.add_input("x", TS([4, 512]))
    w = g.add_input("w", TS([512]))
    g.rms_norm(x, w, "norm")
    q = g.add_input("q", TS([4, 512]))
    k = g.add_input("k", TS([512, 4]))
    g.add_output(g.softmax(g.matmul(q, k)))
    out["transformer_block"] = g
    g = DataflowGraph("norm_gemm")
    x = g.add_input("x", TS([256, 512]))
    w = g.add_input("w", TS([512]))
    B = g.add_input("B", TS([512, 384]))
    bias = g.add_input("bias", TS([384]))
    g.add_output(g.add_op(OpType.GELU, [g.add(g.matmul(g.rms_norm(x, w, "norm"), B), bias)]))
    out["norm_gemm"] = g
    g = DataflowGraph("attention_score")
    q = g.add_input("q", TS([256, 128]))
    k = g.add_input("k", TS([512, 128]))
    kt = g.add_op(OpType.TRANSPOSE, [k], "kT")
    sc = g.add_constant("scale", 0.08838834764831845)
    g.add_output(g.softmax(g.mul(g.matmul(q, kt), sc)))
    out["attention_score"] = g
    g = DataflowGraph("norm_rope")
    x = g.add_input("x", TS([2, 16, 4, 64]))
    w = g.add_input("w", TS([64]))
    f = g.add_input("freqs", TS([16, 64]))
    g.add_output(g.rope(g.rms_norm(x, w, "norm"), f))
    out["norm_rope"] = g
    g = DataflowGraph("mixed")
    x = g.add_input("x", TS([16, 32]))
    s1 = g.add_op(OpType.SUM, [x])
    g.ops[s1].reduction_dim = -1
    e = g.add_op(OpType.EXP, [x])
    s2 = g.add_op(OpType.MAX, [e])
    g.ops[s2].reduction_dim = 0
    d = g.div(e, s1)
    g.add_output(g.matmul(d, g.add_input("w", TS([32, 8]))))
    g.add_output(s2)
    out["mixed_reductions"] = g
    return out


@pytest.mark.parametrize("case", sorted(_reference_graphs()))
def test_groups_match_reference(case, ref_groups):
    g = _reference_graphs()[case]
    assert names(g, FusionEngine().fuse(g)) == ref_groups["groups"][case]


def test_optimize_matches_reference(ref_groups):
    g = DataflowGraph("opt")
    x = g.add_input("x", TS([4, 8]))
    one = g.add_constant("one", 1.0)
    zero = g.add_constant("zero", 0.0)
    c2 = g.add_constant("two", 2.0)
    c3 = g.add_constant("three", 3.0)
    five = g.add(c2, c3)
    t = g.mul(x, one)
    t = g.add(t, zero)
    t = g.mul(t, five)
    g.add_output(g.add_op(OpType.RELU, [t]))
    g2 = ZeroCompiler()._optimize(g)
    ops = [[i, o.op_type.name, list(o.inputs), o.attrs.get("value")] for i, o in sorted(g2.ops.items())]
    assert ops == ref_groups["optimize"]["ops"]
    assert names(g2, FusionEngine().fuse(g2)) == ref_groups["optimize"]["groups"]
