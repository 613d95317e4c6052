"""Dataflow IR behaviour (reference tests/test_ir.py, plus the additions)."""
import pytest

from molten.ir import DataflowGraph, OpType, TensorShape


def test_builders_count_and_types():
    g = DataflowGraph("t")
    x = g.add_input("x", TensorShape([4, 8]))
    w = g.add_input("w", TensorShape([4, 8]))
    s = g.add(x, w)
    g.add_output(s)
    assert len(g.ops) == 4
    assert g.ops[x].op_type == OpType.INPUT and g.ops[s].op_type == OpType.ADD


def test_topological_order_respects_edges():
    g = DataflowGraph("t")
    x = g.add_input("x", TensorShape([4]))
    y = g.add_input("y", TensorShape([4]))
    z = g.add(x, y)
    o = g.add_output(z)
    order = g.topological_order()
    assert order.index(x) < order.index(z) < order.index(o)
    assert order.index(y) < order.index(z)


def test_topological_order_is_reference_post_order():
    # inputs visited in op-id order, depth first, post order
    g = DataflowGraph("t")
    a = g.add_input("a", TensorShape([4]))
    c = g.add_constant("c", 2.0)
    m = g.mul(a, c)
    b = g.add_input("b", TensorShape([4]))
    s = g.add(b, m)
    assert g.topological_order() == [a, c, m, b, s]


def test_deep_chain_has_no_recursion_limit():
    g = DataflowGraph("deep")
    x = g.add_input("x", TensorShape([4]))
    for _ in range(5000):
        x = g.add_op(OpType.RELU, [x])
    assert len(g.topological_order()) == 5001


def test_consumers_producers():
    g = DataflowGraph("t")
    x = g.add_input("x", TensorShape([4]))
    y = g.add_input("y", TensorShape([4]))
    z = g.add(x, y)
    assert g.consumers(x) == [z]
    assert set(g.producers(z)) == {x, y}


def test_classification():
    g = DataflowGraph("t")
    x = g.add_input("x", TensorShape([4]))
    y = g.add_input("y", TensorShape([4]))
    a = g.add(x, y)
    mm = g.matmul(x, y)
    sm = g.softmax(x)
    r = g.add_op(OpType.RMS, [x])
    c = g.clamp(x, -1, 1)
    assert g.is_elementwise(a) and g.is_elementwise(c)
    assert not g.is_elementwise(mm) and not g.is_elementwise(sm)
    assert g.is_reduction(sm) and g.is_reduction(r)


def test_rms_norm_expansion_and_eps():
    g = DataflowGraph("rms")
    x = g.add_input("x", TensorShape([4, 8]))
    w = g.add_input("w", TensorShape([8]))
    out = g.rms_norm(x, w, "norm", eps=1e-5)
    kinds = [g.ops[i].op_type for i in g.topological_order()]
    assert kinds == [OpType.INPUT, OpType.INPUT, OpType.RMS, OpType.DIV, OpType.MUL]
    rms = [o for o in g.ops.values() if o.op_type == OpType.RMS][0]
    assert rms.attrs["eps"] == 1e-5 and g.ops[out].op_type == OpType.MUL


def test_softmax_records_dim_and_causal_mask_constant():
    g = DataflowGraph("t")
    x = g.add_input("x", TensorShape([2, 4]))
    m = g.causal_mask(period=4, offset=1)
    s = g.softmax(g.add(x, m), dim=-1)
    assert g.ops[s].reduction_dim == -1
    assert g.ops[m].op_type == OpType.CONSTANT and g.ops[m].attrs["kind"] == "causal_mask"


def test_repr_and_shapes():
    g = DataflowGraph("named")
    g.add_input("x", TensorShape([4]))
    assert "named" in repr(g)
    s = TensorShape([4, 8, 16])
    assert s.ndim == 3 and s.is_fully_known
    s = TensorShape(["batch", 8, "seq"])
    assert s.ndim == 3 and not s.is_fully_known


def test_op_type_members_match_reference_order():
    names = [m.name for m in OpType]
    assert names[:16] == ["ADD", "SUB", "MUL", "DIV", "NEG", "SQRT", "RSQRT", "EXP", "LOG",
                          "TANH", "SIGMOID", "GELU", "SILU", "RELU", "ABS", "CLAMP"]
    assert names[-3:] == ["INPUT", "OUTPUT", "CONSTANT"] and len(names) == 35
    assert OpType.ADD.value == 1 and OpType.CONSTANT.value == 35
