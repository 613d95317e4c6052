"""Helpers shared by the tests: golden fixtures -> (graph, inputs, reference)."""
import json
import os

import numpy as np

from molten_b200 import graphs
from molten_b200.ir import DataflowGraph, OpType, TensorShape

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CASES = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))

NP_OF = {"float32": np.float32, "bfloat16": np.uint16, "float16": np.float16}


def load(case):
    d = np.load(os.path.join(GOLDEN, case + ".npz"))
    meta = json.loads(str(d["meta"]))
    inputs = {k: d["in_" + k] for k in meta["inputs"]}
    return meta, inputs, d["ref_f32"], d["ref_out"]


def input_dtype(arr):
    return "bfloat16" if arr.dtype == np.uint16 else ("float16" if arr.dtype == np.float16 else "float32")


def graph_for(meta, inputs):
    """The molten graph whose evaluation the fixture holds."""
    kind = meta["kind"]
    first = inputs[meta["inputs"][0]]
    dt = input_dtype(first)
    if kind == "rmsnorm":
        r, c = first.shape
        return graphs.rmsnorm(r, c, dtype=dt, eps=meta["eps"])
    if kind == "rmsnorm_silu_gate":
        r, c = first.shape
        return graphs.rmsnorm_silu_gate(r, c, dtype=dt, eps=meta["eps"])
    if kind == "softmax":
        return graphs.softmax(tuple(first.shape), dtype=dt, causal=meta["causal"])
    if kind == "chain":
        r, c = first.shape
        return graphs.chain(r, c, dtype=dt)
    if kind == "gemm_bias_gelu":
        m, k = first.shape
        n = inputs["B"].shape[1]
        return graphs.gemm_bias_gelu(m, k, n, dtype=dt)
    if kind == "attention_score":
        m, d = first.shape
        return graphs.attention_score(m, inputs["k"].shape[0], d, dtype=dt, scale=meta["scale"])
    if kind == "rope":
        b, sq, h, d = first.shape
        return graphs.rope(b, sq, h, d, dtype=dt, table_dtype=input_dtype(inputs["cos"]))
    if kind == "gelu_add":
        r, c = first.shape
        g = DataflowGraph("gelu_add")
        x = g.add_input("x", TensorShape([r, c]), dtype=dt)
        b = g.add_input("bias", TensorShape([c]), dtype=dt)
        g.add_output(g.add(g.gelu(x), b))
        return g
    raise KeyError(kind)


def bf16_ulp_diff(a_bits, b_bits):
    """|difference| in bf16 units in the last place (same-sign values)."""
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # map sign-magnitude to a monotone integer line
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), a + 0x8000)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), b + 0x8000)
    return np.abs(a - b)


def rounded_operand_bound(a_f32, b_f32, dtype, slope=1.0):
    """Extra tolerance for a GEMM whose A operand is computed (not a graph
    input): the tensor cores take A rounded once to ``dtype``, which moves
    each output by at most u * sum_k |a_k| |b_kn| (u = 2^-8 for bf16, 2^-11
    for fp16; Higham's first-order bound for perturbing every a_k by a
    relative u), times ``slope`` >= max |f'| of an elementwise epilogue f."""
    u = 2.0 ** -8 if dtype == "bfloat16" else 2.0 ** -11
    return slope * u * (np.abs(a_f32.astype(np.float64)) @ np.abs(b_f32.astype(np.float64)))


def assert_close(out_f32, ref_f32, dtype, what="", extra_abs=None):
    """The parity bar of this project.

    fp32:        |out - ref| <= 1e-5 |ref| + 1e-6 * max|ref|
    bf16 / fp16: |out - ref| <= 1e-2 |ref| + 1e-3 * rms(ref)
    (ref is the fp32-accumulated reference; the absolute term only covers
    values that cancel to near zero, e.g. y*0.5 + r or GELU at large -v).
    ``extra_abs`` (same shape as ref) adds a per-element bound, e.g.
    ``rounded_operand_bound`` for a GEMM fed by a computed operand.
    """
    out_f32 = np.asarray(out_f32, dtype=np.float32)
    ref_f32 = np.asarray(ref_f32, dtype=np.float32)
    assert out_f32.shape == ref_f32.shape, (what, out_f32.shape, ref_f32.shape)
    fin = np.isfinite(ref_f32)
    assert np.array_equal(np.isnan(out_f32), np.isnan(ref_f32)), f"{what}: NaN pattern differs"
    assert np.array_equal(np.isinf(out_f32) & ~fin, np.isinf(ref_f32)), f"{what}: inf pattern differs"
    o, r = out_f32[fin].astype(np.float64), ref_f32[fin].astype(np.float64)
    if r.size == 0:
        return
    if dtype == "float32":
        tol = 1e-5 * np.abs(r) + 1e-6 * np.abs(r).max()
    else:
        tol = 1e-2 * np.abs(r) + 1e-3 * np.sqrt(np.mean(r * r))
    if extra_abs is not None:
        tol = tol + np.broadcast_to(np.asarray(extra_abs, np.float64), ref_f32.shape)[fin]
    err = np.abs(o - r)
    bad = err > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} outside tolerance; "
                           f"max err {err.max():.3e}, worst at ref {r[np.argmax(err - tol)]:.6g}")
