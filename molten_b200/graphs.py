"""The five fused graphs of the benchmark set, built through the public IR.

Each builder returns a DataflowGraph whose fusion yields exactly one group:

* ``rmsnorm``          RMS -> DIV -> MUL (``ir.py:169-173``), fp32
* ``rmsnorm_silu_gate``  rmsnorm(x, w) * silu(g)  (``ops.py:38-42``), bf16
* ``softmax``          [ADD(causal mask) ->] SOFTMAX, fp32 or bf16
* ``chain``            gelu(x*a+b)*s + r -> clamp(-6, 6) -> *0.5 + r, bf16
* ``gemm_bias_gelu``   MATMUL -> ADD(bias) -> GELU, bf16

and the RoPE pattern of ``benchmarks/ops.py:24-35`` (``rope``) and the
attention-score pattern of ``benchmarks/ops.py:55-59`` (``attention_score``).
"""

from __future__ import annotations

from .ir import DataflowGraph, OpType, TensorShape


def rmsnorm(rows=2048, cols=5120, dtype="float32", eps=1e-6) -> DataflowGraph:
    g = DataflowGraph("fused_rmsnorm")
    x = g.add_input("x", TensorShape([rows, cols]), dtype=dtype)
    w = g.add_input("w", TensorShape([cols]), dtype=dtype)
    g.add_output(g.rms_norm(x, w, "norm", eps=eps))
    return g


def rmsnorm_silu_gate(rows=8192, cols=3584, dtype="bfloat16", eps=1e-6) -> DataflowGraph:
    g = DataflowGraph("rmsnorm_silu_gate")
    x = g.add_input("x", TensorShape([rows, cols]), dtype=dtype)
    w = g.add_input("w", TensorShape([cols]), dtype=dtype)
    gate = g.add_input("gate", TensorShape([rows, cols]), dtype=dtype)
    normed = g.rms_norm(x, w, "norm", eps=eps)
    g.add_output(g.mul(normed, g.silu(gate, "silu"), "gated"))
    return g


def softmax(shape=(32, 2048, 2048), dtype="float32", causal=False) -> DataflowGraph:
    g = DataflowGraph("softmax_causal" if causal else "softmax")
    x = g.add_input("logits", TensorShape(list(shape)), dtype=dtype)
    if causal:
        x = g.add(x, g.causal_mask(period=None), "masked")
    g.add_output(g.softmax(x, -1, "probs"))
    return g


def chain(rows=16384, cols=8192, dtype="bfloat16") -> DataflowGraph:
    """y = gelu_tanh(x*a + b)*s + r; y = clamp(y, -6, 6); y = y*0.5 + r."""
    g = DataflowGraph("ew_chain8")
    x = g.add_input("x", TensorShape([rows, cols]), dtype=dtype)
    r = g.add_input("r", TensorShape([rows, cols]), dtype=dtype)
    a = g.add_input("a", TensorShape([cols]), dtype=dtype)
    b = g.add_input("b", TensorShape([cols]), dtype=dtype)
    s = g.add_input("s", TensorShape([cols]), dtype=dtype)
    half = g.add_constant("half", 0.5)
    t = g.mul(x, a)
    t = g.add(t, b)
    t = g.gelu(t)
    t = g.mul(t, s)
    t = g.add(t, r)
    t = g.clamp(t, -6.0, 6.0)
    t = g.mul(t, half)
    t = g.add(t, r)
    g.add_output(t)
    return g


def gemm_bias_gelu(m=8192, k=4096, n=14336, dtype="bfloat16") -> DataflowGraph:
    g = DataflowGraph("gemm_bias_gelu")
    a = g.add_input("A", TensorShape([m, k]), dtype=dtype)
    b = g.add_input("B", TensorShape([k, n]), dtype=dtype)
    bias = g.add_input("bias", TensorShape([n]), dtype=dtype)
    y = g.gelu(g.add(g.matmul(a, b), bias))
    g.add_output(y)
    return g


BUILDERS = {
    "rmsnorm": rmsnorm,
    "rmsnorm_silu_gate": rmsnorm_silu_gate,
    "softmax": softmax,
    "chain": chain,
    "gemm_bias_gelu": gemm_bias_gelu,
}


def rope(batch=1, seq=4096, heads=32, head_dim=128, dtype="bfloat16", table_dtype="float32",
         style=None, packed=False) -> DataflowGraph:
    """ROTATE(x, cos, sin) on x [batch, seq, heads, head_dim] with cos/sin
    [seq, head_dim/2] (``ops.py:24-35``); ``packed`` uses the reference
    builder's two-input form, one [seq, head_dim] table of (cos, sin) pairs."""
    g = DataflowGraph("rope")
    x = g.add_input("x", TensorShape([batch, seq, heads, head_dim]), dtype=dtype)
    if packed:
        f = g.add_input("freqs", TensorShape([seq, head_dim]), dtype=table_dtype)
        g.add_output(g.rope(x, f, "rope", style=style))
    else:
        c = g.add_input("cos", TensorShape([seq, head_dim // 2]), dtype=table_dtype)
        s = g.add_input("sin", TensorShape([seq, head_dim // 2]), dtype=table_dtype)
        g.add_output(g.rope(x, c, "rope", sin=s, style=style))
    return g


BUILDERS["rope"] = rope


def attention_score(m=2048, n=2048, d=128, dtype="bfloat16", scale=None,
                    heads=None) -> DataflowGraph:
    """softmax(Q @ K^T * scale) with Q [m, d], K [n, d] -- or [heads, m, d],
    [heads, n, d], one problem per head (``ops.py:55-59``); scale defaults
    to 1/sqrt(d)."""
    g = DataflowGraph("attention_score")
    lead = [heads] if heads else []
    q = g.add_input("q", TensorShape(lead + [m, d]), dtype=dtype)
    k = g.add_input("k", TensorShape(lead + [n, d]), dtype=dtype)
    s = g.add_constant("scale", float(scale if scale is not None else d ** -0.5))
    g.add_output(g.softmax(g.mul(g.matmul(q, g.transpose(k, "kT"), "scores"), s), -1, "probs"))
    return g


BUILDERS["attention_score"] = attention_score


def rmsnorm_gemm(m=8192, k=4096, n=14336, dtype="bfloat16", eps=1e-6) -> DataflowGraph:
    """GELU(rmsnorm(x, w) @ B + bias): the RMSNorm -> GEMM prologue pattern
    (one fusion group [RMS, DIV, MUL, MATMUL, ADD, GELU])."""
    g = DataflowGraph("rmsnorm_gemm")
    x = g.add_input("x", TensorShape([m, k]), dtype=dtype)
    w = g.add_input("w", TensorShape([k]), dtype=dtype)
    B = g.add_input("B", TensorShape([k, n]), dtype=dtype)
    bias = g.add_input("bias", TensorShape([n]), dtype=dtype)
    g.add_output(g.gelu(g.add(g.matmul(g.rms_norm(x, w, "norm", eps=eps), B, "mm"), bias)))
    return g


BUILDERS["rmsnorm_gemm"] = rmsnorm_gemm
