"""Generate the golden fixtures in tests/golden from the reference itself.

Run in a container that has the reference checkout, naming it as the
argument or in MOLTEN_REFERENCE:

    python tests/golden/make_golden.py REFERENCE_CHECKOUT

It imports the reference's own CPU semantics (``benchmarks/ops.py``) and its
front end (``molten/ir.py``, ``molten/fusion.py``, ``molten/compiler.py``)
from that checkout, evaluates them on small seeded inputs, and writes:

* ``<case>.npz``         inputs (bf16 as uint16 bits), the reference's fp32
                         result, and that result rounded to the output dtype;
* ``fusion_groups.json`` the reference FusionEngine's groups (op type names)
                         for every benchmark graph and every graph of the
                         reference's unit tests, plus ZeroCompiler._optimize
                         results.

The fixtures are committed; tests never read the reference checkout.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REF = None      # the reference checkout, set by main() from argv / MOLTEN_REFERENCE


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_modules():
    """(ops, ir, fusion, compiler) of the reference, imported by path."""
    # the reference package is also called `molten`; make sure its own
    # `from molten.ir import ...` statements resolve to the reference
    for k in [k for k in sys.modules if k == "molten" or k.startswith("molten.")]:
        del sys.modules[k]
    sys.path.insert(0, str(REF))
    try:
        import molten.ir as ir                 # noqa: E402
        import molten.fusion as fusion         # noqa: E402
        import molten.compiler as compiler     # noqa: E402
    finally:
        sys.path.pop(0)
    ops = _load("ref_ops", REF / "benchmarks" / "ops.py")
    assert Path(ir.__file__).resolve().is_relative_to(REF.resolve()), ir.__file__
    return ops, ir, fusion, compiler


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def normal(g, shape, mean=0.0, std=1.0, dtype=torch.float32):
    return (torch.randn(*shape, generator=g) * std + mean).to(dtype)


def uniform(g, shape, lo, hi, dtype):
    return (torch.rand(*shape, generator=g) * (hi - lo) + lo).to(dtype)


def causal(rows, cols, period=None):
    p = period or cols
    r = torch.arange(rows) % p
    c = torch.arange(cols)
    return torch.where(c[None, :] > r[:, None], torch.tensor(float("-inf")), torch.tensor(0.0))


def save(name, out_dtype, inputs: dict, ref_f32: torch.Tensor, meta: dict):
    d = {f"in_{k}": bits(v) for k, v in inputs.items()}
    d["ref_f32"] = ref_f32.float().numpy()
    rounded = ref_f32.to(out_dtype)
    d["ref_out"] = bits(rounded)
    d["meta"] = np.array(json.dumps(dict(meta, out_dtype=str(out_dtype).replace("torch.", ""),
                                         inputs=list(inputs))))
    np.savez_compressed(HERE / f"{name}.npz", **d)


def make_numeric(ops):
    bf16 = torch.bfloat16
    # 1) fused RMSNorm, fp32 (ops.py:13-16)
    g = gen(0)
    x = normal(g, (2, 5120))
    w = normal(g, (5120,), 1.0, 0.1)
    save("rmsnorm_f32", torch.float32, {"x": x, "w": w},
         ops.rmsnorm_pytorch(x, w, 1e-6), {"kind": "rmsnorm", "eps": 1e-6})
    # odd width and a single row
    g = gen(1)
    x = normal(g, (3, 1000))
    w = normal(g, (1000,), 1.0, 0.1)
    save("rmsnorm_f32_ragged", torch.float32, {"x": x, "w": w},
         ops.rmsnorm_pytorch(x, w, 1e-6), {"kind": "rmsnorm", "eps": 1e-6})
    # 2) RMSNorm * SiLU(gate), bf16 in, fp32 math (ops.py:38-42)
    for rows, seed in ((3, 0), (1, 2)):
        g = gen(seed)
        x = normal(g, (rows, 3584), dtype=bf16)
        w = normal(g, (3584,), 1.0, 0.1, dtype=bf16)
        gt = normal(g, (rows, 3584), dtype=bf16)
        ref = ops.fused_rmsnorm_silu_gate_pytorch(x.float(), w.float(), gt.float(), 1e-6)
        save(f"rmsnorm_silu_bf16_r{rows}", bf16, {"x": x, "w": w, "gate": gt}, ref,
             {"kind": "rmsnorm_silu_gate", "eps": 1e-6})
    # 3) softmax (ops.py:45-47), with and without the causal mask
    g = gen(0)
    x = normal(g, (6, 2048), 0.0, 3.0)
    save("softmax_f32", torch.float32, {"logits": x}, ops.softmax_pytorch(x),
         {"kind": "softmax", "causal": False})
    save("softmax_f32_causal", torch.float32, {"logits": x},
         ops.softmax_pytorch(x + causal(6, 2048)), {"kind": "softmax", "causal": True})
    g = gen(3)
    x = normal(g, (1, 32768), 0.0, 3.0)
    save("softmax_f32_long", torch.float32, {"logits": x}, ops.softmax_pytorch(x),
         {"kind": "softmax", "causal": False})
    g = gen(4)
    x = normal(g, (4, 2048), 0.0, 3.0, dtype=bf16)
    save("softmax_bf16_causal", bf16, {"logits": x},
         ops.softmax_pytorch(x.float() + causal(4, 2048)), {"kind": "softmax", "causal": True})
    # 4) 8-op elementwise chain, bf16 (GELU per ops.py:52, per-column
    #    broadcast per reference_kernels.cu:180-184)
    g = gen(0)
    x = normal(g, (2, 8192), dtype=bf16)
    r = normal(g, (2, 8192), dtype=bf16)
    a = uniform(g, (8192,), -1.0, 1.0, bf16)
    b = uniform(g, (8192,), -1.0, 1.0, bf16)
    s = uniform(g, (8192,), -1.0, 1.0, bf16)
    xf, rf = x.float(), r.float()
    y = F.gelu(xf * a.float() + b.float(), approximate="tanh") * s.float() + rf
    y = torch.clamp(y, -6.0, 6.0) * 0.5 + rf
    save("chain_bf16", bf16, {"x": x, "r": r, "a": a, "b": b, "s": s}, y, {"kind": "chain"})
    # gelu_add exactly as the reference's helper (ops.py:50-52)
    g = gen(5)
    x = normal(g, (4, 512))
    bias = normal(g, (512,))
    save("gelu_add_f32", torch.float32, {"x": x, "bias": bias}, ops.gelu_add_pytorch(x, bias),
         {"kind": "gelu_add"})
    # 5) MatMul + bias + GELU, bf16 in, fp32 accumulate (ops.py:58 matmul)
    g = gen(0)
    A = normal(g, (48, 256), dtype=bf16)
    B = normal(g, (256, 192), 0.0, (1.0 / 256) ** 0.5, dtype=bf16)
    bias = normal(g, (192,), 0.0, 0.02, dtype=bf16)
    ref = F.gelu(torch.matmul(A.double(), B.double()).float() + bias.float(), approximate="tanh")
    save("gemm_bias_gelu_bf16", bf16, {"A": A, "B": B, "bias": bias}, ref,
         {"kind": "gemm_bias_gelu"})
    # 6) RoPE exactly as the reference's helper (ops.py:24-35): x (batch,
    #    seq, heads, head_dim), cos/sin (seq, head_dim/2); fp32 tables
    g = gen(6)
    x = normal(g, (2, 16, 4, 64))
    ang = torch.rand(16, 32, generator=g) * 6.2831853
    cos, sin = torch.cos(ang), torch.sin(ang)
    save("rope_f32", torch.float32, {"x": x, "cos": cos, "sin": sin},
         ops.rope_pytorch(x, cos, sin), {"kind": "rope"})
    g = gen(7)
    x = normal(g, (1, 8, 8, 128), dtype=bf16)
    ang = torch.rand(8, 64, generator=g) * 6.2831853
    cos, sin = torch.cos(ang), torch.sin(ang)
    # the fp32 result before the helper's final cast to x.dtype
    save("rope_bf16", bf16, {"x": x, "cos": cos, "sin": sin},
         ops.rope_pytorch(x.float(), cos, sin), {"kind": "rope"})
    # 7) attention scores exactly as the reference's helper (ops.py:55-59),
    #    bf16 Q and K, fp32 arithmetic (fp64-accumulated product)
    g = gen(8)
    q = normal(g, (64, 128), dtype=bf16)
    k = normal(g, (192, 128), dtype=bf16)
    scale = 1.0 / 128 ** 0.5
    save("attention_score_bf16", bf16, {"q": q, "k": k},
         ops.attention_score_pytorch(q.double(), k.double(), scale).float(),
         {"kind": "attention_score", "scale": scale})


def make_fusion(ir, fusion, compiler):
    OT, TS, DG = ir.OpType, ir.TensorShape, ir.DataflowGraph

    def groups(g):
        eng = fusion.FusionEngine()
        return [[g.ops[i].op_type.name for i in grp.op_ids] for grp in eng.fuse(g)]

    cases = {}
    g = DG("rmsnorm")
    x = g.add_input("x", TS([2048, 5120]))
    w = g.add_input("w", TS([5120]))
    g.add_output(g.rms_norm(x, w, "norm"))
    cases["rmsnorm"] = groups(g)

    g = DG("rms_silu")
    x = g.add_input("x", TS([8192, 3584]))
    w = g.add_input("w", TS([3584]))
    gt = g.add_input("gate", TS([8192, 3584]))
    n = g.rms_norm(x, w, "norm")
    g.add_output(g.mul(n, g.add_op(OT.SILU, [gt], "silu"), "gated"))
    cases["rmsnorm_silu_gate"] = groups(g)

    g = DG("softmax")
    x = g.add_input("x", TS([32, 2048, 2048]))
    g.add_output(g.softmax(x))
    cases["softmax"] = groups(g)

    g = DG("softmax_causal")
    x = g.add_input("x", TS([32, 2048, 2048]))
    m = g.add_op(OT.CONSTANT, name="causal_mask", kind="causal_mask", period=None, offset=0, value=None)
    g.add_output(g.softmax(g.add(x, m)))
    cases["softmax_causal"] = groups(g)

    g = DG("chain")
    x = g.add_input("x", TS([16384, 8192]))
    r = g.add_input("r", TS([16384, 8192]))
    a = g.add_input("a", TS([8192]))
    b = g.add_input("b", TS([8192]))
    s = g.add_input("s", TS([8192]))
    half = g.add_constant("half", 0.5)
    t = g.mul(x, a)
    t = g.add(t, b)
    t = g.add_op(OT.GELU, [t])
    t = g.mul(t, s)
    t = g.add(t, r)
    t = g.add_op(OT.CLAMP, [t], min=-6.0, max=6.0)
    t = g.mul(t, half)
    t = g.add(t, r)
    g.add_output(t)
    cases["chain"] = groups(g)

    g = DG("gemm")
    A = g.add_input("A", TS([8192, 4096]))
    B = g.add_input("B", TS([4096, 14336]))
    bias = g.add_input("bias", TS([14336]))
    g.add_output(g.add_op(OT.GELU, [g.add(g.matmul(A, B), bias)]))
    cases["gemm_bias_gelu"] = groups(g)

    # the reference's unit-test graphs (tests/test_fusion.py, test_codegen.py)
    g = DG("elem_chain")
    x = g.add_input("x", TS([4, 8]))
    y = g.add_input("y", TS([4, 8]))
    g.add_output(g.add_op(OT.RELU, [g.mul(g.add(x, y), x)]))
    cases["elem_chain"] = groups(g)

    g = DG("two_matmul")
    x = g.add_input("x", TS([4, 8]))
    w1 = g.add_input("w1", TS([8, 16]))
    w2 = g.add_input("w2", TS([16, 8]))
    g.add_output(g.matmul(g.matmul(x, w1), w2))
    cases["two_matmul"] = groups(g)

    g = DG("matmul_epilogue")
    x = g.add_input("x", TS([4, 8]))
    w = g.add_input("w", TS([8, 16]))
    b = g.add_input("bias", TS([16]))
    g.add_output(g.add_op(OT.RELU, [g.add(g.matmul(x, w), b)]))
    cases["matmul_epilogue"] = groups(g)

    g = DG("transformer_block")
    x = g.add_input("x", TS([4, 512]))
    w = g.add_input("w", TS([512]))
    g.rms_norm(x, w, "norm")
    q = g.add_input("q", TS([4, 512]))
    k = g.add_input("k", TS([512, 4]))
    g.add_output(g.softmax(g.matmul(q, k)))
    cases["transformer_block"] = groups(g)

    # RMSNorm feeding a GEMM with a bias + GELU epilogue
    g = DG("norm_gemm")
    x = g.add_input("x", TS([256, 512]))
    w = g.add_input("w", TS([512]))
    B = g.add_input("B", TS([512, 384]))
    bias = g.add_input("bias", TS([384]))
    g.add_output(g.add_op(OT.GELU, [g.add(g.matmul(g.rms_norm(x, w, "norm"), B), bias)]))
    cases["norm_gemm"] = groups(g)

    # attention scores, ops.py:55-59: softmax(Q @ K^T * scale)
    g = DG("attention_score")
    q = g.add_input("q", TS([256, 128]))
    k = g.add_input("k", TS([512, 128]))
    kt = g.add_op(OT.TRANSPOSE, [k], "kT")
    sc = g.add_constant("scale", 0.08838834764831845)
    g.add_output(g.softmax(g.mul(g.matmul(q, kt), sc)))
    cases["attention_score"] = groups(g)

    # RoPE after RMSNorm (the reference builder's two-input rope, ir.py:175)
    g = DG("norm_rope")
    x = g.add_input("x", TS([2, 16, 4, 64]))
    w = g.add_input("w", TS([64]))
    f = g.add_input("freqs", TS([16, 64]))
    g.add_output(g.rope(g.rms_norm(x, w, "norm"), f))
    cases["norm_rope"] = groups(g)

    # mixed reductions with different dims, and a reduction feeding a matmul
    g = DG("mixed")
    x = g.add_input("x", TS([16, 32]))
    s1 = g.add_op(OT.SUM, [x])
    s1o = g.ops[s1]
    s1o.reduction_dim = -1
    e = g.add_op(OT.EXP, [x])
    s2 = g.add_op(OT.MAX, [e])
    g.ops[s2].reduction_dim = 0
    d = g.div(e, s1)
    mm = g.matmul(d, g.add_input("w", TS([32, 8])))
    g.add_output(mm)
    g.add_output(s2)
    cases["mixed_reductions"] = groups(g)

    # ZeroCompiler._optimize: constant folding and identity elimination
    opt = {}
    g = DG("opt")
    x = g.add_input("x", TS([4, 8]))
    one = g.add_constant("one", 1.0)
    zero = g.add_constant("zero", 0.0)
    c2 = g.add_constant("two", 2.0)
    c3 = g.add_constant("three", 3.0)
    five = g.add(c2, c3)
    t = g.mul(x, one)
    t = g.add(t, zero)
    t = g.mul(t, five)
    g.add_output(g.add_op(OT.RELU, [t]))
    zc = compiler.ZeroCompiler()
    g2 = zc._optimize(g)
    opt["ops"] = [[i, o.op_type.name, list(o.inputs), o.attrs.get("value")]
                  for i, o in sorted(g2.ops.items())]
    opt["groups"] = groups(g2)
    return {"groups": cases, "optimize": opt}


def main():
    global REF
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOLTEN_REFERENCE")
    if not arg:
        sys.exit("usage: make_golden.py REFERENCE_CHECKOUT (or set MOLTEN_REFERENCE)")
    REF = Path(arg)
    ops, ir, fusion, compiler = reference_modules()
    torch.manual_seed(0)
    make_numeric(ops)
    data = make_fusion(ir, fusion, compiler)
    (HERE / "fusion_groups.json").write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")), "and fusion_groups.json")


if __name__ == "__main__":
    main()
