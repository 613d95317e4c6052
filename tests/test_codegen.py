"""Code generation: reference-compatible surface, pattern families, and
that every emitted module compiles for sm_100a."""
import re

import pytest

from molten.codegen import CodeGenerator, GeneratedKernel, KernelConfig, compile_graph
from molten.compiler import ZeroCompiler
from molten.fusion import FusionEngine
from molten.ir import DataflowGraph, OpType, TensorShape
from molten_b200 import graphs
from molten_b200.build import build_cubin
from molten_b200.lowering import LoweringError

TS = TensorShape


def test_elementwise_kernel_source():
    g = DataflowGraph("add_relu")
    x = g.add_input("x", TS([1024]))
    y = g.add_input("y", TS([1024]))
    g.add_output(g.add_op(OpType.RELU, [g.add(x, y)]))
    ks = compile_graph(g)
    assert len(ks) >= 1
    k = ks[0]
    assert "molten_fused" in k.name and "__global__" in k.source and "fmaxf" in k.source
    assert k.plan.kernels[0].family == "ew"


def test_softmax_kernel_source():
    g = DataflowGraph("softmax")
    x = g.add_input("x", TS([32, 128]))
    g.add_output(g.softmax(x))
    src = compile_graph(g)[0].source
    assert "__shared__" in src and "expf" in src


def test_matmul_kernel_source():
    g = DataflowGraph("gemm")
    a = g.add_input("a", TS([64, 128]))
    b = g.add_input("b", TS([128, 64]))
    g.add_output(g.matmul(a, b))
    k = compile_graph(g)[0]                   # the reference's default: fp32
    assert "TILE" in k.source and "__syncthreads" in k.source
    assert "gemm_roles<" in k.source and "molten/gemm_sm100.cuh" in k.source
    assert k.config.block_size_y > 1          # the reference's "matmul" marker
    # fp32 operands: split into bf16 planes, then the bf16x3 tensor-core GEMM
    assert [sk.family for sk in k.plan.kernels] == ["split3", "split3", "gemm"]
    assert k.plan.kernels[2].config["split3"]
    kb = compile_graph(g, dtype="bfloat16")[0]
    assert [sk.family for sk in kb.plan.kernels] == ["gemm"]


def test_rms_norm_kernel_and_transformer_block():
    g = DataflowGraph("rmsnorm")
    x = g.add_input("x", TS([4, 512]))
    w = g.add_input("w", TS([512]))
    g.rms_norm(x, w, "norm")          # no add_output: the sink is the output
    ks = compile_graph(g)
    assert len(ks) == 1 and ks[0].config.shared_mem_bytes > 0

    g = DataflowGraph("transformer_block")
    x = g.add_input("x", TS([4, 512]))
    w = g.add_input("w", TS([512]))
    g.rms_norm(x, w, "norm")
    q = g.add_input("q", TS([4, 512]))
    k = g.add_input("k", TS([512, 4]))
    g.add_output(g.softmax(g.matmul(q, k)))
    ks = compile_graph(g)
    assert len(ks) >= 1 and all(k.source and k.name for k in ks)
    # MATMUL -> SOFTMAX is one fusion group run as GEMM + row kernel (fp32:
    # after the kernels that split q and k into bf16 planes)
    fams = [sk.family for sk in ks[1].plan.kernels]
    assert fams == ["split3", "split3", "gemm", "row"] and "_k0" in ks[1].source \
        and "_k3" in ks[1].source
    fams = [sk.family for sk in compile_graph(g, dtype="bfloat16")[1].plan.kernels]
    assert fams == ["gemm", "row"]


def test_names_follow_reference_rule():
    assert compile_graph(graphs.rmsnorm_silu_gate(4, 64, dtype="bfloat16"),
                         dtype="bfloat16")[0].name == "molten_fused_rms_div_mul_silu"
    assert compile_graph(graphs.chain(4, 64), dtype="bfloat16")[0].name == \
        "molten_fused_mul_add_gelu_clamp"


@pytest.mark.parametrize("kind,args,fam,engine", [
    ("rmsnorm", (2048, 5120), "row", "tma"),
    ("rmsnorm", (1024, 5120), "row", "regs"),
    ("rmsnorm_silu_gate", (2048, 3584), "row", "tma"),
    ("rmsnorm_silu_gate", (8192, 3584), "row", "tma"),
    ("rmsnorm_silu_gate", (1, 3584), "row", "regs"),
    ("softmax", ((32, 2048, 2048),), "row", "regs"),
    ("chain", (64, 8192), "ew", None),
    ("chain", (16384, 8192), "row", "tma"),
    ("gemm_bias_gelu", (8192, 4096, 14336), "gemm", None),
])
def test_families(kind, args, fam, engine):
    """Pattern family and engine per benchmark graph: row counts from 2048
    on (elementwise groups from 4096 on) stream through the TMA ring, the
    rest keep rows in registers."""
    dt = "float32" if kind in ("rmsnorm", "softmax") else "bfloat16"
    g = graphs.BUILDERS[kind](*args, dtype=dt)
    ks = compile_graph(g, dtype=dt)
    assert len(ks) == 1 and [sk.family for sk in ks[0].plan.kernels] == [fam]
    assert ks[0].plan.kernels[0].config.get("engine") == engine


def test_specialised_dtypes_and_promotion():
    g = graphs.rmsnorm(8, 64)
    grp = FusionEngine().fuse(g)[0]
    gen = CodeGenerator()
    k = gen.generate(g, grp, {0: (8, 64), 1: (64,)}, {0: "bfloat16", 1: "float32"})
    assert k.plan.output_dtypes == ["float32"]           # bf16 x fp32 -> fp32
    assert "const bf16*" in k.source and "float* __restrict__ out0" in k.source


def test_long_rows_use_a_cluster():
    """Rows needing more than 1024 threads run on a cluster; fp32 rows of
    513..1024 threads on one 1024-thread CTA."""
    g = graphs.softmax((64, 65536))
    k = compile_graph(g)[0]
    sk = k.plan.kernels[0]
    assert sk.config["cl"] > 1 and k.config.cluster_x == sk.config["cl"]
    for causal in (False, True):
        g = graphs.softmax((4096, 32768), causal=causal)
        k = CodeGenerator(tune={"row": {"causal_split": False}}).generate(g, FusionEngine().fuse(g)[0])
        sk = k.plan.kernels[0]
        assert (sk.config["tpc"], sk.config["cl"], sk.config["block"]) == (1024, 1, 1024)
        assert k.config.cluster_x == 1 and not sk.config.get("stream")


def test_silu_of_the_gate_is_computed_in_the_reduction_pass():
    """RMSNorm * SiLU(gate) in the register engine: silu(gate) depends only on
    the row's own elements, so it is computed next to the sum of squares and
    kept in registers for the output pass."""
    (k,) = compile_graph(graphs.rmsnorm_silu_gate(1024, 3584), dtype="bfloat16")
    c = k.plan.kernels[0].config
    assert c["engine"] == "regs" and len(c["materialize"]) == 1 and c["materialize"][0][1] == 0
    body = k.source.split("// ---- pass 0")[1].split("// ---- final pass")[0]
    assert "m_silu<" in body and "m_silu<" not in k.source.split("// ---- final pass")[1]
    # a plain RMSNorm has nothing to compute early
    (k,) = compile_graph(graphs.rmsnorm(1024, 5120))
    assert k.plan.kernels[0].config["materialize"] == []
    # the TMA ring with teams of warps keeps it too (5 slots per lane)
    (k,) = compile_graph(graphs.rmsnorm_silu_gate(2048, 3584), dtype="bfloat16")
    c = k.plan.kernels[0].config
    assert c["engine"] == "tma" and c["tw"] > 1 and len(c["materialize"]) == 1
    assert "team_allreduce<0, 1, TW>" in k.source


def test_causal_zero_tail_selection():
    """Bulk zero stores for the masked row tails of a causal softmax: in the
    register form with one team of >= 256 threads per CTA, not in the
    bulk-staged stream form, not for short rows (several rows per CTA).
    (Long causal rows default to the split causal kernel; the row engine's
    forms are asked for here.)"""
    def row_engine(g, dt="float32"):
        gen = CodeGenerator(dtype=dt, tune={"row": {"causal_split": False}})
        return gen.generate(g, FusionEngine().fuse(g)[0]).source
    src = row_engine(graphs.softmax((4096, 32768), causal=True))
    assert "bulk_zero_tail" in src and "bulk_zero_drain" in src and "zero_shared_for_bulk" in src
    src = row_engine(graphs.softmax((4096, 32768), dtype="bfloat16", causal=True), "bfloat16")
    assert "bulk_zero_tail" not in src and "store_zero_slot" in src
    src = compile_graph(graphs.softmax((65536, 2048), causal=True))[0].source
    assert "bulk_zero_tail" not in src
    src = compile_graph(graphs.softmax((4096, 32768)))[0].source       # no mask, no tail
    assert "bulk_zero_tail" not in src and "zbuf" not in src


def test_long_16bit_rows_take_the_stream_form():
    """bf16 rows long enough for a cluster run as one CTA per row (512
    threads when 8 slots per thread hold the row) in the persistent stream
    form; fp32 rows as one 1024-thread CTA in the register form."""
    sk = compile_graph(graphs.softmax((4096, 32768), dtype="bfloat16"), dtype="bfloat16")[0] \
        .plan.kernels[0]
    assert (sk.config["tpc"], sk.config["cl"], sk.config["stream"], sk.config["nv"]) == (512, 1, 3, 8)
    assert sk.config["bulk"] and sk.config["smem"] == 3 * 32768 * 2
    sk = compile_graph(graphs.softmax((4096, 32768)))[0].plan.kernels[0]
    assert sk.config["cl"] == 1 and not sk.config.get("stream")


def test_stream_forms_compile_for_sm100a(tmp_path):
    """Stream kernels: per-thread cp.async staging, row-invariant operands
    hoisted, cluster partials pushed with st.async (cl > 1)."""
    cases = [
        (graphs.softmax((300, 32768), dtype="bfloat16", causal=True), {"stream": 3}, "bfloat16"),
        (graphs.rmsnorm(999, 8192), {"stream": 3, "engine": "regs", "tpc": 128, "cl": 4}, "float32"),
        (graphs.rmsnorm_silu_gate(1000, 3584), {"stream": 4, "engine": "regs"}, "bfloat16"),
    ]
    for g, tune, dt in cases:
        grp = FusionEngine().fuse(g)[0]
        ins = sorted(i for i, o in g.ops.items() if o.op_type.name == "INPUT")
        shapes = {i: tuple(g.ops[i].shape.dims) for i in ins}
        k = CodeGenerator(tune={"row": tune}).generate(g, grp, shapes, {i: dt for i in ins})
        c = k.plan.kernels[0].config
        assert c["stream"] >= 2
        assert "cp_async16" in k.source
        assert ("reduce_push" in k.source or "reduce_softmax_push" in k.source) == (c["cl"] > 1)
        assert build_cubin(k.source, k.name, tmp_path).stat().st_size > 1000


def test_fp16_flag_and_save(tmp_path):
    g = graphs.rmsnorm(8, 256)
    kernels = ZeroCompiler(fp16=True).compile(g)
    assert "f16" in kernels[0].source
    ZeroCompiler().save(kernels, str(tmp_path))
    assert (tmp_path / f"{kernels[0].name}.cu").exists()
    assert (tmp_path / "molten_generated.h").read_text().startswith("#pragma once")
    assert (tmp_path / "molten" / "row_engine.cuh").exists()


def test_unsupported_ops_raise():
    g = DataflowGraph("transpose")
    x = g.add_input("x", TS([4, 8]))
    g.add_output(g.add_op(OpType.TRANSPOSE, [x]))
    with pytest.raises(LoweringError):
        compile_graph(g)


def test_rope_shapes_are_checked():
    g = DataflowGraph("rope2d")
    x = g.add_input("x", TS([4, 8]))
    f = g.add_input("f", TS([4, 8]))
    g.add_output(g.rope(x, f))
    with pytest.raises(LoweringError):          # x must be [..., seq, heads, head_dim]
        compile_graph(g)
    g = DataflowGraph("rope_bad_table")
    x = g.add_input("x", TS([1, 16, 4, 64]))
    c = g.add_input("cos", TS([16, 64]))
    sn = g.add_input("sin", TS([16, 32]))
    g.add_output(g.rope(x, c, sin=sn))
    with pytest.raises(LoweringError):
        compile_graph(g)


@pytest.mark.parametrize("style,packed", [(None, False), ("half", False), (None, True),
                                          ("half", True)])
def test_rope_kernels(tmp_path, style, packed):
    g = graphs.rope(2, 64, 8, 128, style=style, packed=packed)
    ins = sorted(i for i, o in g.ops.items() if o.op_type == OpType.INPUT)
    dts = {ins[0]: "bfloat16", **{i: "float32" for i in ins[1:]}}
    k = CodeGenerator().generate(g, FusionEngine().fuse(g)[0],
                                 {i: tuple(g.ops[i].shape.dims) for i in ins}, dts)
    (sk,) = k.plan.kernels
    assert sk.family == "rope" and k.plan.output_dtypes == ["bfloat16"]   # out.to(x.dtype)
    assert sk.config["vec"] == 8 and not sk.config["scalar"]
    assert "pdl_enter" in k.source and "% SEQ" in k.source
    assert build_cubin(k.source, k.name, tmp_path).stat().st_size > 1000


def test_attention_score_plan(tmp_path):
    """[TRANSPOSE, MATMUL, MUL, SOFTMAX] (one group, as the reference fuses
    it) runs as one fused kernel: K read K-major, scale * log2(e) baked in,
    two tensor-core passes, TMA stores of the probabilities."""
    (k,) = compile_graph(graphs.attention_score(256, 512, 128), dtype="bfloat16")
    assert k.name == "molten_fused_transpose_matmul_mul_softmax"
    (sk,) = k.plan.kernels
    assert sk.family == "attn" and (sk.m, sk.n, sk.k) == (256, 512, 128)
    c = sk.config
    assert c["bn"] == 256 and c["dch"] == 2 and c["tma_store"] and c["batch"] == 1
    assert c["smem_bytes"] <= 232448 and abs(c["scale"] - 128 ** -0.5) < 1e-12
    assert "attn_roles<" in k.source and ", bf16, true, true, 0, 0, false, false>(sh, args," in k.source
    rec = k.config.launches[0]
    assert rec["family"] == "attn" and rec["smem"] == c["smem_bytes"]
    assert build_cubin(k.source, k.name, tmp_path).stat().st_size > 1000


def test_attention_score_store_paths():
    """TMA stores need 16-byte rows (n % 8 == 0) and store boxes that stay in
    one head (m % 32 == 0, or a single head); otherwise direct stores."""
    def cfg(**kw):
        (k,) = compile_graph(graphs.attention_score(**kw), dtype="bfloat16")
        return k.plan.kernels[0].config
    assert cfg(m=96, n=136, d=128, heads=5)["tma_store"]
    assert not cfg(m=200, n=300, d=64, heads=3)["tma_store"]          # m % 32
    assert cfg(m=200, n=304, d=64)["tma_store"]                        # one head: clipped
    c = cfg(m=100, n=77, d=72)
    assert not c["tma_store"] and not c["rows_aligned"]
    assert c["bn"] == 128 and c["dch"] == 2
    assert cfg(m=64, n=1000, d=256, heads=2)["stages"] == 2
    assert cfg(m=64, n=1000, d=128)["stages"] == 3


def test_attention_score_unfused_plan(tmp_path):
    """With {"attn": {"fused": False}}: a K-major-B GEMM with the scale in
    its epilogue, then a row softmax; the TRANSPOSE is no kernel."""
    g = graphs.attention_score(256, 512, 128)
    k = CodeGenerator(dtype="bfloat16", tune={"attn": {"fused": False}}).generate(
        g, FusionEngine().fuse(g)[0])
    gemm, row = k.plan.kernels
    assert gemm.family == "gemm" and gemm.config["b_kmajor"] and (gemm.m, gemm.n, gemm.k) == (256, 512, 128)
    assert row.family == "row"
    assert ", true, NoPrologue, false>(sh, args)" in k.source
    assert build_cubin(k.source, k.name, tmp_path).stat().st_size > 1000


def test_attention_pattern_needs_the_exact_group():
    """Only softmax(matmul(q, transpose(k)) [* constant]) fuses; a tensor
    scale or an extra output keeps the two-kernel form."""
    g = DataflowGraph("s")
    q = g.add_input("q", TS([128, 64]), dtype="bfloat16")
    kk = g.add_input("k", TS([256, 64]), dtype="bfloat16")
    sc = g.add_input("sc", TS([256]), dtype="bfloat16")
    g.add_output(g.softmax(g.mul(g.matmul(q, g.transpose(kk)), sc)))
    (k,) = compile_graph(g, dtype="bfloat16")
    assert [sk.family for sk in k.plan.kernels] == ["gemm", "row"]
    g = DataflowGraph("s2")
    q = g.add_input("q", TS([128, 64]), dtype="bfloat16")
    kk = g.add_input("k", TS([256, 64]), dtype="bfloat16")
    g.add_output(g.softmax(g.matmul(q, g.transpose(kk))))
    (k,) = compile_graph(g, dtype="bfloat16")
    assert [sk.family for sk in k.plan.kernels] == ["attn"]
    assert k.plan.kernels[0].config["scale"] == 1.0
    (k,) = compile_graph(graphs.attention_score(64, 64, 64, scale=-0.5), dtype="bfloat16")
    assert [sk.family for sk in k.plan.kernels] == ["gemm", "row"]     # max of raw scores needs scale > 0


def test_transpose_elsewhere_is_rejected():
    g = DataflowGraph("t")
    x = g.add_input("x", TS([8, 16]))
    g.add_output(g.relu(g.transpose(x)))
    with pytest.raises(LoweringError):
        compile_graph(g)


def test_rope_after_rmsnorm_splits_the_group():
    """The reference fuses [RMS, DIV, MUL, ROTATE] into one group; it runs as
    a row kernel and a RoPE kernel with an fp32 intermediate."""
    g = DataflowGraph("norm_rope")
    x = g.add_input("x", TS([2, 16, 4, 64]))
    w = g.add_input("w", TS([64]))
    f = g.add_input("freqs", TS([16, 64]))
    g.add_output(g.rope(g.rms_norm(x, w, "norm"), f))
    (k,) = compile_graph(g, dtype="bfloat16")
    assert [sk.family for sk in k.plan.kernels] == ["row", "rope"]
    assert [d for _, d in k.plan.temps.values()] == ["float32"]
    assert k.name == "molten_fused_rms_div_mul_rotate"


def test_float32_gemm_runs_as_bf16_planes():
    """fp32 GEMM operands (the reference's default dtype) are split into
    three bf16 planes by a kernel each, then the tensor-core GEMM takes the
    six plane products; an fp32 x bf16 pair is split too, bf16 x fp16 is not
    a GEMM the tensor cores take, and the RMSNorm prologue wants 16-bit x."""
    g = graphs.gemm_bias_gelu(64, 64, 64, dtype="float32")
    (k,) = compile_graph(g, dtype="float32")
    split_a, split_b, gemm = k.plan.kernels
    assert (split_a.family, split_b.family, gemm.family) == ("split3", "split3", "gemm")
    assert gemm.config["split3"] and not gemm.config["streamk"]
    assert k.plan.temps[gemm.config["planes"][0]] == ((3, 64, 64), "bfloat16")
    assert "split3_value" in k.source and ", true>(sh, args)" in k.source
    gen = CodeGenerator()
    grp = FusionEngine().fuse(g)[0]
    mixed = gen.generate(g, grp, {0: (64, 64), 1: (64, 64), 2: (64,)},
                         {0: "float32", 1: "bfloat16", 2: "float32"})
    assert [sk.family for sk in mixed.plan.kernels] == ["split3", "split3", "gemm"]
    with pytest.raises(LoweringError):
        gen.generate(g, grp, {0: (64, 64), 1: (64, 64), 2: (64,)},
                     {0: "bfloat16", 1: "float16", 2: "float32"})
    gn = graphs.rmsnorm_gemm(64, 64, 64, dtype="float32")
    with pytest.raises(LoweringError):
        CodeGenerator(dtype="float32", tune={"gemm": {"prologue": True}}).generate(
            gn, FusionEngine().fuse(gn)[0])


def _all_pattern_sources():
    out = []
    for name, g, dt in [
        ("rmsnorm", graphs.rmsnorm(), "float32"),
        ("rmsnorm_ragged", graphs.rmsnorm(3, 1000), "float32"),
        ("rms_silu", graphs.rmsnorm_silu_gate(), "bfloat16"),
        ("softmax", graphs.softmax(), "float32"),
        ("softmax_causal_bf16", graphs.softmax(causal=True), "bfloat16"),
        ("softmax_long", graphs.softmax((4096, 32768), causal=True), "float32"),
        ("chain", graphs.chain(), "bfloat16"),
        ("gemm_f32", graphs.gemm_bias_gelu(256, 512, 384, dtype="float32"), "float32"),
        ("gemm", graphs.gemm_bias_gelu(), "bfloat16"),
    ]:
        out.append((name, compile_graph(g, dtype=dt)[0]))
    return out


def test_every_pattern_compiles_for_sm100a(tmp_path):
    from concurrent.futures import ThreadPoolExecutor
    items = _all_pattern_sources()
    with ThreadPoolExecutor(4) as ex:
        cubins = list(ex.map(lambda it: build_cubin(it[1].source, it[1].name, tmp_path), items))
    for c in cubins:
        assert c.exists() and c.stat().st_size > 1000


def test_alignment_rules():
    from molten_b200.runtime import _alignment_rules
    g = graphs.rmsnorm_silu_gate(4, 64, dtype="bfloat16")
    grp = FusionEngine().fuse(g)[0]
    shapes = {0: (4, 64), 1: (64,), 2: (4, 64)}
    dts = {i: "bfloat16" for i in shapes}
    sk = CodeGenerator().generate(g, grp, shapes, dts).plan.kernels[0]
    assert _alignment_rules(sk) == ([16, 16, 16], [16])
    sk = CodeGenerator(tune={"row": {"vec": 1}}).generate(g, grp, shapes, dts).plan.kernels[0]
    assert _alignment_rules(sk) == ([2, 2, 2], [2])
    # the TMA ring engine is opt-in and never used with a vec override
    sk = CodeGenerator(tune={"row": {"engine": "tma", "vec": 1}}).generate(g, grp, shapes, dts)
    assert sk.plan.kernels[0].config["engine"] == "regs"
    sk = CodeGenerator(tune={"row": {"engine": "tma"}}).generate(g, grp, shapes, dts)
    assert sk.plan.kernels[0].config["engine"] == "tma"
    assert _alignment_rules(sk.plan.kernels[0])[0] == [16, 16, 16]


def test_exp2_poly3_error_bound():
    """The FMA-pipe 2^x of molten/common.cuh, evaluated step by step in fp32
    exactly as the device does (round-to-nearest adds, fused multiply-adds,
    exponent added as an integer): relative error below 1e-4 on [-126, 1],
    and the clamp keeps results positive and tiny below -126."""
    import numpy as np
    from molten_b200.build import ENGINE_INCLUDE
    src = (ENGINE_INCLUDE / "molten" / "common.cuh").read_text()
    c = [np.float32(float(re.search(rf"#define MOLTEN_EXP2_C{i} ([0-9.e+-]+)f", src).group(1)))
         for i in range(4)]

    def fma(a, b, d):        # one rounding, as the device's FFMA
        return np.float32(a.astype(np.float64) * b.astype(np.float64) + d.astype(np.float64))

    x = np.concatenate([np.linspace(-126, 1, 2_000_001, dtype=np.float32),
                        np.float32(-126) - np.arange(1, 100, dtype=np.float32)])
    xc = np.maximum(x, np.float32(-126))
    magic = np.float32(12582912.0)
    r = (xc + magic).astype(np.float32)
    f = (xc - (r - magic)).astype(np.float32)
    p = fma(fma(fma(np.full_like(f, c[3]), f, np.full_like(f, c[2])), f, np.full_like(f, c[1])),
            f, np.full_like(f, c[0]))
    bits = (p.view(np.int32).astype(np.int64) + (r.view(np.int32).astype(np.int64) << 23)) % (1 << 32)
    y = bits.astype(np.uint32).view(np.float32).astype(np.float64)
    assert np.all(np.abs(f) <= 0.5)
    ok = x >= -125
    rel = np.abs(y[ok] / np.exp2(x[ok].astype(np.float64)) - 1)
    assert rel.max() < 1e-4, rel.max()
    assert np.all(y[x < -126] >= 0) and np.all(y[x < -126] < 2.0 ** -125)


def test_gemm_sm_pair_plan(tmp_path):
    """From 1024 stacked rows the GEMM runs on SM pairs (clusters of 2 CTAs,
    tcgen05.mma.cta_group::2, 256-row tiles); decode-size GEMMs and the
    RMSNorm prologue keep the one-SM engine."""
    (k,) = compile_graph(graphs.gemm_bias_gelu(8192, 4096, 14336), dtype="bfloat16")
    c = k.plan.kernels[0].config
    assert c["pair"] and c["bm"] == 256 and c["bn"] == 256 and c["smem_bytes"] <= 232448
    assert "gemm2_roles<" in k.source and "molten/gemm2_sm100.cuh" in k.source
    assert build_cubin(k.source, k.name, tmp_path).stat().st_size > 1000
    (k,) = compile_graph(graphs.gemm_bias_gelu(64, 4096, 14336), dtype="bfloat16")
    assert not k.plan.kernels[0].config["pair"]
    g = graphs.rmsnorm_gemm(2048, 1024, 1024)
    k = CodeGenerator(dtype="bfloat16", tune={"gemm": {"prologue": True}}).generate(
        g, FusionEngine().fuse(g)[0])
    (sk,) = k.plan.kernels
    assert sk.config.get("prologue") and not sk.config["pair"]


def test_run_host_row_split_rules():
    """run_host splits 2-D row-indexed inputs by rows; row-invariant inputs
    (weights, GEMM B) go up whole; attention and 4-D RoPE run as one block."""
    import torch
    from molten_b200.runtime import CompiledKernel

    def flags(g, tensors, dtype="bfloat16"):
        (k,) = compile_graph(g, dtype=dtype)
        return CompiledKernel(name=k.name, source=k.source, config=k.config, kernel=k).row_chunkable(tensors)

    e = lambda *s: torch.empty(*s)
    assert flags(graphs.rmsnorm_silu_gate(64, 256), [e(64, 256), e(256), e(64, 256)]) == [True, False, True]
    assert flags(graphs.softmax((96, 256), causal=True), [e(96, 256)], "float32") == [True]
    assert flags(graphs.gemm_bias_gelu(128, 64, 64), [e(128, 64), e(64, 64), e(64)]) == [True, False, False]
    assert flags(graphs.attention_score(64, 64, 64), [e(64, 64), e(64, 64)]) is None
    assert flags(graphs.rope(1, 16, 4, 128), [e(1, 16, 4, 128), e(16, 64), e(16, 64)]) is None


def test_host_row_blocks():
    """Row blocks of a host-buffer call tile the rows in order; the last
    two are 3/4 and 1/4 of a regular block; no block is empty."""
    from molten_b200.runtime import host_row_blocks
    assert host_row_blocks(8192, 5) == [(0, 2048), (2048, 4096), (4096, 6144), (6144, 7680),
                                        (7680, 8192)]
    assert host_row_blocks(100, 1) == [(0, 100)] and host_row_blocks(100, 2) == [(0, 50), (50, 100)]
    for rows in (1, 2, 3, 7, 1000, 8193):
        for chunks in (1, 2, 3, 4, 5, 8, 16):
            b = host_row_blocks(rows, chunks)
            assert b[0][0] == 0 and b[-1][1] == rows and all(r1 > r0 for r0, r1 in b)
            assert all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))


def test_stream_k_plan():
    """Stream-K for GEMMs with at most half the SMs' worth of tiles, a long
    K and few rows, with at most SK_MAX_PIECES CTAs per tile; the workspace
    slot count follows the device's range arithmetic."""
    from molten_b200.gemm_config import SK_MAX_PIECES, stream_k_max_segments
    (k,) = compile_graph(graphs.gemm_bias_gelu(16, 8192, 1024), dtype="bfloat16")
    c = k.plan.kernels[0].config
    assert c["streamk"] and c["sk_ctas"] == 148 and c["sk_tiles"] == 16
    assert c["sk_maxseg"] == stream_k_max_segments(16, 128, 148) <= SK_MAX_PIECES + 1
    assert "gemm_sk_roles<" in k.source and "molten/gemm_sk_sm100.cuh" in k.source
    assert k.config.launches[0]["family"] == "gemm"
    assert k.config.launches[0]["grid"] == 148
    (k,) = compile_graph(graphs.gemm_bias_gelu(1, 4096, 256), dtype="bfloat16")
    c = k.plan.kernels[0].config
    assert c["streamk"] and c["sk_tiles"] == 4 and c["sk_ctas"] == 4 * SK_MAX_PIECES
    # decode 64 x 4096 x 14336 has 112 tiles: the plain persistent kernel
    for big in [(64, 4096, 14336), (64, 4096, 8192), (8192, 4096, 14336), (256, 512, 384),
                (1024, 256, 512)]:
        (k,) = compile_graph(graphs.gemm_bias_gelu(*big), dtype="bfloat16")
        assert not k.plan.kernels[0].config["streamk"], big
    # every tile is covered by owner(last) - owner(first) + 1 CTAs, at most 2
    # when each CTA has at least one tile's worth of k-blocks
    assert stream_k_max_segments(100, 64, 148) <= 3
    assert stream_k_max_segments(148, 10, 148) == 1


def test_causal_softmax_split_plan():
    """softmax(x + causal_mask) over long rows plans as the split causal
    kernel (row CTAs + zero tiles); short rows, explicit row-engine tunes,
    masks that could hide a whole row, and anything else in the group keep
    the row engine."""
    g = graphs.softmax((4096, 32768), dtype="bfloat16", causal=True)
    (k,) = compile_graph(g, dtype="bfloat16")
    (sk,) = k.plan.kernels
    assert sk.family == "causal" and sk.config["zt"] == 4 and sk.config["zcols"] == 8192
    assert "causal_softmax_cta<bf16, 256, 32768LL, 32768LL, 0LL, 4, 8192LL, false, true, true, 0>" in k.source
    assert k.config.family == "row" and k.config.shared_mem_bytes > 0
    k32 = compile_graph(graphs.softmax((4096, 32768), causal=True))[0]
    # fp32 rows too take the EX2-unit exponentials (within the fp32 bar)
    assert k32.plan.kernels[0].config["zt"] == 8 and not k32.plan.kernels[0].config["precise"]
    assert compile_graph(graphs.softmax((32, 2048, 2048), dtype="bfloat16", causal=True),
                         dtype="bfloat16")[0].plan.kernels[0].family == "row"
    gen = CodeGenerator(dtype="bfloat16", tune={"row": {"stream": 3}})
    assert gen.generate(g, FusionEngine().fuse(g)[0]).plan.kernels[0].family == "row"
    gn = DataflowGraph("neg")
    x = gn.add_input("x", TS([4096, 32768]), dtype="bfloat16")
    gn.add_output(gn.softmax(gn.add(x, gn.causal_mask(offset=-1)), -1))
    assert compile_graph(gn, dtype="bfloat16")[0].plan.kernels[0].family == "row"
    gs = DataflowGraph("scaled")
    x = gs.add_input("x", TS([4096, 32768]), dtype="bfloat16")
    gs.add_output(gs.softmax(gs.add(gs.mul(x, gs.add_constant("half", 0.5)), gs.causal_mask()), -1))
    assert compile_graph(gs, dtype="bfloat16")[0].plan.kernels[0].family == "row"


def test_ring_selection_rules():
    """TMA-ring choices: teams whose last slot round wastes at most 10%,
    one warp per row for long row counts of rows of at most 14 slots a
    lane, elementwise groups only with rows of >= 8 KB, 4..8 teams before
    fewer, the ring from 6 stages."""
    def cfg(g, dt="bfloat16", tune=None):
        (k,) = compile_graph(g, dtype=dt) if tune is None else \
            [CodeGenerator(dtype=dt, tune=tune).generate(g, FusionEngine().fuse(g)[0])]
        return k.plan.kernels[0].family, k.plan.kernels[0].config
    fam, c = cfg(graphs.rmsnorm_silu_gate(8192, 3584))
    assert (c["engine"], c["nc"], c["tw"], c["stages"]) == ("tma", 7, 1, 14)     # the headline
    fam, c = cfg(graphs.rmsnorm_silu_gate(2048, 3584))
    assert (c["engine"], c["nc"], c["tw"]) == ("tma", 7, 3)                      # 7% waste
    fam, c = cfg(graphs.rmsnorm_silu_gate(2048, 4096))
    assert (c["nc"], c["tw"]) == (6, 4)                                          # 3 would waste 12.5%
    fam, c = cfg(graphs.rmsnorm_silu_gate(8192, 4096))
    assert c["engine"] == "tma" and c["tw"] == 4                                 # 16 slots a lane: teams
    fam, c = cfg(graphs.rmsnorm_silu_gate(2048, 8192))
    assert c["engine"] == "tma" and c["stages"] == 6
    fam, c = cfg(graphs.rmsnorm(2048, 4096), "float32")
    assert (c["nc"], c["stages"]) == (6, 12)                                     # not 1 team on 13
    fam, c = cfg(graphs.rmsnorm_silu_gate(1024, 3584))
    assert c["engine"] == "regs"                                                 # below 2048 rows
    fam, c = cfg(graphs.chain(4096, 4096))
    assert fam == "row" and c["engine"] == "tma"                                 # 8 KB rows
    fam, c = cfg(graphs.chain(8192, 2048))
    assert fam == "ew"                                                           # 4 KB rows
    fam, c = cfg(graphs.rmsnorm_silu_gate(2048, 3584), tune={"row": {"tw": 2, "nc": 14}})
    assert (c["nc"], c["tw"], c["stages"]) == (14, 2, 14)


def test_fp32_softmax_exponentials():
    """fp32 softmax: per-element exponentials on the EX2 unit with the max
    subtracted first, the once-per-thread scale with expf; 16-bit outputs
    fold the max into one FFMA."""
    src32 = compile_graph(graphs.softmax((64, 2048)))[0].source
    assert "fast_exp2((" in src32 and "- lz" in src32 and "expf(lm" in src32
    src16 = compile_graph(graphs.softmax((64, 2048), dtype="bfloat16"), dtype="bfloat16")[0].source
    assert "fast_exp2(fmaf(" in src16 and "expf(" not in src16.replace("__expf(", "")
    # the split causal kernel takes the fast form for every output type
    k = compile_graph(graphs.softmax((4096, 32768), causal=True))[0]
    assert k.plan.kernels[0].family == "causal" and not k.plan.kernels[0].config["precise"]


def test_empty_shapes():
    """A MATMUL with an empty dimension is refused with a clear error; row
    and elementwise groups with no rows or no columns compile to a kernel
    that launches nothing (no cubin is built)."""
    from molten_b200.lowering import LoweringError
    from molten_b200.runtime import MoltenRuntime, _empty_outputs
    for m, k, n in ((0, 256, 512), (64, 0, 512), (64, 256, 0)):
        with pytest.raises(LoweringError, match="empty dimension"):
            compile_graph(graphs.gemm_bias_gelu(m, k, n), dtype="bfloat16")
    for g, dt in ((graphs.rmsnorm_silu_gate(0, 3584), "bfloat16"), (graphs.rmsnorm(4, 0), "float32"),
                  (graphs.chain(0, 1024), "bfloat16"), (graphs.softmax((0, 2048)), "float32")):
        (k,) = compile_graph(g, dtype=dt)
        assert _empty_outputs(k)
        ck = MoltenRuntime().compile(k)            # no nvcc run for an empty specialisation
        assert ck._module == "None"
    assert not _empty_outputs(compile_graph(graphs.rmsnorm(4, 64))[0])
