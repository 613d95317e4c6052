"""Parity of the sm_100a kernels with the oracle, on a B200.

Every call goes through MoltenRuntime -> libmolten_rt.so (molten_launch).
Bars (tests/_golden.assert_close): fp32 within 1e-5 relative, bf16 within
1e-2 relative of the fp32-accumulated reference.

* golden cases: the exact inputs of tests/golden, checked against the
  reference's own results;
* full-size benchmark workloads: rows are independent, so a seeded sample of
  rows is checked against the oracle, plus size-independent properties
  (softmax rows sum to 1 and masked entries are exactly 0, repeated runs are
  bit-identical, the GEMM's bounded waits never time out);
* edge cases: one row, ragged widths, misaligned pointers, GEMM shapes that
  are not tile multiples, row-sharded launches with a global row offset.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from molten_b200 import graphs, workloads
from molten_b200.codegen import compile_graph
from molten_b200.fusion import FusionEngine
from molten_b200.runtime import MoltenRuntime
from oracle import graph_oracle as orc
from tests._golden import CASES, assert_close, graph_for, load, rounded_operand_bound

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TORCH_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


@pytest.fixture(scope="module")
def rt():
    return MoltenRuntime()


def to_torch(arr, dev=DEV):
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    return torch.from_numpy(arr.copy()).to(dev)


def to_numpy(t):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f32(t):
    return t.detach().float().cpu().numpy()


def run_graph(rt, g, tensors, dtype, **kw):
    ks = compile_graph(g, dtype=dtype)
    assert len(ks) == 1
    ck = rt.compile(ks[0])
    return ck(*tensors, **kw), ck


@pytest.mark.parametrize("case", CASES)
def test_golden_case(rt, case):
    meta, inputs, ref_f32, ref_out = load(case)
    g = graph_for(meta, inputs)
    tensors = [to_torch(inputs[k]) for k in meta["inputs"]]
    dt = meta["out_dtype"]
    out, _ = run_graph(rt, g, tensors, tensors[0].dtype.__str__().replace("torch.", ""))
    torch.cuda.synchronize()
    assert_close(as_f32(out), ref_f32, dt, case)
    # and against the oracle's once-rounded output
    res = orc.evaluate(g, inputs)
    oid = g.ops[g._outputs[0]].inputs[0]
    assert_close(as_f32(out), res[("f32", oid)], dt, case + " vs oracle")


def _sample_rows(rows, n, seed=0):
    rng = np.random.default_rng(seed)
    pick = set(rng.choice(rows, size=min(n, rows), replace=False).tolist())
    pick |= {0, rows - 1}
    return np.array(sorted(pick))


def _rows_2d(t):
    return t.reshape(-1, t.shape[-1])


FULL = [
    "rmsnorm_f32_2048x5120",
    "rmsnorm_silu_bf16_1x3584",
    "rmsnorm_silu_bf16_2048x3584",
    "rmsnorm_silu_bf16_8192x3584",
    "softmax_f32_65536x2048",
    "softmax_f32_65536x2048_causal",
    "softmax_bf16_65536x2048",
    "softmax_bf16_65536x2048_causal",
    "softmax_f32_4096x32768",
    "softmax_f32_4096x32768_causal",
    "softmax_bf16_4096x32768",
    "softmax_bf16_4096x32768_causal",
    "chain_bf16_16384x8192",
    "rope_bf16_4x4096x32x128",
    "attention_score_bf16_32x2048x2048x128",
]


@pytest.mark.parametrize("name", FULL)
def test_full_size_row_workloads(rt, name):
    w = workloads.WORKLOADS[name]
    g = w.graph()
    xs = workloads.make_inputs(w, seed=0, device=DEV)
    out, ck = run_graph(rt, g, xs, w.dtype)
    out2 = ck(*xs)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16) if out.dtype != torch.float32 else out.view(torch.int32),
                       out2.view(torch.int16) if out2.dtype != torch.float32 else out2.view(torch.int32)), \
        "repeated runs differ"
    rows = _rows_2d(xs[0]).shape[0]
    pick = _sample_rows(rows, 48)
    # evaluate the oracle on the sampled rows only (rows are independent)
    sub_inputs = {}
    names = [g.ops[i].name for i in sorted(i for i, o in g.ops.items() if o.op_type.name == "INPUT")]
    for nm, t in zip(names, xs):
        if t.dim() >= 2 and _rows_2d(t).shape[0] == rows:
            sub_inputs[nm] = to_numpy(_rows_2d(t)[torch.as_tensor(pick, device=t.device)])
        else:
            sub_inputs[nm] = to_numpy(t)
    got = as_f32(_rows_2d(out)[torch.as_tensor(pick, device=out.device)])
    if w.kind == "softmax":
        # the mask depends on the global row: evaluate row by row
        g1 = graphs.softmax((1, got.shape[1]), causal=w.params["causal"])
        oid = g1.ops[g1._outputs[0]].inputs[0]
        ref = np.concatenate([
            orc.evaluate(g1, {"logits": sub_inputs["logits"][i:i + 1]},
                         row_offset=int(r))[("f32", oid)]
            for i, r in enumerate(pick)])
        full = as_f32(_rows_2d(out))
        sums = full.astype(np.float64).sum(axis=1)
        tol = 1e-5 if w.dtype == "float32" else 2e-2
        assert np.all(np.abs(sums - 1.0) < tol * max(1, np.sqrt(full.shape[1]) / 8)), "row sums"
        assert np.all(full >= 0)
        if w.params["causal"]:
            cols = full.shape[1]
            r = np.arange(full.shape[0]) % cols
            masked = np.arange(cols)[None, :] > r[:, None]
            assert np.all(full[masked] == 0.0), "masked entries must be exactly 0"
    elif w.kind == "attention_score":
        # row r of the stacked scores: head r // m, query r % m
        p = w.params
        q, k = to_numpy(xs[0]), to_numpy(xs[1])
        g1 = graphs.attention_score(1, p["n"], p["d"])
        oid = g1.ops[g1._outputs[0]].inputs[0]
        ref = np.concatenate([
            orc.evaluate(g1, {"q": q[r // p["m"], r % p["m"]][None, :], "k": k[r // p["m"]]})[("f32", oid)]
            for r in pick])
    elif w.kind == "rope":
        # each sampled row at its own position ((row // heads) % seq)
        p = w.params
        xr = orc.to_f32(sub_inputs["x"], w.dtype)
        cos, sin = sub_inputs["cos"], sub_inputs["sin"]
        pos = (pick // p["heads"]) % p["seq"]
        ref = np.concatenate([
            orc.rope(xr[i].reshape(1, 1, 1, -1), [cos[q:q + 1], sin[q:q + 1]]).reshape(1, -1)
            for i, q in enumerate(pos)])
    else:
        sg = w.graph(rows=len(pick))
        res = orc.evaluate(sg, sub_inputs)
        ref = res[("f32", sg.ops[sg._outputs[0]].inputs[0])]
    assert_close(got, ref, w.dtype, name)


def test_full_size_gemm(rt):
    w = workloads.WORKLOADS["gemm_bias_gelu_bf16_8192x4096x14336"]
    A, B, bias = workloads.make_inputs(w, seed=0, device=DEV)
    out, ck = run_graph(rt, w.graph(), [A, B, bias], "bfloat16")
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0, "a bounded wait timed out"
    pick = _sample_rows(A.shape[0], 6)
    Ar = to_numpy(A[torch.as_tensor(pick, device=DEV)])
    cols = _sample_rows(B.shape[1], 512, seed=1)
    Bc = to_numpy(B[:, torch.as_tensor(cols, device=DEV)].contiguous())
    bc = to_numpy(bias[torch.as_tensor(cols, device=DEV)])
    sg = graphs.gemm_bias_gelu(len(pick), A.shape[1], len(cols))
    res = orc.evaluate(sg, {"A": Ar, "B": Bc, "bias": bc})
    ref = res[("f32", sg.ops[sg._outputs[0]].inputs[0])]
    got = as_f32(out[torch.as_tensor(pick, device=DEV)][:, torch.as_tensor(cols, device=DEV)])
    assert_close(got, ref, "bfloat16", "gemm full size")
    out2 = ck(A, B, bias)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16)), "repeated runs differ"


@pytest.mark.parametrize("m,k,n", [(128, 64, 64), (200, 72, 136), (1, 4096, 256), (257, 512, 320),
                                   (1024, 1024, 1024)])
def test_gemm_shapes(rt, m, k, n):
    g = graphs.gemm_bias_gelu(m, k, n)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m * 7 + n)
    A = torch.randn(m, k, generator=gen, device=DEV).to(torch.bfloat16)
    B = (torch.randn(k, n, generator=gen, device=DEV) / k ** 0.5).to(torch.bfloat16)
    bias = (torch.randn(n, generator=gen, device=DEV) * 0.02).to(torch.bfloat16)
    out, _ = run_graph(rt, g, [A, B, bias], "bfloat16")
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"A": to_numpy(A), "B": to_numpy(B), "bias": to_numpy(bias)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16",
                 f"gemm {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n,kmajor,batch,bdt,epi", [
    (64, 128, 64, False, 1, "float32", False),      # the reference's test_matmul_kernel
    (256, 512, 384, False, 1, "float32", True),
    (300, 200, 504, False, 1, "float32", True),
    (1024, 256, 512, False, 1, "float32", True),
    (513, 1024, 768, False, 1, "float32", True),
    (300, 512, 384, True, 1, "float32", True),      # B given as transpose(Bt)
    (200, 128, 300, True, 3, "float32", True),      # 3 stacked problems, K-major B
    (256, 136, 520, False, 2, "float32", True),
    (256, 512, 384, False, 1, "bfloat16", True),    # fp32 A x bf16 B
    (512, 4096, 1024, False, 1, "float32", True),   # long K
    (128, 16384, 256, False, 1, "float32", True),   # longer K
])
def test_gemm_float32(rt, m, k, n, kmajor, batch, bdt, epi):
    """fp32 MATMUL (+ bias + GELU): each fp32 operand is split into three
    bf16 planes, the tensor cores sum the six plane products in chunks of
    four k-blocks and the epilogue adds the chunks in fp32 registers; held
    to the fp32 bar against the oracle (fp64 accumulation, one rounding)."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    lead = [batch] if batch > 1 else []
    g = DataflowGraph("gemm_f32")
    a = g.add_input("A", TS(lead + [m, k]), dtype="float32")
    if kmajor:
        bmat = g.transpose(g.add_input("Bt", TS(lead + [n, k]), dtype=bdt))
    else:
        bmat = g.add_input("B", TS(lead + [k, n]), dtype=bdt)
    mm = g.matmul(a, bmat)
    if epi:
        bias = g.add_input("bias", TS([n]), dtype="float32")
        mm = g.gelu(g.add(mm, bias))
    g.add_output(mm)
    kern = CodeGenerator(dtype="float32").generate(g, FusionEngine().fuse(g)[0])
    fams = [sk.family for sk in kern.plan.kernels]
    assert fams == ["split3", "split3", "gemm"] and kern.plan.kernels[-1].config["split3"]
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m + 5 * n + 3 * k)
    A = torch.randn(*lead, m, k, generator=gen, device=DEV)
    bshape = (*lead, n, k) if kmajor else (*lead, k, n)
    B = (torch.randn(*bshape, generator=gen, device=DEV) / k ** 0.5).to(TORCH_DT[bdt])
    ins = [A, B]
    names = ["A", "Bt" if kmajor else "B"]
    if epi:
        ins.append(0.02 * torch.randn(n, generator=gen, device=DEV))
        names.append("bias")
    ck = rt.compile(kern)
    out = ck(*ins)
    out2 = ck(*ins)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    assert out.dtype == torch.float32
    assert torch.equal(out.view(torch.int32), out2.view(torch.int32)), "repeated runs differ"
    res = orc.evaluate(g, dict(zip(names, [to_numpy(t) for t in ins])))
    ref = res[("f32", g.ops[g._outputs[0]].inputs[0])]
    got = as_f32(out)
    rel = np.abs(got - ref).max() / np.abs(ref).max()
    print(f"fp32 gemm {batch}x{m}x{k}x{n}: max |err| / max |ref| = {rel:.2e}")
    assert_close(got, ref, "float32", f"fp32 gemm {batch}x{m}x{k}x{n} kmajor {kmajor}")


@pytest.mark.parametrize("m,k,n,bn,kmajor,batch", [
    (256, 64, 256, 256, False, 1), (300, 200, 504, 256, False, 1), (1000, 72, 136, 128, False, 1),
    (513, 1024, 768, 256, False, 1), (2048, 512, 1024, None, False, 1),
    (300, 512, 384, 256, True, 1), (200, 128, 300, 128, True, 3), (256, 136, 520, 256, False, 2)])
def test_gemm_sm_pair(rt, m, k, n, bn, kmajor, batch):
    """The SM-pair engine (cluster of 2 CTAs, tcgen05.mma.cta_group::2, a
    256-row tile per pair, each CTA staging half of A's rows and half of B's
    columns): ragged m, n, k, both B majors, stacked problems."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    lead = [batch] if batch > 1 else []
    g = DataflowGraph("gemm_pair")
    a = g.add_input("A", TS(lead + [m, k]), dtype="bfloat16")
    if kmajor:
        bt = g.add_input("Bt", TS(lead + [n, k]), dtype="bfloat16")
        bmat = g.transpose(bt)
    else:
        bmat = g.add_input("B", TS(lead + [k, n]), dtype="bfloat16")
    bias = g.add_input("bias", TS([n]), dtype="bfloat16")
    g.add_output(g.gelu(g.add(g.matmul(a, bmat), bias)))
    tune = {"gemm": {"pair": True, **({"bn": bn} if bn else {})}}
    kern = CodeGenerator(dtype="bfloat16", tune=tune).generate(g, FusionEngine().fuse(g)[0])
    (sk,) = kern.plan.kernels
    assert sk.family == "gemm" and sk.config["pair"] and sk.config["b_kmajor"] == kmajor
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m + 3 * n + k)
    A = torch.randn(*lead, m, k, generator=gen, device=DEV).to(torch.bfloat16)
    bshape = (*lead, n, k) if kmajor else (*lead, k, n)
    B = (torch.randn(*bshape, generator=gen, device=DEV) / k ** 0.5).to(torch.bfloat16)
    bb = (0.02 * torch.randn(n, generator=gen, device=DEV)).to(torch.bfloat16)
    ck = rt.compile(kern)
    out = ck(A, B, bb)
    out2 = ck(A, B, bb)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16)), "repeated runs differ"
    names = ["A", "Bt" if kmajor else "B", "bias"]
    res = orc.evaluate(g, dict(zip(names, [to_numpy(A), to_numpy(B), to_numpy(bb)])))
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16",
                 f"pair gemm {batch}x{m}x{k}x{n} bn {bn} kmajor {kmajor}")


@pytest.mark.parametrize("m,k,n,batch,dtype,kmajor", [
    (64, 4096, 2048, 1, "bfloat16", False), (1, 4096, 256, 1, "bfloat16", False),
    (37, 4000, 384, 1, "bfloat16", False), (50, 1024, 320, 3, "bfloat16", False),
    (64, 2048, 1024, 1, "float16", False), (64, 4096, 1024, 1, "bfloat16", True)])
def test_gemm_stream_k(rt, m, k, n, batch, dtype, kmajor):
    """Fewer tiles than SMs: the tiles x k-blocks iteration space is spread
    over every SM; CTAs sharing a tile write fp32 partials and the last to
    arrive sums them in slot order -- deterministic, and the per-tile
    counters are back at 0 after every call (the repeat must match bit for
    bit)."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    lead = [batch] if batch > 1 else []
    g = DataflowGraph("gemm_sk")
    a = g.add_input("A", TS(lead + [m, k]), dtype=dtype)
    if kmajor:
        bmat = g.transpose(g.add_input("Bt", TS(lead + [n, k]), dtype=dtype))
    else:
        bmat = g.add_input("B", TS(lead + [k, n]), dtype=dtype)
    bias = g.add_input("bias", TS([n]), dtype=dtype)
    g.add_output(g.gelu(g.add(g.matmul(a, bmat), bias)))
    kern = CodeGenerator(dtype=dtype, tune={"gemm": {"streamk": True}}).generate(g, FusionEngine().fuse(g)[0])
    (sk,) = kern.plan.kernels
    assert sk.config["streamk"] and sk.config["sk_maxseg"] >= 2
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m * 17 + n + k)
    T = TORCH_DT[dtype]
    A = torch.randn(*lead, m, k, generator=gen, device=DEV).to(T)
    bshape = (*lead, n, k) if kmajor else (*lead, k, n)
    B = (torch.randn(*bshape, generator=gen, device=DEV) / k ** 0.5).to(T)
    bb = (0.02 * torch.randn(n, generator=gen, device=DEV)).to(T)
    ck = rt.compile(kern)
    out = ck(A, B, bb)
    out2 = ck(A, B, bb)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16)), "repeated runs differ"
    names = ["A", "Bt" if kmajor else "B", "bias"]
    res = orc.evaluate(g, dict(zip(names, [to_numpy(A), to_numpy(B), to_numpy(bb)])))
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dtype,
                 f"stream-K gemm {batch}x{m}x{k}x{n}")


def test_gemm_plain_matmul_fp16(rt):
    g = graphs.gemm_bias_gelu(256, 256, 256, dtype="float16")
    gen = torch.Generator(device=DEV)
    gen.manual_seed(5)
    A = torch.randn(256, 256, generator=gen, device=DEV).half()
    B = (torch.randn(256, 256, generator=gen, device=DEV) / 16).half()
    bias = (torch.randn(256, generator=gen, device=DEV) * 0.02).half()
    out, _ = run_graph(rt, g, [A, B, bias], "float16")
    torch.cuda.synchronize()
    res = orc.evaluate(g, {"A": to_numpy(A), "B": to_numpy(B), "bias": to_numpy(bias)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "float16", "fp16 gemm")


@pytest.mark.parametrize("rows,cols,dtype", [(1, 5120, "float32"), (5, 1000, "float32"),
                                             (3, 3583, "bfloat16"), (7, 24, "bfloat16"),
                                             (33, 128, "float16"), (2, 32768, "bfloat16")])
def test_rmsnorm_edge_shapes(rt, rows, cols, dtype):
    g = graphs.rmsnorm_silu_gate(rows, cols, dtype=dtype)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows * 131 + cols)
    x = torch.randn(rows, cols, generator=gen, device=DEV).to(TORCH_DT[dtype])
    wt = (1 + 0.1 * torch.randn(cols, generator=gen, device=DEV)).to(TORCH_DT[dtype])
    gt = torch.randn(rows, cols, generator=gen, device=DEV).to(TORCH_DT[dtype])
    out, _ = run_graph(rt, g, [x, wt, gt], dtype)
    torch.cuda.synchronize()
    res = orc.evaluate(g, {"x": to_numpy(x), "w": to_numpy(wt), "gate": to_numpy(gt)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dtype,
                 f"rmsnorm_silu {rows}x{cols} {dtype}")


@pytest.mark.parametrize("rows,cols,dtype", [(1, 3584, "bfloat16"), (37, 3584, "bfloat16"),
                                             (300, 1024, "bfloat16"), (150, 5120, "float32")])
def test_tma_ring_engine(rows, cols, dtype):
    """The TMA-staged ring engine, forced on at sizes where the automatic
    choice would not pick it (fewer rows than CTAs, ragged last wave)."""
    rt = MoltenRuntime(tune={"row": {"engine": "tma"}})
    g = graphs.rmsnorm_silu_gate(rows, cols, dtype=dtype)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=gen, device=DEV).to(TORCH_DT[dtype])
    wt = (1 + 0.1 * torch.randn(cols, generator=gen, device=DEV)).to(TORCH_DT[dtype])
    gt = torch.randn(rows, cols, generator=gen, device=DEV).to(TORCH_DT[dtype])
    from molten_b200.codegen import CodeGenerator
    from molten_b200.fusion import FusionEngine
    gk = CodeGenerator(tune=rt.tune).generate(g, FusionEngine().fuse(g)[0],
                                              {0: (rows, cols), 1: (cols,), 2: (rows, cols)},
                                              {0: dtype, 1: dtype, 2: dtype})
    assert gk.plan.kernels[0].config["engine"] == "tma"
    out = rt.compile(gk)(x, wt, gt)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"x": to_numpy(x), "w": to_numpy(wt), "gate": to_numpy(gt)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dtype,
                 f"tma ring {rows}x{cols} {dtype}")


TEAM_CASES = [
    # (graph, rows, cols, dtype, tune): teams of TW warps per row in the ring
    ("rmsnorm_silu_gate", 300, 1000, "bfloat16", {"row": {"engine": "tma", "tw": 3, "nc": 7}}),
    ("rmsnorm_silu_gate", 2048, 3584, "bfloat16", {"row": {"engine": "tma", "tw": 1}}),
    ("rmsnorm_silu_gate", 4099, 3584, "float16", {"row": {"engine": "tma", "tw": 2, "nc": 14}}),
    ("rmsnorm", 150, 5120, "float32", {"row": {"engine": "tma", "tw": 5, "nc": 2}}),
    ("rmsnorm", 5000, 64, "float32", {"row": {"engine": "tma", "tw": 2, "nc": 7}}),
    ("chain", 300, 1024, "bfloat16", {"ew": {"engine": "tma", "tw": 4}}),
    ("rmsnorm_silu_gate", 2048, 8192, "bfloat16", None),
    ("chain", 4096, 4096, "bfloat16", None),
    ("chain", 4096, 2048, "bfloat16", {"ew": {"engine": "tma"}}),
]


@pytest.mark.parametrize("kind,rows,cols,dtype,tune", TEAM_CASES)
def test_tma_ring_teams(kind, rows, cols, dtype, tune):
    """The TMA ring with a team of warps per row (reductions combined across
    the team's warps in shared memory): ragged slot counts, one-warp teams,
    rows shorter than a team, elementwise groups; checked against the oracle,
    and two runs are bit-identical."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.fusion import FusionEngine
    rt = MoltenRuntime(tune=tune)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows * 7 + cols)
    T = TORCH_DT[dtype]
    if kind == "chain":
        g = graphs.chain(rows, cols, dtype=dtype)
        names = ["x", "r", "a", "b", "s"]
        tensors = [torch.randn(rows, cols, generator=gen, device=DEV).to(T) for _ in range(2)]
        tensors += [(2 * torch.rand(cols, generator=gen, device=DEV) - 1).to(T) for _ in range(3)]
    else:
        g = graphs.BUILDERS[kind](rows, cols, dtype=dtype)
        names = ["x", "w", "gate"][:3 if kind == "rmsnorm_silu_gate" else 2]
        tensors = [torch.randn(rows, cols, generator=gen, device=DEV).to(T),
                   (1 + 0.1 * torch.randn(cols, generator=gen, device=DEV)).to(T)]
        if kind == "rmsnorm_silu_gate":
            tensors.append(torch.randn(rows, cols, generator=gen, device=DEV).to(T))
    grp = FusionEngine().fuse(g)[0]
    ins = sorted(i for i, o in g.ops.items() if o.op_type.name == "INPUT")
    gk = CodeGenerator(tune=tune).generate(g, grp, {i: tuple(t.shape) for i, t in zip(ins, tensors)},
                                           {i: dtype for i in ins})
    c = gk.plan.kernels[0].config
    assert c["engine"] == "tma"
    if tune:
        want = (tune.get("row") or tune.get("ew"))
        assert c["tw"] == want.get("tw", c["tw"])
    ck = rt.compile(gk)
    out = ck(*tensors)
    again = ck(*tensors)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    assert torch.equal(out, again)
    res = orc.evaluate(g, {n: to_numpy(t) for n, t in zip(names, tensors)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dtype,
                 f"tma teams {kind} {rows}x{cols} {dtype} {tune}")


STREAM_CASES = [
    # (graph, rows, cols, dtype, row tune) -- persistent stream form forced on
    ("softmax", 300, 32768, "bfloat16", {"stream": 3}),
    ("softmax", 300, 32768, "bfloat16", {"stream": 3, "tpc": 1024, "cl": 1}),
    ("softmax_causal", 777, 4096, "float32", {"stream": 3}),
    ("softmax_causal", 2000, 8192, "bfloat16", {"stream": 3, "tpc": 256, "cl": 4}),
    ("softmax", 3001, 2048, "bfloat16", {"stream": 4}),
    ("rmsnorm", 5000, 5120, "float32", {"stream": 3, "engine": "regs"}),
    ("rmsnorm", 999, 8192, "float32", {"stream": 3, "engine": "regs", "tpc": 128, "cl": 4}),
    ("softmax", 1000, 32768, "float32", {"stream": 3, "tpc": 1024, "cl": 2, "min_blocks": 1}),
    ("rmsnorm_silu", 1000, 3584, "bfloat16", {"stream": 4, "engine": "regs"}),
    # bulk staging: one bulk copy per row and staged operand, mbarrier per stage
    ("softmax", 300, 32768, "bfloat16", {"stream": 3, "tpc": 1024, "cl": 1, "bulk": True}),
    ("softmax_causal", 700, 8192, "bfloat16", {"stream": 3, "tpc": 1024, "cl": 1, "bulk": True}),
    # masked row tails written by bulk zero stores from shared memory
    ("softmax_causal", 700, 8192, "bfloat16", {"stream": 3, "tpc": 1024, "cl": 1, "bulk": True,
                                               "zero_tail": True}),
    ("rmsnorm_silu", 1000, 3584, "bfloat16", {"stream": 4, "engine": "regs", "bulk": True}),
]


def _stream_graph(kind, rows, cols, dtype):
    if kind == "rmsnorm":
        return graphs.rmsnorm(rows, cols, dtype=dtype), ["x", "w"]
    if kind == "rmsnorm_silu":
        return graphs.rmsnorm_silu_gate(rows, cols, dtype=dtype), ["x", "w", "gate"]
    return graphs.softmax((rows, cols), dtype=dtype, causal=kind.endswith("causal")), ["logits"]


@pytest.mark.parametrize("kind,rows,cols,dtype,tune", STREAM_CASES)
def test_stream_row_engine(kind, rows, cols, dtype, tune):
    """The persistent stream form of the register engine (rows staged per
    thread with cp.async, several rows per team, cluster partials pushed into
    exchange areas that alternate by row parity), forced on; also launched
    as two row-offset halves, which must give the same bits."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.fusion import FusionEngine
    rt = MoltenRuntime(tune={"row": dict(tune)})
    g, names = _stream_graph(kind, rows, cols, dtype)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows * 7 + cols)
    xs = []
    for nm in names:
        if nm == "w":
            xs.append((1 + 0.1 * torch.randn(cols, generator=gen, device=DEV)).to(TORCH_DT[dtype]))
        else:
            scale = 3.0 if kind.startswith("softmax") else 1.0
            xs.append((scale * torch.randn(rows, cols, generator=gen, device=DEV)).to(TORCH_DT[dtype]))
    shapes = {i: tuple(t.shape) for i, t in enumerate(xs)}
    gk = CodeGenerator(tune=rt.tune).generate(g, FusionEngine().fuse(g)[0], shapes,
                                              {i: dtype for i in shapes})
    assert gk.plan.kernels[0].config.get("stream", 0) >= 2, gk.plan.kernels[0].config
    assert bool(gk.plan.kernels[0].config.get("bulk")) == bool(tune.get("bulk"))
    ck = rt.compile(gk)
    out = ck(*xs)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0, "a bounded wait gave up"
    res = orc.evaluate(g, {nm: to_numpy(t) for nm, t in zip(names, xs)})
    ref = res[("f32", g.ops[g._outputs[0]].inputs[0])]
    assert_close(as_f32(out), ref, dtype, f"stream {kind} {rows}x{cols} {dtype} {tune}")
    # two launches over row halves, each told its first global row
    half = rows // 2 + 1
    outs = []
    for a, b in ((0, half), (half, rows)):
        part = [t if t.dim() == 1 else t[a:b] for t in xs]
        outs.append(ck(*part, row_offset=a))
    torch.cuda.synchronize()
    bits = (lambda t: t.view(torch.int16)) if out.dtype != torch.float32 else \
        (lambda t: t.view(torch.int32))
    assert torch.equal(bits(torch.cat(outs)), bits(out))


@pytest.mark.parametrize("rows,cols,dtype,tune", [
    (333, 8192, "float32", {"zero_tail": True}),
    (4100, 32768, "float32", {"zero_tail": True}),
    (300, 32768, "bfloat16", {"tpc": 1024, "cl": 1, "zero_tail": True}),
])
def test_causal_zero_tail(rows, cols, dtype, tune):
    """Causal softmax in the register form with the masked tail of each row
    written by bulk zero stores (TMA engine, shared zero buffer) instead of
    the threads: matches the oracle, every fully masked column is exactly
    0, and two row-offset halves give the same bits (the tail starts where
    each row's global limit puts it)."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.fusion import FusionEngine
    rt = MoltenRuntime(tune={"row": dict(tune)})
    g = graphs.softmax((rows, cols), dtype=dtype, causal=True)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows + cols)
    x = (3.0 * torch.randn(rows, cols, generator=gen, device=DEV)).to(TORCH_DT[dtype])
    gk = CodeGenerator(tune=rt.tune).generate(g, FusionEngine().fuse(g)[0], {0: (rows, cols)},
                                              {0: dtype})
    assert "bulk_zero_tail" in gk.source and not gk.plan.kernels[0].config.get("stream")
    ck = rt.compile(gk)
    out = ck(x)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    # the mask: column c of row r is visible iff c <= r mod cols
    cidx = torch.arange(cols, device=DEV)[None, :]
    ridx = (torch.arange(rows, device=DEV) % cols)[:, None]
    assert torch.all(out.float()[cidx > ridx] == 0)
    # the oracle on sampled rows, each at its global row (the mask follows it)
    pick = _sample_rows(rows, 24)
    g1 = graphs.softmax((1, cols), dtype=dtype, causal=True)
    oid = g1.ops[g1._outputs[0]].inputs[0]
    xn = to_numpy(x)
    ref = np.concatenate([orc.evaluate(g1, {"logits": xn[r:r + 1]}, row_offset=int(r))[("f32", oid)]
                          for r in pick])
    got = as_f32(out[torch.as_tensor(pick, device=DEV)])
    assert_close(got, ref, dtype, f"zero tail {rows}x{cols} {dtype}")
    half = rows // 2 + 1
    outs = [ck(x[a:b], row_offset=a) for a, b in ((0, half), (half, rows))]
    torch.cuda.synchronize()
    bits = (lambda t: t.view(torch.int16)) if out.dtype != torch.float32 else \
        (lambda t: t.view(torch.int32))
    assert torch.equal(bits(torch.cat(outs)), bits(out))


@pytest.mark.parametrize("rows,cols,dtype,period,offset,tune", [
    (4100, 32768, "float32", None, 0, {}),
    (333, 8192, "bfloat16", None, 0, {}),
    (700, 8192, "float16", None, 0, {}),
    (1000, 16384, "bfloat16", 5000, 3, {}),
    (160, 8200, "bfloat16", None, 0, {"causal_split": True}),          # a ragged last zero tile
    (300, 2048, "bfloat16", None, 0, {"causal_split": True}),          # row CTAs store the zeros
    (257, 4096, "float32", 1000, 0, {"causal_split": True, "causal_zero_tiles": 3}),
    (229, 8196, "float32", None, 0, {"causal_split": True, "causal_zero_tiles": 2}),   # 16-byte rows
    (333, 8200, "bfloat16", None, 0, {"causal_split": True, "causal_interleave": False}),
    (333, 8192, "bfloat16", None, 0, {"causal_split": True, "causal_zero_ctas": 37}),   # persistent
    (1000, 16384, "float32", 5000, 3, {"causal_split": True, "causal_zero_ctas": 296}),
])
def test_causal_split(rows, cols, dtype, period, offset, tune):
    """The split causal softmax (row CTAs for the visible logits, zero-tile
    CTAs for the masked rest): matches the oracle on sampled rows at their
    global rows, every masked element is exactly 0, and two row-offset
    halves give the same bits."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    rt = MoltenRuntime(tune={"row": dict(tune)})

    def graph(r):
        g = DataflowGraph("causal")
        x = g.add_input("logits", TS([r, cols]), dtype=dtype)
        g.add_output(g.softmax(g.add(x, g.causal_mask(period=period, offset=offset)), -1))
        return g
    g = graph(rows)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows + 3 * cols)
    x = (3.0 * torch.randn(rows, cols, generator=gen, device=DEV)).to(TORCH_DT[dtype])
    gk = CodeGenerator(tune=rt.tune).generate(g, FusionEngine().fuse(g)[0], {0: (rows, cols)},
                                              {0: dtype})
    (sk,) = gk.plan.kernels
    assert sk.family == "causal", sk.family
    ck = rt.compile(gk)
    out = ck(x)
    torch.cuda.synchronize()
    P = period or cols
    cidx = torch.arange(cols, device=DEV)[None, :]
    ridx = (torch.arange(rows, device=DEV) % P + offset)[:, None]
    assert torch.all(out.float()[cidx > ridx] == 0), "masked entries must be exactly 0"
    pick = _sample_rows(rows, 24)
    g1 = graph(1)
    oid = g1.ops[g1._outputs[0]].inputs[0]
    xn = to_numpy(x)
    ref = np.concatenate([orc.evaluate(g1, {"logits": xn[r:r + 1]}, row_offset=int(r))[("f32", oid)]
                          for r in pick])
    assert_close(as_f32(out[torch.as_tensor(pick, device=DEV)]), ref, dtype,
                 f"causal split {rows}x{cols} {dtype} P {period} off {offset} {tune}")
    sums = out.double().sum(dim=1)
    assert torch.all((sums - 1).abs() < (1e-5 if dtype == "float32" else 2e-2) * max(1, cols ** 0.5 / 8))
    half = rows // 2 + 1
    outs = [ck(x[a:b], row_offset=a) for a, b in ((0, half), (half, rows))]
    torch.cuda.synchronize()
    bits = (lambda t: t.view(torch.int16)) if out.dtype != torch.float32 else \
        (lambda t: t.view(torch.int32))
    assert torch.equal(bits(torch.cat(outs)), bits(out))


FP16_CASES = [
    ("rmsnorm", {"rows": 300, "cols": 5120}),
    ("rmsnorm_silu_gate", {"rows": 257, "cols": 3584}),
    ("softmax", {"shape": (600, 2048), "causal": True}),
    ("softmax", {"shape": (64, 32768), "causal": False}),      # stream form (16-bit long rows)
    ("chain", {"rows": 512, "cols": 8192}),
]


@pytest.mark.parametrize("kind,params", FP16_CASES)
def test_fp16_row_patterns(rt, kind, params):
    """fp16 I/O through the reference's own switch, ZeroCompiler(fp16=True)
    (compiler.py / cli.py --fp16), for every row pattern."""
    from molten_b200.compiler import ZeroCompiler
    w = workloads.Workload(f"{kind}_fp16", kind, params, "float16")
    g = w.graph()
    xs = workloads.make_inputs(w, seed=3, device=DEV)
    ks = ZeroCompiler(fp16=True).compile(g)
    assert len(ks) == 1 and ks[0].plan.input_dtypes == ["float16"] * len(xs)
    out = rt.compile(ks[0])(*xs)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    names = [g.ops[i].name for i in sorted(i for i, o in g.ops.items() if o.op_type.name == "INPUT")]
    res = orc.evaluate(g, {nm: to_numpy(t) for nm, t in zip(names, xs)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "float16",
                 f"fp16 {kind} {params}")


def test_cli_benchmark_runs_on_the_gpu(capsys):
    from molten_b200 import cli
    assert cli.main(["benchmark", "--dim", "3584", "--seq", "256", "--dtype", "float16", "--run"]) == 0
    assert "us/call" in capsys.readouterr().out


ROPE_CASES = [
    # batch, seq, heads, head_dim, x dtype, table dtype, style, packed table
    (2, 64, 8, 128, "bfloat16", "float32", None, False),
    (1, 33, 5, 64, "float32", "float32", None, False),
    (2, 64, 8, 128, "bfloat16", "float32", "half", False),
    (2, 24, 4, 128, "float16", "float16", None, True),
    (1, 40, 4, 80, "bfloat16", "bfloat16", "half", True),
]


def _rope_inputs(b, sq, h, d, xdt, tdt, packed, seed):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    x = torch.randn(b, sq, h, d, generator=gen, device=DEV).to(TORCH_DT[xdt])
    ang = torch.rand(sq, d // 2, generator=gen, device=DEV) * 6.283185307179586
    c, s = torch.cos(ang).to(TORCH_DT[tdt]), torch.sin(ang).to(TORCH_DT[tdt])
    if packed:
        return [x, torch.stack([c, s], -1).reshape(sq, d)], ["x", "freqs"]
    return [x, c, s], ["x", "cos", "sin"]


@pytest.mark.parametrize("b,sq,h,d,xdt,tdt,style,packed", ROPE_CASES)
def test_rope(rt, b, sq, h, d, xdt, tdt, style, packed):
    """RoPE (ops.py:24-35) against the oracle: both pairings, separate or
    packed tables, fp32 / bf16 / fp16; batch halves launched with their
    global row offset give the same bits; a misaligned x runs the scalar
    kernel."""
    g = graphs.rope(b, sq, h, d, xdt, tdt, style=style, packed=packed)
    xs, names = _rope_inputs(b, sq, h, d, xdt, tdt, packed, seed=b * 1000 + sq + d)
    ck = rt.compile(compile_graph(g, dtype=xdt)[0])
    out = ck(*xs)
    torch.cuda.synchronize()
    assert out.dtype == TORCH_DT[xdt] and ck.specialization(*xs).plan.kernels[0].family == "rope"
    res = orc.evaluate(g, {nm: to_numpy(t) for nm, t in zip(names, xs)})
    ref = res[("f32", g.ops[g._outputs[0]].inputs[0])]
    assert_close(as_f32(out), ref, xdt, f"rope {b}x{sq}x{h}x{d} {xdt}/{tdt} {style} {packed}")
    bits = (lambda t: t.view(torch.int32)) if xdt == "float32" else (lambda t: t.view(torch.int16))
    if b >= 2:
        parts = [ck(xs[0][i:i + 1], *xs[1:], row_offset=i * sq * h) for i in range(b)]
        torch.cuda.synchronize()
        assert torch.equal(bits(torch.cat(parts)), bits(out))
    # x at an odd element offset: not 16-byte aligned -> the scalar form
    base = torch.empty(xs[0].numel() + 1, dtype=xs[0].dtype, device=DEV)
    xm = base[1:].view(xs[0].shape)
    xm.copy_(xs[0])
    out_m = ck(xm, *xs[1:])
    torch.cuda.synchronize()
    assert ck.specialization(xm, *xs[1:]).plan.kernels[0].config["scalar"]
    assert_close(as_f32(out_m), ref, xdt, "rope misaligned")


def test_rmsnorm_then_rope_group(rt):
    """One fusion group (as the reference groups it): row kernel, fp32
    intermediate, RoPE kernel."""
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    g = DataflowGraph("norm_rope")
    x = g.add_input("x", TS([2, 16, 4, 64]), dtype="bfloat16")
    w = g.add_input("w", TS([64]), dtype="bfloat16")
    f = g.add_input("freqs", TS([16, 64]), dtype="bfloat16")
    g.add_output(g.rope(g.rms_norm(x, w, "norm"), f))
    gen = torch.Generator(device=DEV)
    gen.manual_seed(11)
    xt = torch.randn(2, 16, 4, 64, generator=gen, device=DEV).to(torch.bfloat16)
    wt = (1 + 0.1 * torch.randn(64, generator=gen, device=DEV)).to(torch.bfloat16)
    ang = torch.rand(16, 32, generator=gen, device=DEV) * 6.283185307179586
    ft = torch.stack([torch.cos(ang), torch.sin(ang)], -1).reshape(16, 64).to(torch.bfloat16)
    (k,) = compile_graph(g, dtype="bfloat16")
    assert [sk.family for sk in k.plan.kernels] == ["row", "rope"]
    out = rt.compile(k)(xt, wt, ft)
    torch.cuda.synchronize()
    res = orc.evaluate(g, {"x": to_numpy(xt), "w": to_numpy(wt), "freqs": to_numpy(ft)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16", "norm+rope")


def _attention_kernel(g, dtype, fused):
    from molten_b200.codegen import CodeGenerator
    gen = CodeGenerator(dtype=dtype, tune=None if fused else {"attn": {"fused": False}})
    (grp,) = FusionEngine().fuse(g)
    kern = gen.generate(g, grp)
    fams = [sk.family for sk in kern.plan.kernels]
    if fused:
        assert fams == ["attn"]
    else:
        assert fams == ["gemm", "row"] and kern.plan.kernels[0].config["b_kmajor"]
    return kern


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "gemm+softmax"])
@pytest.mark.parametrize("m,n,d,dtype", [(256, 512, 128, "bfloat16"), (200, 300, 64, "bfloat16"),
                                         (130, 1000, 256, "float16"), (64, 4096, 128, "bfloat16"),
                                         (100, 77, 72, "bfloat16"), (33, 40, 16, "float16"),
                                         (512, 2048, 128, "bfloat16")])
def test_attention_score(rt, m, n, d, dtype, fused):
    """softmax(Q @ K^T * scale) (ops.py:55-59).  Fused: one kernel, two
    tensor-core passes over K (row statistics, then probabilities), no score
    matrix in HBM.  Unfused: the GEMM reads K's rows K-major (the TRANSPOSE
    costs nothing), scale in its epilogue, fp32 scores, row softmax.  Ragged
    m, n and d: rows past m and columns past n are computed from zero-filled
    or neighbouring data and never stored."""
    g = graphs.attention_score(m, n, d, dtype=dtype)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m + n + d)
    q = torch.randn(m, d, generator=gen, device=DEV).to(TORCH_DT[dtype])
    k = torch.randn(n, d, generator=gen, device=DEV).to(TORCH_DT[dtype])
    kern = _attention_kernel(g, dtype, fused)
    out = rt.compile(kern)(q, k)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"q": to_numpy(q), "k": to_numpy(k)})
    ref = res[("f32", g.ops[g._outputs[0]].inputs[0])]
    assert_close(as_f32(out), ref, dtype, f"attention {m}x{n}x{d} {dtype}")
    sums = as_f32(out).astype(np.float64).sum(axis=1)
    assert np.all(np.abs(sums - 1.0) < 2e-2)


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "gemm+softmax"])
@pytest.mark.parametrize("h,m,n,d", [(3, 200, 300, 64), (4, 256, 512, 128), (5, 96, 136, 128),
                                     (2, 129, 64, 128), (6, 64, 1000, 32)])
def test_multihead_attention_score(rt, h, m, n, d, fused):
    """One problem per head, heads stacked along the rows: a row block past
    m reads the next head's rows, which are never stored (TMA stores only
    when m is a multiple of 32, so that no 32-row store box crosses a head)."""
    g = graphs.attention_score(m, n, d, heads=h)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(h * 100 + m)
    q = torch.randn(h, m, d, generator=gen, device=DEV).to(torch.bfloat16)
    k = torch.randn(h, n, d, generator=gen, device=DEV).to(torch.bfloat16)
    kern = _attention_kernel(g, "bfloat16", fused)
    assert kern.plan.kernels[0].config["batch"] == h
    out = rt.compile(kern)(q, k)
    torch.cuda.synchronize()
    assert out.shape == (h, m, n) and MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"q": to_numpy(q), "k": to_numpy(k)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16",
                 f"attention {h}x{m}x{n}x{d}")


@pytest.mark.parametrize("tune", [{"poly": [12, 12]}, {"poly": [32, 32]}, {"poly": [0, 16]},
                                  {"sum16": True}, {"sum16": True, "poly": [0, 8]},
                                  {"sum16": False}, {"x2": True}, {"x2": True, "poly": [4, 8]},
                                  {"bn": 128}, {"bn": 128, "groups": 2}, {"bn": 64}],
                         ids=["poly12", "poly32", "poly0-16", "sum16", "sum16-poly8", "sum32",
                              "x2", "x2-poly", "bn128-4buf", "bn128-groups", "bn64-4buf"])
@pytest.mark.parametrize("h,m,n,d,dtype", [(2, 256, 512, 128, "bfloat16"), (1, 100, 77, 72, "float16"),
                                           (1, 64, 2000, 64, "float16")])
def test_fused_attention_exp2_variants(rt, tune, h, m, n, d, dtype):
    """Exponentials on the FMA pipe (Cody-Waite + a minimax cubic, relative
    error < 1e-4) and pass-0 row sums from f16 exponential pairs: the same
    parity bar as the fp32 EX2 path."""
    from molten_b200.codegen import CodeGenerator
    g = graphs.attention_score(m, n, d, dtype=dtype, heads=h if h > 1 else None)
    kern = CodeGenerator(dtype=dtype, tune={"attn": dict(tune)}).generate(
        g, FusionEngine().fuse(g)[0])
    c = kern.plan.kernels[0].config
    assert all(c[k] == v for k, v in tune.items())
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m * 7 + n)
    lead = (h,) if h > 1 else ()
    q = torch.randn(*lead, m, d, generator=gen, device=DEV).to(TORCH_DT[dtype])
    k = torch.randn(*lead, n, d, generator=gen, device=DEV).to(TORCH_DT[dtype])
    out = rt.compile(kern)(q, k)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"q": to_numpy(q), "k": to_numpy(k)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dtype,
                 f"attention {tune}")


def test_fused_attention_large_logits(rt):
    """Scores far from zero (scale 1, |s| up to ~100): the row maximum is
    subtracted before exponentiation, so nothing overflows and each row's
    largest entry is the one the oracle picks."""
    m, n, d = 128, 384, 64
    g = graphs.attention_score(m, n, d, scale=1.0)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(7)
    q = (torch.randn(m, d, generator=gen, device=DEV) * 1.5).to(torch.bfloat16)
    k = (torch.randn(n, d, generator=gen, device=DEV) * 1.5).to(torch.bfloat16)
    kern = _attention_kernel(g, "bfloat16", True)
    out = rt.compile(kern)(q, k)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    got = as_f32(out)
    assert np.all(np.isfinite(got))
    res = orc.evaluate(g, {"q": to_numpy(q), "k": to_numpy(k)})
    ref = res[("f32", g.ops[g._outputs[0]].inputs[0])]
    assert_close(got, ref, "bfloat16", "attention large logits")


def test_batched_gemm_k_tail(rt):
    """Batched MN-major B with k = 72: the last k block of a problem reaches
    into the next problem's B rows, which meet A's zero-filled columns."""
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    h, m, k, n = 2, 130, 72, 192
    g = DataflowGraph("bmm")
    a = g.add_input("A", TS([h, m, k]), dtype="bfloat16")
    b = g.add_input("B", TS([h, k, n]), dtype="bfloat16")
    bias = g.add_input("bias", TS([n]), dtype="bfloat16")
    g.add_output(g.gelu(g.add(g.matmul(a, b), bias)))
    gen = torch.Generator(device=DEV)
    gen.manual_seed(9)
    A = torch.randn(h, m, k, generator=gen, device=DEV).to(torch.bfloat16)
    B = (torch.randn(h, k, n, generator=gen, device=DEV) / k ** 0.5).to(torch.bfloat16)
    bb = (0.02 * torch.randn(n, generator=gen, device=DEV)).to(torch.bfloat16)
    (kern,) = compile_graph(g, dtype="bfloat16")
    assert kern.plan.kernels[0].config["batch"] == h
    out = rt.compile(kern)(A, B, bb)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"A": to_numpy(A), "B": to_numpy(B), "bias": to_numpy(bb)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16", "bmm")


def test_gemm_with_transposed_b(rt):
    """GELU(A @ Bt^T + bias) with Bt [N, K]: the K-major B path on its own."""
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    m, k, n = 300, 512, 384
    g = DataflowGraph("gemm_bt")
    a = g.add_input("A", TS([m, k]), dtype="bfloat16")
    bt = g.add_input("Bt", TS([n, k]), dtype="bfloat16")
    bias = g.add_input("bias", TS([n]), dtype="bfloat16")
    g.add_output(g.gelu(g.add(g.matmul(a, g.transpose(bt)), bias)))
    gen = torch.Generator(device=DEV)
    gen.manual_seed(77)
    A = torch.randn(m, k, generator=gen, device=DEV).to(torch.bfloat16)
    Bt = (torch.randn(n, k, generator=gen, device=DEV) / k ** 0.5).to(torch.bfloat16)
    bb = (0.02 * torch.randn(n, generator=gen, device=DEV)).to(torch.bfloat16)
    (kern,) = compile_graph(g, dtype="bfloat16")
    assert [sk.family for sk in kern.plan.kernels] == ["gemm"] and kern.plan.kernels[0].config["b_kmajor"]
    out = rt.compile(kern)(A, Bt, bb)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"A": to_numpy(A), "Bt": to_numpy(Bt), "bias": to_numpy(bb)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16", "gemm Bt")


def _norm_gemm_graph(m, k, n, dt, wdt, norm_out=False):
    from molten_b200.ir import DataflowGraph, TensorShape as TS
    g = DataflowGraph("norm_gemm")
    x = g.add_input("x", TS([m, k]), dtype=dt)
    w = g.add_input("w", TS([k]), dtype=wdt)
    B = g.add_input("B", TS([k, n]), dtype=dt)
    bias = g.add_input("bias", TS([n]), dtype=dt)
    normed = g.rms_norm(x, w, "norm")
    g.add_output(g.gelu(g.add(g.matmul(normed, B), bias)))
    if norm_out:
        g.add_output(normed)
    return g


def _normed(xs):
    """fp32 x / sqrt(mean(x^2) + 1e-6) * w, the GEMM's computed A operand
    (1.13 bounds |GELU'| for the bias + GELU epilogue)."""
    x, w = as_f32(xs[0]).astype(np.float64), as_f32(xs[1]).astype(np.float64)
    return (x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-6) * w).astype(np.float32)


def _norm_gemm_inputs(m, k, n, dt, wdt, seed):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    x = torch.randn(m, k, generator=gen, device=DEV).to(TORCH_DT[dt])
    w = (1 + 0.1 * torch.randn(k, generator=gen, device=DEV)).to(TORCH_DT[wdt])
    B = (torch.randn(k, n, generator=gen, device=DEV) / k ** 0.5).to(TORCH_DT[dt])
    bias = (0.02 * torch.randn(n, generator=gen, device=DEV)).to(TORCH_DT[dt])
    return [x, w, B, bias]


@pytest.mark.parametrize("m,k,n,dt,wdt", [(256, 512, 384, "bfloat16", "bfloat16"),
                                          (300, 520, 136, "bfloat16", "float32"),
                                          (64, 4096, 1024, "float16", "float16"),
                                          (1, 3584, 512, "bfloat16", "bfloat16")])
def test_rmsnorm_gemm_prologue(rt, m, k, n, dt, wdt):
    """RMSNorm -> GEMM (+ bias + GELU), one fusion group as the reference
    groups it, run (opt-in) as ONE tcgen05 GEMM that normalises A as it is
    staged (x * w in shared memory, 1/rms on the accumulator rows)."""
    g = _norm_gemm_graph(m, k, n, dt, wdt)
    xs = _norm_gemm_inputs(m, k, n, dt, wdt, seed=m + k + n)
    rt = MoltenRuntime(tune={"gemm": {"prologue": True}})
    from molten_b200.codegen import CodeGenerator
    ck = rt.compile(CodeGenerator(dtype=dt, tune=rt.tune).generate(g, FusionEngine().fuse(g)[0]))
    out = ck(*xs)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    (sk,) = ck.specialization(*xs).plan.kernels
    assert sk.family == "gemm" and sk.config["prologue"]["kind"] == "rmsnorm"
    res = orc.evaluate(g, {"x": to_numpy(xs[0]), "w": to_numpy(xs[1]), "B": to_numpy(xs[2]),
                           "bias": to_numpy(xs[3])})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dt,
                 f"rmsnorm->gemm {m}x{k}x{n} {dt}/{wdt}",
                 extra_abs=rounded_operand_bound(_normed(xs), as_f32(xs[2]), dt, slope=1.13))


def test_rmsnorm_gemm_unfused_when_the_norm_is_an_output(rt):
    g = _norm_gemm_graph(128, 512, 256, "bfloat16", "bfloat16", norm_out=True)
    xs = _norm_gemm_inputs(128, 512, 256, "bfloat16", "bfloat16", seed=5)
    # the normalised x is also an output: two kernels even with the prologue on
    from molten_b200.codegen import CodeGenerator
    kern = CodeGenerator(dtype="bfloat16", tune={"gemm": {"prologue": True}}).generate(
        g, FusionEngine().fuse(g)[0])
    assert [sk.family for sk in kern.plan.kernels] == ["row", "gemm"]
    assert "prologue" not in kern.plan.kernels[1].config
    outs = dict(zip(kern.plan.outputs, rt.compile(kern)(*xs)))   # by producing op id
    y, normed = (outs[g.ops[o].inputs[0]] for o in g._outputs)
    torch.cuda.synchronize()
    res = orc.evaluate(g, {"x": to_numpy(xs[0]), "w": to_numpy(xs[1]), "B": to_numpy(xs[2]),
                           "bias": to_numpy(xs[3])})
    assert_close(as_f32(y), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16", "gemm",
                 extra_abs=rounded_operand_bound(_normed(xs), as_f32(xs[2]), "bfloat16", slope=1.13))
    assert_close(as_f32(normed), res[("f32", g.ops[g._outputs[1]].inputs[0])], "bfloat16", "norm")


def test_misaligned_pointers_take_the_scalar_path(rt):
    g = graphs.rmsnorm(4, 512)
    base = torch.randn(4 * 512 + 1, device=DEV)
    x = base[1:].view(4, 512)                         # 4-byte offset: not 16-byte aligned
    wt = torch.randn(512, device=DEV)
    ck = rt.compile(compile_graph(g)[0])
    out = ck(x, wt)
    torch.cuda.synchronize()
    sk = ck.specialization(x, wt).plan.kernels[0]
    assert sk.config["vec"] == 1 and sk.config.get("engine") != "tma"
    res = orc.evaluate(g, {"x": to_numpy(x), "w": to_numpy(wt)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "float32", "misaligned")


def test_misaligned_output_is_refused_before_launch(rt):
    g = graphs.rmsnorm(4, 512)
    ck = rt.compile(compile_graph(g)[0])
    x = torch.randn(4, 512, device=DEV)
    wt = torch.randn(512, device=DEV)
    base = torch.empty(4 * 512 + 1, device=DEV)
    with pytest.raises(RuntimeError):          # shape/contiguity check or alignment guard
        ck(x, wt, out=base[1:].view(4, 512))
    torch.cuda.synchronize()                   # the context is still healthy
    assert torch.isfinite(ck(x, wt)).all()


def test_row_sharded_launches_match_whole(rt):
    """Rank-style row blocks with their global row offset reproduce the
    single launch bit for bit (causal mask included)."""
    from molten_b200.shard import row_shards
    g = graphs.softmax((96, 256), causal=True)
    x = 3 * torch.randn(96, 256, device=DEV)
    ck = rt.compile(compile_graph(g)[0])
    whole = ck(x)
    parts = []
    for start, stop in row_shards(96, 3):
        gs = graphs.softmax((stop - start, 256), causal=True)
        cks = rt.compile(compile_graph(gs)[0])
        parts.append(cks(x[start:stop], row_offset=start))
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts), whole)


def test_out_argument_and_stream(rt):
    g = graphs.chain(64, 1024)
    w = workloads.scaled(workloads.WORKLOADS["chain_bf16_16384x8192"], rows=64, cols=1024)
    xs = workloads.make_inputs(w, seed=3, device=DEV)
    ck = rt.compile(compile_graph(g, dtype="bfloat16")[0])
    out = torch.empty(64, 1024, dtype=torch.bfloat16, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        r = ck(*xs, out=out)
    s.synchronize()
    assert r is out
    res = orc.evaluate(g, {n: to_numpy(t) for n, t in zip(["x", "r", "a", "b", "s"], xs)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16", "out=")


def test_multi_kernel_group_gemm_then_softmax(rt):
    """MATMUL -> SOFTMAX (one fusion group) runs as GEMM + row kernel."""
    from molten_b200.ir import DataflowGraph, TensorShape
    g = DataflowGraph("scores")
    q = g.add_input("q", TensorShape([128, 64]), dtype="bfloat16")
    k = g.add_input("k", TensorShape([64, 256]), dtype="bfloat16")
    g.add_output(g.softmax(g.matmul(q, k)))
    Q = torch.randn(128, 64, device=DEV).to(torch.bfloat16)
    K = (torch.randn(64, 256, device=DEV) / 8).to(torch.bfloat16)
    ks = compile_graph(g, dtype="bfloat16")
    ck = rt.compile(ks[0])
    out = ck(Q, K)
    torch.cuda.synchronize()
    res = orc.evaluate(g, {"q": to_numpy(Q), "k": to_numpy(K)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16", "scores")


@pytest.mark.parametrize("case", ["rms_silu", "softmax_causal", "gemm", "attention"])
def test_run_host_matches_one_device_call(rt, case):
    """Host buffers in and out, rows split into chunks whose uploads,
    kernels and downloads overlap on three streams (each chunk launched with
    its global row offset): bit-identical to one call on device tensors."""
    gen = torch.Generator().manual_seed(21)
    bf = torch.bfloat16
    if case == "rms_silu":
        g = graphs.rmsnorm_silu_gate(1000, 3584)
        xs = [torch.randn(1000, 3584, generator=gen).to(bf), (1 + 0.1 * torch.randn(3584, generator=gen)).to(bf),
              torch.randn(1000, 3584, generator=gen).to(bf)]
        dt = "bfloat16"
    elif case == "softmax_causal":
        g = graphs.softmax((999, 2048), causal=True)
        xs = [3 * torch.randn(999, 2048, generator=gen)]
        dt = "float32"
    elif case == "gemm":
        g = graphs.gemm_bias_gelu(1100, 256, 512)
        xs = [torch.randn(1100, 256, generator=gen).to(bf), (torch.randn(256, 512, generator=gen) / 16).to(bf),
              (0.02 * torch.randn(512, generator=gen)).to(bf)]
        dt = "bfloat16"
    else:
        g = graphs.attention_score(256, 512, 128, heads=2)
        xs = [torch.randn(2, 256, 128, generator=gen).to(bf), torch.randn(2, 512, 128, generator=gen).to(bf)]
        dt = "bfloat16"
    ck = rt.compile(compile_graph(g, dtype=dt)[0])
    whole = ck(*[t.to(DEV) for t in xs])
    host = [t.pin_memory() for t in xs]
    got = ck.run_host(*host, chunks=4, device=0)
    torch.cuda.synchronize()
    assert not got.is_cuda and got.shape == whole.shape
    w = whole.cpu()
    assert torch.equal(got.view(torch.int16) if got.dtype == bf else got, w.view(torch.int16) if w.dtype == bf else w)
    assert MoltenRuntime.read_status(0) == 0


def test_wrong_inputs_raise(rt):
    g = graphs.rmsnorm(4, 64)
    ck = rt.compile(compile_graph(g)[0])
    x = torch.randn(4, 64, device=DEV)
    with pytest.raises(RuntimeError, match="takes 2 tensors"):
        ck(x)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        ck(x.cpu(), torch.randn(64))


GUARD_CASES = [
    # (label, graph builder, inputs builder, dtype); shapes with ragged tails
    ("row regs ragged", lambda: graphs.rmsnorm_silu_gate(37, 1004, dtype="bfloat16"), "rms3", "bfloat16"),
    ("row tma teams", lambda: graphs.rmsnorm_silu_gate(2100, 3584, dtype="bfloat16"), "rms3", "bfloat16"),
    ("row tma fp32", lambda: graphs.rmsnorm(2051, 5120), "rms2", "float32"),
    ("softmax causal small CTAs", lambda: graphs.softmax((129, 2048), causal=True), "logits", "float32"),
    ("softmax causal split", lambda: graphs.softmax((150, 8192), dtype="bfloat16", causal=True),
     "logits", "bfloat16"),
    ("softmax stream bulk", lambda: graphs.softmax((151, 32768), dtype="bfloat16"), "logits", "bfloat16"),
    ("chain ew", lambda: graphs.chain(300, 1000), "chain", "bfloat16"),
    ("chain tma teams", lambda: graphs.chain(4096, 2048), "chain", "bfloat16"),
    ("gemm one SM", lambda: graphs.gemm_bias_gelu(300, 256, 520), "gemm", "bfloat16"),
    ("gemm SM pair", lambda: graphs.gemm_bias_gelu(1100, 256, 1024), "gemm", "bfloat16"),
    ("gemm stream-K", lambda: graphs.gemm_bias_gelu(64, 2048, 512), "gemm", "bfloat16"),
    ("gemm fp32 bf16x3", lambda: graphs.gemm_bias_gelu(130, 256, 384, dtype="float32"), "gemm", "float32"),
    ("attention fused", lambda: graphs.attention_score(200, 300, 64, heads=2), "attn", "bfloat16"),
    ("rope", lambda: graphs.rope(1, 16, 4, 128), "rope", "bfloat16"),
]


def _guard_inputs(kind, g, dtype, gen):
    T = TORCH_DT[dtype]
    shapes = {o.name: tuple(int(d) for d in o.shape.dims) for o in g.ops.values() if o.op_type.name == "INPUT"}
    names = [g.ops[i].name for i in sorted(i for i, o in g.ops.items() if o.op_type.name == "INPUT")]
    out = []
    for nm in names:
        shp = shapes[nm]
        if kind == "rope" and nm in ("cos", "sin"):
            ang = torch.rand(*shp, generator=gen, device=DEV) * 6.283185307179586
            out.append(torch.cos(ang) if nm == "cos" else torch.sin(ang))
        elif nm in ("w",):
            out.append((1 + 0.1 * torch.randn(*shp, generator=gen, device=DEV)).to(T))
        elif nm == "B":
            out.append((torch.randn(*shp, generator=gen, device=DEV) / shp[0] ** 0.5).to(T))
        elif nm in ("a", "b", "s"):
            out.append((2 * torch.rand(*shp, generator=gen, device=DEV) - 1).to(T))
        else:
            scale = 3.0 if kind == "logits" else 1.0
            out.append((scale * torch.randn(*shp, generator=gen, device=DEV)).to(T))
    return out


@pytest.mark.parametrize("label,build,kind,dtype", GUARD_CASES, ids=[c[0] for c in GUARD_CASES])
def test_outputs_stay_inside_their_buffers(rt, label, build, kind, dtype):
    """Guard bands: every kernel family writes its output through a view into
    a larger buffer whose 4 KB before and after hold random bytes; the bytes
    must be untouched, the inputs unchanged, and the output equal to a call
    that allocates its own (ragged tails, split/stream/ring/team forms)."""
    g = build()
    gen = torch.Generator(device=DEV)
    gen.manual_seed(len(label) * 97 + 5)
    tensors = _guard_inputs(kind, g, dtype, gen)
    before = [t.clone() for t in tensors]
    (kern,) = compile_graph(g, dtype=dtype)
    ck = rt.compile(kern)
    ref = ck(*tensors)
    torch.cuda.synchronize()
    nbytes = ref.numel() * ref.element_size()
    guard = 4096
    big = torch.randint(0, 256, (guard + nbytes + guard,), dtype=torch.uint8, device=DEV, generator=gen)
    pattern = big.clone()
    view = big[guard:guard + nbytes].view(ref.dtype).view(ref.shape)
    ck(*tensors, out=view)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    assert torch.equal(big[:guard], pattern[:guard]), f"{label}: wrote before its output"
    assert torch.equal(big[guard + nbytes:], pattern[guard + nbytes:]), f"{label}: wrote past its output"
    assert torch.equal(view, ref), f"{label}: output through a view differs"
    for t, b in zip(tensors, before):
        assert torch.equal(t, b), f"{label}: an input was modified"


def test_bad_modules_and_launches_are_refused():
    """Host-side failure detection with a GPU present: an image that is not
    a cubin and an unknown kernel name come back as status codes with a
    message; nothing is launched."""
    import ctypes
    from molten_b200 import _capi
    lib = _capi.load_library()
    junk = b"this is not an sm_100a cubin " * 64
    h = ctypes.c_void_p()
    rc = lib.molten_module_load_data(junk, len(junk), 0, ctypes.byref(h))
    assert rc != 0 and lib.molten_last_error()
    rt = MoltenRuntime()
    ck = rt.compile(compile_graph(graphs.rmsnorm(4, 64))[0])
    ck(torch.randn(4, 64, device=DEV), torch.ones(64, device=DEV))    # loads the module
    spec = next(iter(ck._specs.values()))
    mod = spec.module(0).handle
    cfg = _capi.LaunchCfg()
    cfg.grid[:] = [1, 1, 1]
    cfg.block[:] = [32, 1, 1]
    cfg.cluster[:] = [1, 1, 1]
    params = ctypes.create_string_buffer(8)
    rc = lib.molten_launch(mod, b"no_such_kernel", ctypes.byref(cfg), params, 8, None)
    assert rc != 0 and b"no_such_kernel" in lib.molten_last_error()
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0


@pytest.mark.parametrize("rows,cols,causal,shift,spread", [
    (300, 2048, False, 1000.0, 20.0),
    (151, 32768, False, -500.0, 50.0),
    (160, 8192, True, 250.0, 30.0),
    (129, 2048, True, 0.0, 40.0),
])
def test_fp32_softmax_large_logits(rt, rows, cols, causal, shift, spread):
    """fp32 softmax takes its exponentials on the EX2 unit as 2^((x - m)
    log2e): with logits far from zero and widely spread, the result must
    still meet the fp32 bar against the oracle (subtracting the max first
    keeps the argument's error proportional to x - m, not to x)."""
    g = graphs.softmax((rows, cols), causal=causal)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows + cols)
    x = shift + spread * torch.randn(rows, cols, generator=gen, device=DEV)
    out, _ = run_graph(rt, g, [x], "float32")
    torch.cuda.synchronize()
    res = orc.evaluate(g, {"logits": to_numpy(x)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], "float32",
                 f"softmax fp32 {rows}x{cols} causal={causal} logits {shift}+{spread}N")


def _two_pass_graph(rows, cols, dtype):
    """LayerNorm without affine terms, then shifted by the row max:
    y = (x - mean(x)) * rsqrt(mean((x - mean(x))^2) + eps); out = y - max(y)
    -- reductions in three passes (mean; the centred second moment; a max)."""
    from molten_b200.ir import DataflowGraph, OpType, TensorShape
    g = DataflowGraph("two_pass")
    x = g.add_input("x", TensorShape([rows, cols]), dtype=dtype)
    mu = g.add_op(OpType.MEAN, [x])
    g.ops[mu].reduction_dim = -1
    d = g.sub(x, mu)
    var = g.add_op(OpType.MEAN, [g.mul(d, d)])
    g.ops[var].reduction_dim = -1
    y = g.mul(d, g.add_op(OpType.RSQRT, [g.add(var, g.add_constant("eps", 1e-5))]))
    mx = g.add_op(OpType.MAX, [y])
    g.ops[mx].reduction_dim = -1
    g.add_output(g.sub(y, mx))
    return g


@pytest.mark.parametrize("rows,cols,dtype,tune", [
    (2048, 4096, "float32", None),
    (2050, 3584, "bfloat16", None),
    (2048, 4096, "bfloat16", {"row": {"engine": "tma", "tw": 1}}),
    (300, 2048, "float32", {"row": {"engine": "tma", "tw": 5, "nc": 2}}),
])
def test_tma_ring_teams_multi_pass(rows, cols, dtype, tune):
    """Reductions in several passes (sum, sum, max) on the TMA ring with
    teams of warps per row: each pass's team reduction alternates between
    the team's two shared-memory buffers; checked against the oracle."""
    from molten_b200.codegen import CodeGenerator
    from molten_b200.fusion import FusionEngine
    g = _two_pass_graph(rows, cols, dtype)
    groups = FusionEngine().fuse(g)
    assert len(groups) == 1
    gk = CodeGenerator(dtype=dtype, tune=tune).generate(g, groups[0])
    (sk,) = gk.plan.kernels
    assert sk.family == "row" and sk.config["engine"] == "tma" and sk.passes == 3
    gen = torch.Generator(device=DEV)
    gen.manual_seed(rows + cols)
    x = (0.5 + 2 * torch.randn(rows, cols, generator=gen, device=DEV)).to(TORCH_DT[dtype])
    ck = MoltenRuntime(tune=tune).compile(gk)
    out = ck(x)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"x": to_numpy(x)})
    assert_close(as_f32(out), res[("f32", g.ops[g._outputs[0]].inputs[0])], dtype,
                 f"two-pass ring {rows}x{cols} {dtype} {tune}")


@pytest.mark.parametrize("kind,shape,dtype", [
    ("rmsnorm_silu_gate", (0, 3584), "bfloat16"),
    ("rmsnorm", (4, 0), "float32"),
    ("softmax", (0, 2048), "float32"),
    ("chain", (0, 1024), "bfloat16"),
])
def test_empty_inputs_give_empty_outputs(rt, kind, shape, dtype):
    """No rows (or no columns): the call returns an empty output of the
    right shape and dtype and launches nothing; so does the host-buffer
    call."""
    rows, cols = shape
    T = TORCH_DT[dtype]
    if kind == "softmax":
        g, tensors = graphs.softmax((rows, cols), dtype=dtype), [torch.empty(rows, cols, dtype=T, device=DEV)]
    elif kind == "chain":
        g = graphs.chain(rows, cols, dtype=dtype)
        tensors = [torch.empty(rows, cols, dtype=T, device=DEV) for _ in range(2)]
        tensors += [torch.zeros(cols, dtype=T, device=DEV) for _ in range(3)]
    else:
        g = graphs.BUILDERS[kind](rows, cols, dtype=dtype)
        tensors = [torch.empty(rows, cols, dtype=T, device=DEV), torch.ones(cols, dtype=T, device=DEV)]
        if kind == "rmsnorm_silu_gate":
            tensors.append(torch.empty(rows, cols, dtype=T, device=DEV))
    ck = rt.compile(compile_graph(g, dtype=dtype)[0])
    out = ck(*tensors)
    host = ck.run_host(*[t.cpu() for t in tensors], device=0)
    torch.cuda.synchronize()
    assert out.shape == (rows, cols) and out.dtype == T and out.device.type == "cuda"
    assert tuple(host.shape) == (rows, cols) and host.dtype == T
    assert MoltenRuntime.read_status(0) == 0
