"""Lowering of one fusion group to kernel plans.

A fusion group (``fusion.py``) is lowered for one concrete specialisation
(shapes and dtypes of its external inputs) into one or more *sub-kernels*:

* ``row``  -- row patterns with last-dim reductions (RMSNorm, RMSNorm*SiLU,
  softmax, any reduction + elementwise DAG).  A row is register-resident.
* ``ew``   -- pure elementwise DAGs with numpy broadcasting of per-column,
  per-row and scalar operands (the N-op chains).
* ``gemm`` -- MATMUL followed by an elementwise epilogue (bias, GELU ...).

A group that cannot run as one kernel (a MATMUL whose result feeds a row
reduction, or elementwise ops feeding a MATMUL) is split into consecutive
sub-kernels whose intermediates the runtime allocates.

Semantics follow the reference's CPU definitions (``benchmarks/ops.py``):
RMS(x) = sqrt(mean(x^2, -1) + eps) (``ops.py:15``), softmax over the last
dim (``ops.py:45-47``), tanh-form GELU (``ops.py:52``, ``codegen.py:63``),
SiLU(g) = g * sigmoid(g) (``ops.py:19-21``).  All arithmetic is fp32; inputs
are widened exactly and outputs are rounded once (round to nearest even).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from .ir import DataflowGraph, OpType, ELEMENTWISE_OPS, REDUCTION_OPS


class LoweringError(NotImplementedError):
    """The group (or this specialisation of it) has no sm_100a lowering."""


# ------------------------------------------------------------------- dtypes
_DTYPE_ALIASES = {
    "float32": "float32", "float": "float32", "fp32": "float32", "f32": "float32",
    "bfloat16": "bfloat16", "bf16": "bfloat16",
    "float16": "float16", "half": "float16", "fp16": "float16", "f16": "float16",
}
DTYPE_SIZE = {"float32": 4, "bfloat16": 2, "float16": 2}
DTYPE_CTYPE = {"float32": "float", "bfloat16": "bf16", "float16": "f16"}


def canon_dtype(d) -> str:
    s = str(d).replace("torch.", "")
    if s not in _DTYPE_ALIASES:
        raise LoweringError(f"unsupported dtype {d!r} (float32, bfloat16, float16)")
    return _DTYPE_ALIASES[s]


def promote(dtypes) -> str:
    """torch-style promotion among the three float types."""
    ds = set(dtypes)
    if not ds:
        return "float32"
    if len(ds) == 1:
        return ds.pop()
    return "float32"


# ------------------------------------------------------------------- shapes
def broadcast_shapes(a: tuple, b: tuple) -> tuple:
    n = max(len(a), len(b))
    a = (1,) * (n - len(a)) + tuple(a)
    b = (1,) * (n - len(b)) + tuple(b)
    out = []
    for x, y in zip(a, b):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise LoweringError(f"shapes {a} and {b} do not broadcast")
    return tuple(out)


def prod(xs) -> int:
    p = 1
    for x in xs:
        p *= int(x)
    return p


def is_mask_const(op) -> bool:
    return op.op_type == OpType.CONSTANT and op.attrs.get("kind") == "causal_mask"


def _reduces_last_dim(op, ndim: int) -> bool:
    d = op.reduction_dim
    return d is None or d == -1 or (ndim > 0 and d == ndim - 1)


def infer_shapes(graph: DataflowGraph, op_ids, known: dict) -> dict:
    """Concrete shape of every op in ``op_ids`` (topological order) given
    the shapes in ``known`` (external inputs).  Reductions keep the reduced
    dim as size 1, like ``mean(-1, keepdim=True)`` in ``ops.py:15``."""
    shapes = dict(known)
    for oid in op_ids:
        op = graph.ops[oid]
        ins = [shapes[i] for i in op.inputs]
        t = op.op_type
        if t in ELEMENTWISE_OPS:
            s = ()
            for x in ins:
                s = broadcast_shapes(s, x)
        elif t == OpType.SOFTMAX:
            s = ins[0]
            if not _reduces_last_dim(op, len(s)):
                raise LoweringError("softmax only over the last dim")
        elif t in REDUCTION_OPS:
            s = ins[0]
            if not _reduces_last_dim(op, len(s)):
                raise LoweringError(f"{t.name} only over the last dim")
            s = tuple(s[:-1]) + (1,) if len(s) else (1,)
        elif t == OpType.ROTATE:
            s = ins[0]
            check_rope_shapes(op, ins)
        elif t == OpType.TRANSPOSE:
            if len(ins[0]) < 2:
                raise LoweringError("TRANSPOSE needs rank >= 2")
            s = tuple(ins[0][:-2]) + (ins[0][-1], ins[0][-2])
        elif t == OpType.MATMUL:
            a, b = ins
            if len(b) < 2 or len(a) < 2:
                raise LoweringError("MATMUL needs A [..., M, K] and B [K, N] or [..., K, N]")
            if len(b) > 2 and tuple(a[:-2]) != tuple(b[:-2]):
                raise LoweringError(f"batched MATMUL needs equal batch dims: {a} @ {b}")
            if a[-1] != b[-2]:
                raise LoweringError(f"MATMUL inner dims differ: {a} @ {b}")
            s = tuple(a[:-1]) + (b[-1],)
        else:
            raise LoweringError(f"{t.name} has no sm_100a lowering")
        shapes[oid] = tuple(int(d) for d in s)
    return shapes


ROPE_STYLES = ("interleaved", "half")


def check_rope_shapes(op, ins):
    """ROTATE(x, cos, sin) / ROTATE(x, freqs) shapes (``ops.py:24-35``): x is
    [..., seq, heads, head_dim] with an even head_dim; cos and sin are
    [seq, head_dim/2]; a packed freqs table is [seq, head_dim]."""
    x = tuple(ins[0])
    if len(x) < 3:
        raise LoweringError(f"ROTATE needs x of rank >= 3 ([..., seq, heads, head_dim]), got {x}")
    seq, d = int(x[-3]), int(x[-1])
    if d % 2:
        raise LoweringError(f"ROTATE needs an even head_dim, got {d}")
    style = op.attrs.get("style") or "interleaved"
    if style not in ROPE_STYLES:
        raise LoweringError(f"ROTATE style {style!r} (interleaved, half)")
    if len(ins) == 2:
        want = [(seq, d)]
    elif len(ins) == 3:
        want = [(seq, d // 2), (seq, d // 2)]
    else:
        raise LoweringError("ROTATE takes (x, freqs) or (x, cos, sin)")
    for t, w in zip(ins[1:], want):
        t = tuple(int(v) for v in t)
        while len(t) > 2 and t[0] == 1:
            t = t[1:]
        if t != w:
            raise LoweringError(f"ROTATE table of shape {tuple(t)}; expected {w}")


# ----------------------------------------------------------- plan objects
@dataclass
class Operand:
    """An external input of a sub-kernel."""
    index: int            # position in the kernel's input pointer array
    op_id: int            # graph op (or sub-kernel value) providing it
    name: str
    dtype: str
    shape: tuple
    last: str             # "vec": varies along columns; "bcast": size 1 there
    row_map: str          # "full", "zero" or "general"
    row_terms: tuple = () # general: ((div, mod, stride), ...) over global row


@dataclass
class OutputSpec:
    index: int
    op_id: int
    dtype: str
    shape: tuple
    kind: str             # "full" (rows x cols) or "row" (one value per row)


@dataclass
class Value:
    """Node of a per-row expression DAG."""
    id: int
    kind: str             # "const" | "row" | "elem"
    op: str
    args: tuple = ()
    attrs: dict = field(default_factory=dict)
    avail: int = 0        # first pass in which the value can be computed


@dataclass
class SubKernel:
    family: str           # "row" | "ew" | "gemm"
    op_ids: list          # graph ops computed here (topological order)
    operands: list        # [Operand]
    outputs: list         # [OutputSpec]
    rows: int = 1
    cols: int = 1
    values: list = field(default_factory=list)      # [Value] (topological)
    out_values: list = field(default_factory=list)  # value id per output
    passes: int = 0
    precise: bool = True
    config: dict = field(default_factory=dict)
    # gemm only
    m: int = 0
    n: int = 0
    k: int = 0
    a_operand: Optional[int] = None
    b_operand: Optional[int] = None


@dataclass
class GroupPlan:
    name: str
    inputs: list          # graph op ids the caller passes, in order
    input_dtypes: list
    input_shapes: list
    outputs: list         # graph op ids returned, in order
    output_dtypes: list
    output_shapes: list
    kernels: list         # [SubKernel]
    temps: dict           # op id -> (shape, dtype) of intermediates


# ------------------------------------------------------------ group split
def group_topo(graph: DataflowGraph, op_ids) -> list:
    members = set(op_ids)
    return [i for i in graph.topological_order() if i in members]


def _deps_within(graph, root, members) -> set:
    out, stack = set(), [root]
    while stack:
        cur = stack.pop()
        for i in graph.ops[cur].inputs:
            if i in members and i not in out:
                out.add(i)
                stack.append(i)
    return out


def group_boundary(graph: DataflowGraph, op_ids):
    """(external inputs, outputs, live ops) of a group.

    Outputs are members consumed by an OUTPUT op or by an op outside the
    group; with none of those, the group's sinks (ops nobody consumes) are the
    outputs, which matches the reference emitting the last op's value.  Ops no
    output depends on (e.g. left behind by identity elimination) are dropped.
    """
    members = set(op_ids)
    consumers = {i: [] for i in members}
    for oid, op in graph.ops.items():
        for i in op.inputs:
            if i in consumers:
                consumers[i].append(oid)
    outs = [i for i in group_topo(graph, op_ids)
            if any(c not in members or graph.ops[c].op_type == OpType.OUTPUT
                   for c in consumers[i])]
    if not outs:
        outs = [i for i in group_topo(graph, op_ids) if not consumers[i]]
    live = set(outs)
    for o in outs:
        live |= _deps_within(graph, o, members)
    ordered = [i for i in group_topo(graph, op_ids) if i in live]
    ext = []
    for i in ordered:
        for j in graph.ops[i].inputs:
            if j not in members and j not in ext:
                ext.append(j)
    ext.sort()
    return ext, outs, ordered


def rms_prologue(graph: DataflowGraph, m: int, members: set, outs=()):
    """(rms, div, mul) op ids when MATMUL ``m``'s A operand is
    ``x / RMS(x) * w`` (``DataflowGraph.rms_norm``, ``ir.py:169-173``) and each
    of those ops is used only along that chain and is not a group output;
    else None.  Such a group runs as one GEMM that normalises A as it is
    staged (the RMSNorm -> GEMM prologue)."""
    a = graph.ops[m].inputs[0]
    mul = graph.ops[a]
    if a not in members or mul.op_type != OpType.MUL or a in outs or a == graph.ops[m].inputs[1]:
        return None
    for d_id, w_id in ((mul.inputs[0], mul.inputs[1]), (mul.inputs[1], mul.inputs[0])):
        d = graph.ops[d_id]
        if d_id not in members or d.op_type != OpType.DIV or d_id in outs:
            continue
        x_id, r_id = d.inputs
        r = graph.ops[r_id]
        if r_id not in members or r.op_type != OpType.RMS or r.inputs != [x_id] or r_id in outs:
            continue
        chain = {r_id, d_id, a}
        if x_id in chain or w_id in chain:
            continue
        users = {o: [u for u in members if o in graph.ops[u].inputs] for o in chain}
        if users[r_id] == [d_id] and users[d_id] == [a] and users[a] == [m]:
            return [r_id, d_id, a]
    return None


def attention_pattern(graph: DataflowGraph, ordered: list, outs=()):
    """(transpose, matmul, mul or None, softmax) when the group is exactly
    softmax(matmul(q, transpose(k)) [* scalar constant]) over the last dim,
    with only the softmax leaving the group; else None."""
    if len(ordered) not in (3, 4):
        return None
    by = {graph.ops[i].op_type: i for i in ordered}
    if len(by) != len(ordered) or not {OpType.TRANSPOSE, OpType.MATMUL, OpType.SOFTMAX} <= set(by):
        return None
    t, m, sm = by[OpType.TRANSPOSE], by[OpType.MATMUL], by[OpType.SOFTMAX]
    mul = by.get(OpType.MUL)
    if len(ordered) == 4 and mul is None:
        return None
    if graph.ops[m].inputs[1] != t or graph.ops[m].inputs[0] == t:
        return None
    members = set(ordered)
    if any(o in outs for o in (t, m, mul) if o is not None) or sm not in outs and outs:
        return None
    users = lambda o: [u for u in members if o in graph.ops[u].inputs]
    if users(t) != [m]:
        return None
    if mul is not None:
        others = [i for i in graph.ops[mul].inputs if i != m]
        if len(others) != 1 or users(m) != [mul] or graph.ops[sm].inputs != [mul]:
            return None
        c = graph.ops[others[0]]
        if c.op_type != OpType.CONSTANT or c.attrs.get("kind") or c.attrs.get("value") is None:
            return None
        v = float(c.attrs["value"])
        if not (v > 0.0 and v < float("inf")):       # the row max is taken on raw scores
            return None
    elif graph.ops[sm].inputs != [m]:
        return None
    d = graph.ops[sm].reduction_dim
    if d not in (None, -1):
        return None
    return t, m, mul, sm


def split_group(graph: DataflowGraph, ordered: list, outs=(), fuse_prologue: bool = True,
                fuse_attention: bool = True) -> list:
    """Split a group's live ops into (family, ops) sub-kernels.

    ROTATE (RoPE) reads each element's pair partner, so it runs as a
    sub-kernel of its own between what it depends on and what follows (the
    fusion rules put it in any group: it is neither elementwise nor a
    reduction, ``fusion.py:65``)."""
    if fuse_attention and attention_pattern(graph, ordered, set(outs)):
        return [("attn", list(ordered))]
    rot = [i for i in ordered if graph.ops[i].op_type == OpType.ROTATE]
    if rot:
        r = rot[0]
        pre_set = _deps_within(graph, r, set(ordered))
        pre = [i for i in ordered if i in pre_set]
        rest = [i for i in ordered if i not in pre_set and i != r]
        return ((split_group(graph, pre, outs, fuse_prologue) if pre else []) + [("rope", [r])]
                + (split_group(graph, rest, outs, fuse_prologue) if rest else []))
    mm = [i for i in ordered if graph.ops[i].op_type == OpType.MATMUL]
    if not mm:
        fam = "row" if any(graph.is_reduction(i) for i in ordered) else "ew"
        return [(fam, list(ordered))]
    m = mm[0]
    members = set(ordered)
    pre_set = _deps_within(graph, m, members)
    # a TRANSPOSE that is only this MATMUL's B operand is no kernel: the GEMM
    # reads the untransposed matrix's rows K-major
    absorbed = []
    bt = graph.ops[m].inputs[1]
    if bt in pre_set and graph.ops[bt].op_type == OpType.TRANSPOSE:
        users = [o for o in members if bt in graph.ops[o].inputs]
        if users == [m] and graph.ops[m].inputs[0] != bt:
            absorbed = [bt]
            pre_set = pre_set - {bt}        # what bt reads is still computed first
    # RMSNorm feeding A only: normalised inside the GEMM as A is staged
    prologue = (rms_prologue(graph, m, members, set(outs)) or []) if fuse_prologue else []
    pre_set = pre_set - set(prologue)
    absorbed = absorbed + prologue
    pre = [i for i in ordered if i in pre_set]
    post = [i for i in ordered if i not in pre_set and i != m and i not in absorbed]
    post_set = set(post)
    epi, rest = [m], []
    epi_set = {m}
    for i in post:
        op = graph.ops[i]
        depends = any(j in epi_set for j in op.inputs)
        ok_inputs = all(j in epi_set or j not in post_set for j in op.inputs)
        if graph.is_elementwise(i) and depends and ok_inputs:
            epi.append(i)
            epi_set.add(i)
        else:
            rest.append(i)
    out = []
    if pre:
        out.append(("row" if any(graph.is_reduction(i) for i in pre) else "ew", pre))
    out.append(("gemm", epi + absorbed))
    if rest:
        out.append(("row" if any(graph.is_reduction(i) for i in rest) else "ew", rest))
    return out


# ------------------------------------------------------- operand analysis
def classify_operand(shape: tuple, it_shape: tuple):
    """(last, row_map, row_terms) of an operand broadcast to ``it_shape``."""
    n = len(it_shape)
    if len(shape) > n:
        raise LoweringError(f"operand {shape} has more dims than {it_shape}")
    s = (1,) * (n - len(shape)) + tuple(shape)
    cols = it_shape[-1] if n else 1
    last_dim = s[-1] if n else 1
    if last_dim == cols:
        last = "vec"
    elif last_dim == 1:
        last = "bcast"
    else:
        raise LoweringError(f"operand {shape} does not broadcast to {it_shape}")
    lead_it, lead_op = it_shape[:-1], s[:-1]
    if tuple(lead_op) == tuple(lead_it):
        return last, "full", ()
    if all(d == 1 for d in lead_op):
        return last, "zero", ()
    terms = []
    for d in range(len(lead_it)):
        if lead_op[d] == 1:
            continue
        if lead_op[d] != lead_it[d]:
            raise LoweringError(f"operand {shape} does not broadcast to {it_shape}")
        div = prod(lead_it[d + 1:])
        stride = prod(lead_op[d + 1:])
        terms.append((div, int(lead_it[d]), stride))
    return last, "general", tuple(terms)


_UNARY = {
    OpType.NEG: "neg", OpType.SQRT: "sqrt", OpType.RSQRT: "rsqrt",
    OpType.EXP: "exp", OpType.LOG: "log", OpType.TANH: "tanh",
    OpType.SIGMOID: "sigmoid", OpType.GELU: "gelu", OpType.SILU: "silu",
    OpType.RELU: "relu", OpType.ABS: "abs", OpType.CLAMP: "clamp",
}
_BINARY = {OpType.ADD: "add", OpType.SUB: "sub", OpType.MUL: "mul", OpType.DIV: "div"}
_KIND_RANK = {"const": 0, "row": 1, "elem": 2}
EXPENSIVE = {"exp", "log", "tanh", "sigmoid", "gelu", "silu", "sqrt", "rsqrt", "div"}


class _DagBuilder:
    def __init__(self, cols: int):
        self.values: list = []
        self.cols = cols
        self._memo: dict = {}

    def add(self, kind, op, args=(), attrs=None, avail=None) -> int:
        attrs = attrs or {}
        key = (op, tuple(args), tuple(sorted((k, repr(v)) for k, v in attrs.items())))
        if op not in ("load",) and key in self._memo:
            return self._memo[key]
        if avail is None:
            avail = max([self.values[a].avail for a in args], default=0)
        vid = len(self.values)
        self.values.append(Value(vid, kind, op, tuple(args), attrs, avail))
        self._memo[key] = vid
        return vid

    def kind_of(self, args) -> str:
        return max((self.values[a].kind for a in args), key=_KIND_RANK.get, default="const")

    def const(self, x: float) -> int:
        return self.add("const", "const", (), {"value": float(x)})

    def unary(self, op, a, attrs=None):
        va = self.values[a]
        if op == "rcp" and va.op == "sqrt" and va.kind == "row":
            # 1 / sqrt(x) per row -> rsqrtf(x) (2 ulp, one MUFU op)
            return self.add("row", "rsqrt", va.args)
        return self.add(self.kind_of([a]), op, (a,), attrs)

    def binary(self, op, a, b):
        va, vb = self.values[a], self.values[b]
        if op == "div" and va.kind == "row" and vb.op == "const" and vb.attrs["value"] not in (0.0,):
            # per-row value over a constant: one multiply by the reciprocal
            return self.add("row", "mul", (a, self.const(1.0 / vb.attrs["value"])))
        return self.add(self.kind_of([a, b]), op, (a, b))

    def reduce(self, op, a) -> int:
        v = self.values[a]
        if v.kind != "elem":
            # reduction of a value constant along the row
            if op == "rsum":
                return self.binary("mul", a, self.const(self.cols))
            return a
        return self.add("row", op, (a,), avail=v.avail + 1)


def acc_op_present(b) -> bool:
    return any(v.op == "acc" for v in b.values)


def build_dag(graph: DataflowGraph, op_ids: list, operands: list, cols: int,
              acc_op: Optional[int] = None):
    """Translate graph ops into a Value DAG.  Returns (values, env)."""
    b = _DagBuilder(cols)
    env: dict = {}
    if acc_op is not None:
        env[acc_op] = b.add("elem", "acc", ())
    for opd in operands:
        src = graph.ops.get(opd.op_id)
        kind = "elem" if opd.last == "vec" else "row"
        env[opd.op_id] = b.add(kind, "load", (), {"operand": opd.index})
    for oid in op_ids:
        op = graph.ops[oid]
        for i in op.inputs:
            if i in env:
                continue
            src = graph.ops[i]
            if is_mask_const(src):
                env[i] = b.add("elem", "mask", (), {"period": src.attrs.get("period"),
                                                   "offset": int(src.attrs.get("offset", 0))})
            elif src.op_type == OpType.CONSTANT:
                env[i] = b.const(src.attrs.get("value", 0.0) or 0.0)
            else:
                raise LoweringError(f"operand op {i} of op {oid} is not available")
        args = [env[i] for i in op.inputs]
        t = op.op_type
        if t in _BINARY:
            if len(args) != 2:
                raise LoweringError(f"{t.name} needs two inputs")
            if t == OpType.DIV and b.values[args[1]].kind in ("row", "const") \
                    and b.values[args[0]].kind == "elem":
                # divide by a per-row scalar: one reciprocal per row
                r = b.unary("rcp", args[1])
                env[oid] = b.binary("mul", args[0], r)
            else:
                env[oid] = b.binary(_BINARY[t], *args)
        elif t in _UNARY:
            attrs = {}
            if t == OpType.CLAMP:
                attrs = {"min": op.attrs.get("min"), "max": op.attrs.get("max")}
            env[oid] = b.unary(_UNARY[t], args[0], attrs)
        elif t == OpType.SOFTMAX:
            x = args[0]
            if b.values[x].kind == "elem" and not acc_op_present(b):
                # one-round online softmax: computed in the pass of x, usable
                # from the next one (the row engine keeps e = exp(x - m_thread))
                env[oid] = b.add("elem", "softmax", (x,), avail=b.values[x].avail + 1)
            else:
                mx = b.reduce("rmax", x)
                e = b.unary("exp", b.binary("sub", x, mx))
                s = b.reduce("rsum", e)
                env[oid] = b.binary("mul", e, b.unary("rcp", s))
        elif t == OpType.SUM:
            env[oid] = b.reduce("rsum", args[0])
        elif t == OpType.MEAN:
            env[oid] = b.binary("div", b.reduce("rsum", args[0]), b.const(cols))
        elif t == OpType.MAX:
            env[oid] = b.reduce("rmax", args[0])
        elif t == OpType.MIN:
            env[oid] = b.reduce("rmin", args[0])
        elif t == OpType.NORM:
            x = args[0]
            env[oid] = b.unary("sqrt", b.reduce("rsum", b.binary("mul", x, x)))
        elif t == OpType.RMS:
            x = args[0]
            eps = float(op.attrs.get("eps", 1e-6))
            ms = b.binary("div", b.reduce("rsum", b.binary("mul", x, x)), b.const(cols))
            env[oid] = b.unary("sqrt", b.binary("add", ms, b.const(eps)))
        else:
            raise LoweringError(f"{t.name} has no sm_100a lowering")
    return b.values, env


# ------------------------------------------------------------ heuristics
def _pick_vec(cols: int, sizes) -> int:
    smallest = min(sizes) if sizes else 4
    v = max(1, 16 // smallest)
    while v > 1 and cols % v:
        v //= 2
    return v


def _regs_per_slot(sk: SubKernel, vec: int, prefetch: set, materialize) -> int:
    """Registers one slot costs while a row is resident: the compiler keeps
    the widened fp32 copy of a prefetched 16-bit slot once it has been read,
    so every resident element is counted as one fp32 register."""
    r = vec * len([o for o in sk.operands if o.index in prefetch])
    r += vec * len(materialize)
    return max(r, 1)


def choose_row_config(sk: SubKernel, prefetch: set, materialize: set,
                      override: Optional[dict] = None) -> dict:
    sizes = [DTYPE_SIZE[o.dtype] for o in sk.operands if o.last == "vec"]
    sizes += [DTYPE_SIZE[o.dtype] for o in sk.outputs if o.kind == "full"]
    o = dict(override or {})
    vec = o.get("vec") or _pick_vec(sk.cols, sizes)
    nvec = -(-sk.cols // vec)
    per_slot = _regs_per_slot(sk, vec, prefetch, materialize)
    budget = o.get("reg_budget", 64)
    nv_max = max(1, budget // per_slot)
    # a warp per row when a row fits in 8 slots per lane: its reductions are
    # shuffles only, no block barrier (measured best for short rows)
    warp_row = (sk.passes > 0 and nvec > 32 * 2 and nvec <= 32 * 8
                and -(-nvec // 32) * per_slot <= 128 and "reg_budget" not in o)
    if "tpc" in o:
        tpc, cl = o["tpc"], o.get("cl", 1)
        team = tpc * cl
    elif warp_row:
        tpc, cl, team = 32, 1, 32
    elif "reg_budget" not in o and nvec >= 32:
        # 4..8 streamed 16-byte slots in flight per thread, at most ~96
        # resident fp32 values (measured: RMSNorm fp32 x 5120 and softmax
        # fp32 x 2048 best at 5..8 slots, RMSNorm*SiLU bf16 x 3584 at 2 slots
        # of each of its 2 streamed operands); least waste, then more slots
        streams = max(1, len(prefetch))
        hi = max(1, min(max(1, 8 // streams), 96 // per_slot))
        lo = max(1, hi // 2)
        best = None
        for nv_c in range(hi, lo - 1, -1):
            cand = 32 * (-(-(-(-nvec // nv_c)) // 32))
            waste = cand * nv_c - nvec
            key = (waste * 16 > nvec, waste, -nv_c)
            if best is None or key < best[0]:
                best = (key, cand)
        team = best[1]
        max_cta = o.get("max_tpc", 512)
        if ("max_tpc" not in o and 512 < team <= 1024 and prefetch
                and all(DTYPE_SIZE[sk.operands[i].dtype] == 4 for i in prefetch)):
            # 4-byte rows of 513..1024 threads: one 1024-thread CTA rather
            # than a 2-CTA cluster, no cross-CTA exchange per row (measured:
            # softmax fp32 4096 x 32768 189.3 -> 185.8 us, causal 134.6 ->
            # 106.7 us; 16-bit rows take the stream form below instead)
            max_cta = 1024
        cl = 1
        while team // cl > max_cta or (team % cl):
            cl *= 2
        if cl > 8:
            raise LoweringError(f"row of {sk.cols} elements is too long for one cluster")
        tpc = team // cl
        if cl > 1 and tpc % 32:
            tpc = 32 * (-(-tpc // 32))
            team = tpc * cl
    else:
        need = -(-nvec // nv_max)
        if need < 32:
            team = 1
            while team < need:
                team *= 2
        else:
            lo = 32 * (-(-need // 32))
            best = None
            for cand in range(lo, 2 * lo + 1, 32):
                nv = -(-nvec // cand)
                waste = cand * nv - nvec
                key = (waste, cand)
                if best is None or key < best[0]:
                    best = (key, cand)
            team = best[1]
        max_cta = o.get("max_tpc", 512)
        cl = 1
        while team // cl > max_cta or (team % cl):
            cl *= 2
        if cl > 8:
            raise LoweringError(f"row of {sk.cols} elements is too long for one cluster")
        tpc = team // cl
        if cl > 1 and tpc % 32:
            tpc = 32 * (-(-tpc // 32))
            team = tpc * cl
    nv = o.get("nv") or -(-nvec // team)
    stream_auto = 0
    if ("tpc" not in o and "stream" not in o and "reg_budget" not in o and cl > 1
            and tpc * cl <= 1024 and prefetch
            and all(DTYPE_SIZE[sk.operands[i].dtype] == 2 for i in prefetch)):
        # 16-bit rows long enough to need a cluster: one 1024-thread CTA per
        # row in the persistent stream form, 3 rows staged (measured: softmax
        # bf16 x 32768 77% of HBM peak vs 63% with a 2-CTA cluster per row,
        # causal 79 us vs 117 us; 4-byte rows of up to 1024 threads take one
        # 1024-thread CTA in the register form instead, chosen above: an fp32
        # row of that length is a 128 KB stage, which would not fit twice in
        # shared memory)
        tpc, cl, team = tpc * cl, 1, tpc * cl
        if team > 512 and -(-nvec // 512) <= 8 and "nv" not in o:
            # ... of 512 threads when 8 slots per thread hold the row
            # (measured, softmax bf16 4096 x 32768 after a 1 s soak: 1024
            # threads 94.7-95.5 us, 512 91.7-92.2, 256 98.4, 768 103.7)
            tpc = team = 512
            nv = -(-nvec // team)
        stream_auto = 3
    if o.get("rpc"):
        rpc = o["rpc"]
    elif tpc >= 32:
        # 256-thread CTAs; softmax rows in 128-thread CTAs, 64 with a causal
        # mask, whose visible prefixes make rows unequal work (measured with
        # CUDA-graph replay after a 1 s soak, us, 8 -> 2 warp-rows per CTA:
        # bf16 65536 x 2048 causal 71.0 -> 68.0, plain 81.3 -> 80.5 (4 per
        # CTA); fp32 causal, 2-warp rows, 4 -> 1 per CTA 135.1 -> 126.3,
        # plain 160.0 -> 159.2 (2 per CTA))
        target = 256
        if any(v.op == "softmax" for v in sk.values):
            target = 64 if any(v.op == "mask" for v in sk.values) else 128
        rpc = max(1, min(8, target // tpc))
    else:
        rpc = max(1, 256 // tpc)
    if tpc < 32 and (tpc * rpc) % 32:
        rpc = 32 // tpc
    out = {"vec": vec, "nvec": nvec, "tpc": tpc, "nv": nv, "rpc": rpc, "cl": cl,
           "min_blocks": o.get("min_blocks", 0),
           "block": tpc * rpc}
    stages = int(o.get("stream", 0) or 0) or stream_auto
    if stages >= 2:
        out.update(_stream_config(sk, prefetch, vec, nv, tpc * rpc, stages))
        # bulk staging (one bulk copy per row): default for the automatic
        # stream form (measured: softmax bf16 x 32768 97 us vs 100 us with
        # per-thread copies, causal 72.5 vs 78.5 us); slower for short rows
        if (out.get("stream") and o.get("bulk", bool(stream_auto)) and cl == 1 and rpc == 1
                and tpc >= 64):
            out.update(_bulk_stage_config(sk, prefetch, out["stream"]))
    # a causal softmax's masked row tails written by the TMA engine (bulk
    # zero stores) instead of the threads: by default in the register form
    # (measured, causal softmax fp32 4096 x 32768: 106.9 -> 103.7 us); not
    # in the bulk-staged stream form, where they share the SM's TMA unit
    # with the row copies (bf16 4096 x 32768: 57.7 -> 59.7 us)
    out["zero_tail"] = bool(o.get("zero_tail", not out.get("stream")))
    return out


def _bulk_stage_config(sk: SubKernel, prefetch: set, stages: int) -> dict:
    """Bulk-staged stream form: a stage holds whole rows of the row-indexed
    streamed operands (each 128-byte aligned), copied by one thread with one
    bulk copy each."""
    staged = [i for i in sorted(prefetch) if sk.operands[i].row_map != "zero"]
    offs, off = [], 0
    for i in staged:
        offs.append(off)
        off += -(-(sk.cols * DTYPE_SIZE[sk.operands[i].dtype]) // 128) * 128
    while stages > 2 and stages * off > STREAM_SMEM_BUDGET:
        stages -= 1
    if stages * off > STREAM_SMEM_BUDGET:
        return {}
    return {"bulk": True, "stream": stages, "stage_bytes": off, "bulk_offsets": offs,
            "smem": stages * off}


STREAM_SMEM_BUDGET = 200 * 1024


def _stream_config(sk: SubKernel, prefetch: set, vec: int, nv: int, block: int,
                   stages: int) -> dict:
    """Persistent stream form of the register engine: the row-indexed
    streamed operands are staged per thread in 16-byte lanes, ``stages`` rows
    deep (fewer when the shared-memory budget is short).  Empty when the
    form does not apply (no row-indexed streamed operand, slots narrower than
    16 bytes)."""
    staged = [i for i in sorted(prefetch) if sk.operands[i].row_map != "zero"]
    if not staged or any(DTYPE_SIZE[sk.operands[i].dtype] * vec != 16 for i in staged):
        return {}
    stage_bytes = len(staged) * nv * block * 16
    while stages > 2 and stages * stage_bytes > STREAM_SMEM_BUDGET:
        stages -= 1
    if stages * stage_bytes > STREAM_SMEM_BUDGET:
        return {}
    return {"stream": stages, "stage_bytes": stage_bytes, "smem": stages * stage_bytes}


def choose_ew_config(sk: SubKernel, override: Optional[dict] = None) -> dict:
    sizes = [DTYPE_SIZE[o.dtype] for o in sk.operands if o.last == "vec"]
    sizes += [DTYPE_SIZE[o.dtype] for o in sk.outputs]
    o = dict(override or {})
    vec = o.get("vec") or _pick_vec(sk.cols, sizes)
    nvec = -(-sk.cols // vec)
    if "tpc" in o:
        tpc = o["tpc"]
    else:
        tpc = 128 if nvec >= 128 else max(1, 1 << (max(nvec, 1) - 1).bit_length())
        tpc = min(tpc, 128)
    nv = o.get("nv") or 1
    rpc = o.get("rpc") or max(1, 256 // tpc)
    if (tpc * rpc) % 32:
        rpc = max(rpc, 32 // tpc)
    upt = o.get("upt") or 4
    return {"vec": vec, "nvec": nvec, "tpc": tpc, "nv": nv, "rpc": rpc, "upt": upt,
            "block": tpc * rpc, "tiles": -(-nvec // (tpc * nv)),
            "min_blocks": o.get("min_blocks", 0)}


def choose_rope_config(sk: SubKernel, style: str, seq: int, heads: int,
                       override: Optional[dict] = None) -> dict:
    """RoPE launch shape: one 16-byte slot of x (VEC elements, VEC/2 pairs;
    VEC pairs of the two halves with style "half") per thread, grid-stride.
    ``vec`` = 1 (set by the runtime for pointers that are not 16-byte
    aligned) moves single elements, one pair per thread."""
    o = dict(override or {})
    d = sk.cols
    x, out = sk.operands[0], sk.outputs[0]
    packed = len(sk.operands) == 2
    span = d // 2 if style == "half" else d           # elements one thread row covers
    scalar = o.get("vec") == 1
    if scalar:
        vec = 2 if style != "half" else 1
    else:
        vec = o.get("vec") or 16 // min(DTYPE_SIZE[x.dtype], DTYPE_SIZE[out.dtype])
        while vec > 1 and (span % vec or (style != "half" and vec % 2)):
            vec //= 2
        if style != "half" and vec < 2:
            vec, scalar = 2, True
    block = o.get("block") or 256
    # 2 items per thread at 256 threads (measured on bf16 [4, 4096, 32, 128]:
    # 94.6% of HBM peak; 1 item 77%, 4 items 89%, 512 threads 70%)
    upt = 1 if scalar else (o.get("upt") or 2)
    return {"vec": vec, "scalar": scalar, "style": style, "packed": packed, "seq": seq,
            "heads": heads, "spr": span // vec, "block": block, "upt": upt,
            "min_blocks": o.get("min_blocks", 0)}


SMEM_RING_BUDGET = 220 * 1024
TMA_MIN_ROWS = 2048      # below this the ring's fill time outweighs its depth
EW_TMA_MIN_ROWS = 4096   # elementwise groups take the ring from here on ...
EW_TMA_MIN_ROW_BYTES = 8192  # ... when each streamed operand's row is this long
TMA_MAX_AUTO_STAGES = 14
TMA_CONSUMER_WARPS = 20  # consumer warps per CTA the team width aims at
TMA_TEAM_MAX_ROWS = 4096 # reductions over this many rows: one warp per row,
TMA_ONE_WARP_MAX_SLOTS = 14  # when a lane holds at most this many slots of it


def choose_row_tma_config(sk: SubKernel, prefetch: set, materialize: dict,
                          override: Optional[dict] = None):
    """Config of the TMA-staged row engine, or None when it does not apply.

    Staged operands are the row-indexed ones (``prefetch``); a stage holds one
    row of each, every part 128-byte aligned.  The engine needs whole 16-byte
    slots and at least 6 stages in the shared-memory budget.
    """
    o = dict(override or {})
    # Chosen from 2048 rows on (measured with teams of warps per row, CUDA-
    # graph replay, rotated outputs: RMSNorm*SiLU bf16 x 3584 at 8192 rows
    # 30.0 -> 29.2 us against one warp per row, at 2048 rows 10.0 -> 9.65 us
    # against the register engine; RMSNorm fp32 2048 x 5120 15.8 -> 14.4 us);
    # never under a vec override, which the runtime uses for inputs that are
    # not 16-byte aligned -- bulk copies need 16-byte alignment
    if o.get("engine") in ("regs", "ew") or "vec" in o or not prefetch:
        return None
    if o.get("engine") != "tma" and sk.rows < TMA_MIN_ROWS:
        return None
    if any(v.op == "softmax" for v in sk.values):
        return None
    staged = sorted(prefetch)
    sizes = [DTYPE_SIZE[sk.operands[i].dtype] for i in staged]
    sizes += [DTYPE_SIZE[x.dtype] for x in sk.operands if x.last == "vec"]
    sizes += [DTYPE_SIZE[x.dtype] for x in sk.outputs if x.kind == "full"]
    vec = 16 // min(sizes)
    if sk.cols % vec:
        return None
    offsets, off = [], 0
    for i in staged:
        offsets.append(off)
        off += -(-(sk.cols * DTYPE_SIZE[sk.operands[i].dtype]) // 128) * 128
    stage_bytes = off
    # per-column operands (weights, bias vectors) are copied into shared
    # memory once per CTA instead of being re-read by every row
    consts, const_offsets, coff = [], [], 0
    for x in sk.operands:
        if x.last == "vec" and x.row_map == "zero":
            consts.append(x.index)
            const_offsets.append(coff)
            coff += -(-(sk.cols * DTYPE_SIZE[x.dtype]) // 128) * 128
    s_max = o.get("stages") or min(32, (SMEM_RING_BUDGET - coff) // stage_bytes)
    # at least 6 stages (measured with 6 teams on 6 stages, RMSNorm*SiLU
    # bf16 x 8192 at 2048 / 8192 rows: 19.9 / 70.0 us ring, 20.3 / 73.5
    # register engine)
    if s_max < o.get("min_stages", 6) and o.get("engine") != "tma":
        return None
    # Stage s is always consumed by team s % NC, which needs STAGES % NC == 0:
    # a team then meets the stages it owns in order and can never wait on a
    # phase two ahead of the one in flight (mbarrier parity would alias).
    # A team is TW warps; NC * TW + 1 warps per CTA.  Unless tuned: the most
    # stages up to 14 (15 measured slower on RMSNorm*SiLU 8192 x 3584), NC
    # preferring 7 then 5 teams, and TW for ~20 consumer warps, except one
    # warp per row for reductions over >= 4096 rows.  Measured with CUDA-
    # graph replay after a 1.5 s soak under the 1 kW power cap (SM clock
    # ~1740 MHz), us: RMSNorm fp32 2048 x 5120 15.7 (register engine) ->
    # 14.6 (5 teams of 4 warps) / 14.5 (of 2); RMSNorm*SiLU bf16 2048 x 3584
    # 9.9 -> 9.65 (7 teams of 3); 8-op bf16 chain 16384 x 8192 145.8
    # (elementwise kernel) -> 139.2 (5 teams of 4; of 2: slower than the
    # elementwise kernel); RMSNorm*SiLU 8192 x 3584 30.0 with one warp per
    # row, 30.1 with teams of 2, 30.9 with teams of 3 (at full clocks,
    # before the soak, teams of 3 had been faster: 29.2 vs 30.0) -- one warp
    # per row only while a lane holds at most 14 slots of it: RMSNorm*SiLU
    # bf16 x 4096 (16 slots) at 4096 / 8192 rows 21.3 / 40.1 us with one
    # warp, 18.4 / 35.0 with 6 teams of 4; RMSNorm fp32 8192 x 5120 60.6 vs
    # 58.4.
    tw_req = int(o["tw"]) if "tw" in o else None
    if tw_req is not None and (tw_req < 1 or 32 * (tw_req + 1) > 1024):
        raise LoweringError(f"row ring team of {tw_req} warps does not fit a CTA")
    one_warp = tw_req == 1 or (tw_req is None and sk.passes > 0 and sk.rows >= TMA_TEAM_MAX_ROWS
                               and sk.cols // vec <= 32 * TMA_ONE_WARP_MAX_SLOTS)
    if one_warp:
        # one warp per row: the most stages, 6..8 consumer warps measured best
        st_cap = max(2, s_max)
        nc_ranges = [[o["nc"]]] if "nc" in o else [range(8, 5, -1), range(14, 1, -1)]
    else:
        st_cap = max(2, s_max if "stages" in o else min(s_max, TMA_MAX_AUTO_STAGES))
        # (4..8 teams over any stage count before fewer teams)
        nc_ranges = [[o["nc"]]] if "nc" in o else [[7, 5, 6, 8, 4], [3, 2, 1]]
    nc_ranges = [[nc for nc in r if nc * (tw_req or 1) <= 31] for r in nc_ranges]
    best = None
    for ncs in nc_ranges:
        for st in range(st_cap, 1, -1):
            for nc in ncs:
                if st % nc == 0:
                    best = (st, nc)
                    break
            if best:
                break
        if best:
            break
    if best is None:
        return None
    stages, nc = best
    if one_warp:
        tw = 1
    elif tw_req:
        tw = tw_req
    else:
        # the team width nearest TMA_CONSUMER_WARPS / NC whose last slot
        # round wastes at most 10% of the team's slots (measured, RMSNorm*SiLU
        # bf16 2048 x 4096, 6 teams: 2 / 4 warps (no waste) 10.9 / 10.6 us,
        # 3 warps (12.5% waste) 12.6 us; x 3584, 7 teams: 3 warps (7% waste)
        # 9.65 us, 4 warps (14%) 9.78)
        target = TMA_CONSUMER_WARPS / nc
        nvec_r = sk.cols // vec
        cands = [t for t in range(1, 31 // nc + 1)
                 if -(-nvec_r // (32 * t)) * 32 * t - nvec_r <= 0.1 * nvec_r]
        tw = min(cands, key=lambda t: (abs(t - target), -t)) if cands else \
            max(1, min(31 // nc, round(target)))
    nvec = sk.cols // vec
    nv = -(-nvec // (32 * tw))
    mat = dict(materialize)
    if nv * vec * len(mat) > 64 or not o.get("materialize", True):
        mat = {}                     # recompute instead of holding in registers
    return {"engine": "tma", "vec": vec, "nvec": nvec, "nv": nv, "nc": nc, "tw": tw,
            "stages": stages, "stage_bytes": stage_bytes, "staged": staged,
            "stage_offsets": offsets, "consts": consts, "const_offsets": const_offsets,
            "const_bytes": coff,
            "row_bytes": sum(sk.cols * DTYPE_SIZE[sk.operands[i].dtype] for i in staged),
            "smem": stages * stage_bytes + coff + (2 * stages + 1) * 8 + 16 + 128,
            "materialize": sorted(mat.items()), "prefetch": staged, "cl": 1}
