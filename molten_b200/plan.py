"""Specialise a fusion group for concrete input shapes/dtypes -> GroupPlan."""

from __future__ import annotations

from typing import Optional

from .ir import DataflowGraph, OpType, TensorShape
from .lowering import (
    DTYPE_SIZE, GroupPlan, LoweringError, Operand, OutputSpec, SubKernel,
    broadcast_shapes, build_dag, canon_dtype, choose_ew_config,
    choose_row_config, choose_row_tma_config, choose_rope_config, classify_operand,
    rms_prologue, attention_pattern,
    group_boundary, infer_shapes,
    is_mask_const, prod, promote, split_group, EXPENSIVE, EW_TMA_MIN_ROWS,
    EW_TMA_MIN_ROW_BYTES,
)

DEFAULT_SYMBOLIC_DIM = 1024
ATTN_SMEM_LIMIT = 232448          # dynamic shared memory one sm_100 CTA may opt into
ATTN_POLY = (0, 0)                # exponentials per 32 on the FMA pipe (pass 0, pass 1)
ATTN_SUM16 = False                # pass-0 row sums from f16 exponential pairs
ATTN_X2 = False                   # packed fp32 pairs for exponent arguments and sums


def declared_shape(op, symbols: dict) -> tuple:
    """Concrete stand-in for a declared (possibly symbolic) TensorShape."""
    shp = op.shape
    if shp is None or not isinstance(shp, TensorShape) or not shp.dims:
        return (DEFAULT_SYMBOLIC_DIM,)
    out = []
    for d in shp.dims:
        if isinstance(d, int):
            out.append(d)
        else:
            out.append(symbols.setdefault(str(d), DEFAULT_SYMBOLIC_DIM))
    return tuple(out)


def _op_dtypes(graph, ordered, dtypes: dict) -> dict:
    """torch-style result dtype per op (Python-scalar constants don't promote)."""
    out = dict(dtypes)
    for oid in ordered:
        op = graph.ops[oid]
        ds = []
        for i in op.inputs:
            src = graph.ops[i]
            if src.op_type == OpType.CONSTANT:
                continue
            ds.append(out[i])
        if op.op_type == OpType.ROTATE:
            out[oid] = out[op.inputs[0]]          # out.to(x.dtype), ops.py:35
            continue
        out[oid] = promote(ds) if ds else "float32"
    return out


def plan_group(graph: DataflowGraph, group_op_ids, input_shapes: dict,
               input_dtypes: dict, name: str,
               tune: Optional[dict] = None) -> GroupPlan:
    """Lower one fusion group for the given shapes/dtypes of its inputs.

    ``input_shapes``/``input_dtypes`` map each non-constant external op id
    (graph INPUT ops, or ops computed by another group) to its concrete
    shape / dtype.
    """
    tune = tune or {}
    ext, outs, ordered = group_boundary(graph, group_op_ids)
    inputs = [i for i in ext if graph.ops[i].op_type != OpType.CONSTANT]
    for i in inputs:
        if i not in input_shapes or i not in input_dtypes:
            raise LoweringError(f"no shape/dtype for input op {i}")
    known = {i: tuple(int(d) for d in input_shapes[i]) for i in inputs}
    for i in ext:
        if graph.ops[i].op_type == OpType.CONSTANT:
            known[i] = ()
    shapes = infer_shapes(graph, ordered, known)
    dts = {i: canon_dtype(input_dtypes[i]) for i in inputs}
    dts = _op_dtypes(graph, ordered, dts)

    # {"gemm": {"prologue": True}} runs RMSNorm -> GEMM as one GEMM that
    # normalises A as it is staged; off by default: measured slower than the
    # row kernel + GEMM pair (bf16 8192x4096x14336: 1308 vs 892 us; 64 rows:
    # 64 vs 44 us) -- the in-place transform of every A stage competes with
    # the tensor core for the same shared memory and lengthens each stage
    # {"attn": {"fused": False}} runs attention scores as GEMM + row softmax
    parts = split_group(graph, ordered, outs,
                        fuse_prologue=(tune.get("gemm") or {}).get("prologue", False),
                        fuse_attention=(tune.get("attn") or {}).get("fused", True))
    # intermediates between the sub-kernels of one group are stored in fp32,
    # so a split group still rounds once (at its outputs); a MATMUL operand
    # keeps its 16-bit type because the tensor cores read it
    mm_operands = {i for o in ordered if graph.ops[o].op_type == OpType.MATMUL
                   for i in graph.ops[o].inputs}
    storage = dict(dts)
    produced_by = {}
    for k, (_, ops) in enumerate(parts):
        for o in ops:
            produced_by[o] = k
    out_set = set(outs)
    kernels = []
    temps = {}
    for k, (family, ops) in enumerate(parts):
        ops_set = set(ops)
        sk_ext = []
        for o in ops:
            for j in graph.ops[o].inputs:
                if j not in ops_set and j not in sk_ext:
                    sk_ext.append(j)
        sk_ext.sort()
        later = set()
        for _, ops2 in parts[k + 1:]:
            for o in ops2:
                later.update(graph.ops[o].inputs)
        sk_outs = [o for o in ops if o in out_set or o in later]
        for o in sk_outs:
            if o not in out_set:
                if o not in mm_operands:
                    storage[o] = "float32"
                temps[o] = (shapes[o], storage[o])
        sub = _plan_sub(graph, family, ops, sk_ext, sk_outs, shapes, storage, tune)
        if sub.family == "gemm" and sub.config.get("split3"):
            # fp32 operands: a kernel before the GEMM writes each as three
            # stacked bf16 planes, which the GEMM's TMA copies read
            planes = []
            for idx in (sub.a_operand, sub.b_operand):
                opd = sub.operands[idx]
                key = ("split3", opd.op_id)
                if key not in temps:
                    temps[key] = ((3,) + tuple(int(d) for d in opd.shape), "bfloat16")
                    kernels.append(_plan_split3(opd, key))
                planes.append(key)
            sub.config["planes"] = planes
        kernels.append(sub)

    return GroupPlan(
        name=name, inputs=inputs,
        input_dtypes=[dts[i] for i in inputs],
        input_shapes=[known[i] for i in inputs],
        outputs=list(outs), output_dtypes=[dts[o] for o in outs],
        output_shapes=[shapes[o] for o in outs],
        kernels=kernels, temps=temps)


SPLIT3_BLOCK = 256


def _plan_split3(opd: Operand, key) -> SubKernel:
    """The kernel that writes GEMM operand ``opd`` (fp32, or 16-bit next to
    an fp32 operand) as three bf16 planes x0, x1, x2 with x ~ x0 + x1 + x2,
    stacked as [3, *shape] (molten/gemm_sm100.cuh, SPLIT3)."""
    shape = tuple(int(d) for d in opd.shape)
    cols = shape[-1]
    rows = prod(shape[:-1]) if len(shape) > 1 else 1
    src = Operand(index=0, op_id=opd.op_id, name=opd.name, dtype=opd.dtype, shape=shape,
                  last="vec", row_map="full", row_terms=())
    out = OutputSpec(index=0, op_id=key, dtype="bfloat16", shape=(3,) + shape, kind="full")
    sk = SubKernel(family="split3", op_ids=[], operands=[src], outputs=[out], rows=rows, cols=cols)
    total = rows * cols
    sk.config = {"block": SPLIT3_BLOCK, "total": total, "vec": 4 if total % 4 == 0 else 1}
    return sk


CAUSAL_THREADS = 256
CAUSAL_SPLIT_MIN_COLS = 8192      # rows from which the split causal kernel is the default
CAUSAL_ZERO_SLOTS = 4             # 16-byte zero stores per thread in one zero tile
CAUSAL_INTERLEAVE = True          # launch order: each row CTA next to its zero tiles
CAUSAL_ZERO_CTAS = 0              # persistent zero CTAs (0: one CTA per zero tile)


def _plan_causal_softmax(graph, ops, ext, outs, shapes, dts, tune) -> Optional[SubKernel]:
    """softmax(x + causal_mask) over the last dim, with nothing else in the
    group, as the split causal kernel (molten/causal_softmax.cuh): row CTAs
    for the visible logits, zero-tile CTAs for the masked rest.  None when
    the group is anything else or the split is not chosen."""
    from .lowering import _reduces_last_dim
    if len(ops) != 2 or len(outs) != 1:
        return None
    add, smx = (graph.ops[o] for o in ops)
    if add.op_type != OpType.ADD or smx.op_type != OpType.SOFTMAX or outs[0] != ops[1] \
            or list(smx.inputs) != [ops[0]]:
        return None
    masks = [i for i in add.inputs if is_mask_const(graph.ops[i])]
    xs = [i for i in add.inputs if i not in masks]
    if len(masks) != 1 or len(xs) != 1 or xs[0] not in ext:
        return None
    x_id, mask = xs[0], graph.ops[masks[0]]
    shape = tuple(int(d) for d in shapes[x_id])
    if not shape or tuple(shapes[ops[1]]) != shape or not _reduces_last_dim(smx, len(shape)):
        return None
    dt = dts[x_id]
    if dt not in ("float32", "bfloat16", "float16") or dts[ops[1]] != dt:
        return None
    cols = shape[-1]
    rows = prod(shape[:-1]) if len(shape) > 1 else 1
    esz = DTYPE_SIZE[dt]
    period = int(mask.attrs.get("period") or cols)
    offset = int(mask.attrs.get("offset") or 0)
    if (cols * esz) % 16 or period < 1 or offset < 0:
        return None
    o = tune.get("row") or {}
    # chosen by itself for long rows unless a tune asks for the row engine's
    # own forms
    forced = any(k in o for k in ("stream", "zero_tail", "bulk", "engine", "tpc", "cl"))
    if not o.get("causal_split", cols >= CAUSAL_SPLIT_MIN_COLS and rows >= 148 and not forced):
        return None
    vec = 16 // esz
    zcols = CAUSAL_THREADS * vec * int(o.get("causal_zero_slots", CAUSAL_ZERO_SLOTS))
    zt = -(-cols // zcols) if cols >= CAUSAL_SPLIT_MIN_COLS else 0
    zt = int(o.get("causal_zero_tiles", zt))
    if zt > 0 and zt * zcols < cols:
        # fewer tiles than asked-for tile widths: widen them to cover the row
        zcols = -(-cols // (zt * vec)) * vec
    interleave = bool(o.get("causal_interleave", CAUSAL_INTERLEAVE)) and zt > 0
    # persistent zero CTAs (0: one CTA per zero tile)
    zpersist = int(o.get("causal_zero_ctas", CAUSAL_ZERO_CTAS)) if zt > 0 else 0
    if rows * (1 + zt) >= 2 ** 31:
        return None
    if zt > 0 and rows * zt >= 2 ** 40:
        return None
    src = graph.ops[x_id]
    opd = Operand(index=0, op_id=x_id, name=src.name or f"op{x_id}", dtype=dt, shape=shape,
                  last="vec", row_map="full", row_terms=())
    out = OutputSpec(index=0, op_id=ops[1], dtype=dt, shape=shape, kind="full")
    sk = SubKernel(family="causal", op_ids=list(ops), operands=[opd], outputs=[out],
                   rows=rows, cols=cols)
    # the kernel's exponentials use the EX2 unit (__expf of x - M) and one
    # reciprocal per row for every output type: within the fp32 parity bar
    # (see _softmax_exp in emit.py) and 3% faster on fp32 4096 x 32768
    sk.precise = False
    sk.config = {"threads": CAUSAL_THREADS, "vec": vec, "zt": zt, "zcols": zcols,
                 "period": period, "offset": offset, "precise": sk.precise,
                 "interleave": interleave, "zpersist": zpersist,
                 # 32-byte zero stores when every row starts on a 32-byte boundary
                 "w32": bool(o.get("causal_w32", True)) and (cols * esz) % 32 == 0}
    return sk


def _plan_sub(graph, family, ops, ext, outs, shapes, dts, tune) -> SubKernel:
    if family in ("row", "ew"):
        cs = _plan_causal_softmax(graph, ops, ext, outs, shapes, dts, tune)
        if cs is not None:
            return cs
    if family == "gemm":
        return _plan_gemm(graph, ops, ext, outs, shapes, dts, tune)
    if family == "attn":
        return _plan_attn(graph, ops, outs, shapes, dts, tune)
    if family == "rope":
        return _plan_rope(graph, ops, outs, shapes, dts, tune)
    it = ()
    for o in ops:
        it = broadcast_shapes(it, shapes[o])
    for j in ext:
        src = graph.ops[j]
        if src.op_type == OpType.CONSTANT:
            continue
        it = broadcast_shapes(it, shapes[j])
    if not it:
        it = (1,)
    rows, cols = prod(it[:-1]), int(it[-1])
    operands = []
    for j in ext:
        src = graph.ops[j]
        if src.op_type == OpType.CONSTANT:
            continue
        last, row_map, terms = classify_operand(shapes[j], it)
        operands.append(Operand(index=len(operands), op_id=j, name=src.name or f"op{j}",
                                dtype=dts[j], shape=shapes[j], last=last,
                                row_map=row_map, row_terms=terms))
    outputs = []
    row_shape = tuple(it[:-1]) + (1,)
    for o in outs:
        s = shapes[o]
        s_pad = (1,) * (len(it) - len(s)) + tuple(s)
        if s_pad == tuple(it):
            kind = "full"
        elif s_pad == row_shape:
            kind = "row"
        else:
            raise LoweringError(f"output of op {o} with shape {s} is neither the "
                                f"row shape {it} nor one value per row")
        outputs.append(OutputSpec(index=len(outputs), op_id=o, dtype=dts[o], shape=s, kind=kind))
    values, env = build_dag(graph, ops, operands, cols)
    sk = SubKernel(family=family, op_ids=list(ops), operands=operands, outputs=outputs,
                   rows=rows, cols=cols, values=values,
                   out_values=[env[o] for o in outs])
    sk.precise = any(o.dtype == "float32" for o in outputs)
    needed = _needed(values, sk.out_values)
    sk.passes = max([values[v].avail for v in needed], default=0)
    if family == "ew" and sk.passes:
        family = sk.family = "row"
    key = f"{sk.family}"
    override = tune.get(key) or {}
    if sk.family == "row":
        prefetch, materialize = _row_storage(sk, needed)
        tma = choose_row_tma_config(sk, prefetch, materialize, override)
        if tma is not None:
            sk.config = tma
        else:
            sk.config = choose_row_config(sk, prefetch, materialize, override)
            sk.config["engine"] = "regs"
            sk.config["prefetch"] = sorted(prefetch)
            sk.config["materialize"] = sorted(materialize.items())
    else:
        # the TMA ring with teams of warps per row, from EW_TMA_MIN_ROWS rows
        # of at least EW_TMA_MIN_ROW_BYTES per streamed operand with at least
        # 4 stages, or when asked ({"ew": {"engine": "tma"}}) (measured, the
        # chain at 4096 x 4096: 19.4 us ring, 20.7 elementwise; 8192 x 2048,
        # 4 KB rows: 21.2-21.7 ring, 20.5 elementwise)
        # (measured, 8-op bf16 chain 16384 x 8192: 132.6 us as elementwise
        # kernel, 125.2 us on 5 stages with teams of 4 warps; with one warp
        # per row the ring's consumers were compute-bound at 50% of HBM)
        prefetch = {o.index for o in sk.operands if o.last == "vec" and o.row_map != "zero"}
        tma = None
        if override.get("engine") == "tma":
            tma = choose_row_tma_config(sk, prefetch, {}, dict(override, min_stages=2))
        elif (override.get("engine") is None and "vec" not in override
              and sk.rows >= EW_TMA_MIN_ROWS
              and all(sk.cols * DTYPE_SIZE[sk.operands[i].dtype] >= EW_TMA_MIN_ROW_BYTES
                      for i in prefetch)):
            tma = choose_row_tma_config(sk, prefetch, {},
                                        dict(override, engine="tma", min_stages=4))
            if tma is not None and tma["stages"] < 4:
                tma = None
        if tma is not None:
            sk.family = "row"
            sk.config = tma
        else:
            sk.config = choose_ew_config(sk, override)
    sk.config["needed"] = sorted(needed)
    return sk


def _needed(values, roots) -> set:
    seen, stack = set(), list(roots)
    while stack:
        v = stack.pop()
        if v in seen:
            continue
        seen.add(v)
        stack.extend(values[v].args)
    return seen


def pass_closures(values, sk: SubKernel, needed: set, materialized: dict):
    """Elem values each pass must compute, stopping at materialized ones.

    ``materialized`` maps a value id to the pass that computes and stores it;
    later passes read the stored copy instead of recomputing it.

    Pass p (< passes) computes the arguments of the reductions whose result
    becomes available at p + 1; the final pass computes the outputs.
    """
    roots = {p: [] for p in range(sk.passes + 1)}
    for v in needed:
        val = values[v]
        if val.op in ("rsum", "rmax", "rmin", "softmax"):
            roots[val.avail - 1].append(val.args[0])
    roots[sk.passes] += [v for v in sk.out_values if values[v].kind == "elem"]
    # a value materialized at pass p is computed there, needed there or not
    for v, pm in materialized.items():
        if values[v].kind == "elem" and pm <= sk.passes:
            roots[pm].append(v)
    closures = {}
    for p, rs in roots.items():
        seen, stack = set(), list(rs)
        while stack:
            v = stack.pop()
            if v in seen or values[v].kind != "elem":
                continue
            seen.add(v)
            if v in materialized and p > materialized[v]:
                continue
            stack.extend(values[v].args)
        closures[p] = seen
    return closures


EARLY_OPS = {"exp", "log", "tanh", "sigmoid", "gelu", "silu"}


def _row_storage(sk: SubKernel, needed: set):
    values = sk.values
    # a softmax keeps its exponentials in registers from the pass of its input
    soft = {v: values[v].avail - 1 for v in needed if values[v].op == "softmax"}
    naive = pass_closures(values, sk, needed, soft)
    first = {}
    uses = {}
    for p in sorted(naive):
        for v in naive[p]:
            first.setdefault(v, p)
            uses.setdefault(v, set()).add(p)
    materialize = dict(soft)
    for v, ps in uses.items():
        val = values[v]
        if val.op in EXPENSIVE and max(ps) > first[v] and v not in materialize:
            materialize[v] = first[v]
    # transcendental terms of the row's own elements that only a later pass
    # uses (silu(gate) in RMSNorm * SiLU(gate)): computed in the reduction
    # pass and kept in registers, so their XU work overlaps the row's
    # reduction instead of queueing behind it at the end (measured:
    # RMSNorm * SiLU bf16 2048 x 3584, register engine, 9.32 -> 8.72-8.81 us,
    # bit-identical); at most two, for the register budget
    early = [v for v in sorted(uses) if values[v].op in EARLY_OPS and values[v].kind == "elem"
             and values[v].avail == 0 and first[v] > 0 and v not in materialize]
    for v in early[:2]:
        materialize[v] = 0
    prefetch = set()
    for opd in sk.operands:
        if opd.last == "vec" and opd.row_map != "zero":
            prefetch.add(opd.index)
    return prefetch, materialize


def _plan_rope(graph, ops, outs, shapes, dts, tune) -> SubKernel:
    """One ROTATE: operands x, then freqs or cos and sin, in input order."""
    r = ops[0]
    op = graph.ops[r]
    x_shape = shapes[op.inputs[0]]
    operands = []
    for j in op.inputs:
        src = graph.ops[j]
        if src.op_type == OpType.CONSTANT:
            raise LoweringError("ROTATE operands must be tensors")
        operands.append(Operand(index=len(operands), op_id=j, name=src.name or f"op{j}",
                                dtype=dts[j], shape=shapes[j], last="vec", row_map="full"))
    if outs != [r]:
        raise LoweringError("the ROTATE sub-kernel has one output")
    outputs = [OutputSpec(index=0, op_id=r, dtype=dts[r], shape=shapes[r], kind="full")]
    sk = SubKernel(family="rope", op_ids=[r], operands=operands, outputs=outputs,
                   rows=prod(x_shape[:-1]), cols=int(x_shape[-1]))
    sk.precise = True
    sk.config = choose_rope_config(sk, op.attrs.get("style") or "interleaved",
                                   int(x_shape[-3]), int(x_shape[-2]), tune.get("rope") or {})
    return sk


def _plan_attn(graph, ops, outs, shapes, dts, tune) -> SubKernel:
    """Fused attention scores: P = softmax(q k^T * scale), q [.., m, d],
    k [.., n, d], leading dims = independent problems (heads)."""
    t, m, mul, sm = attention_pattern(graph, ops, set(outs))
    q_id, k_id = graph.ops[m].inputs[0], graph.ops[t].inputs[0]
    qs, ks = tuple(shapes[q_id]), tuple(shapes[k_id])
    if len(qs) < 2 or len(ks) < 2 or qs[-1] != ks[-1] or (len(ks) > 2 and qs[:-2] != ks[:-2]):
        raise LoweringError(f"attention scores need q [.., m, d] and k [.., n, d]: {qs}, {ks}")
    if dts[q_id] != dts[k_id] or dts[q_id] == "float32":
        raise LoweringError("attention scores take bf16 or fp16 q and k")
    batch = prod(ks[:-2]) if len(ks) > 2 else 1
    M = int(qs[-2]) if batch > 1 else prod(qs[:-1])
    N, D = int(ks[-2]), int(qs[-1])
    if D % 8 or D > 256:
        raise LoweringError("attention head dim must be a multiple of 8, at most 256")
    if max(batch * M, batch * N) >= 2 ** 31:
        raise LoweringError("attention rows beyond the 32-bit TMA coordinate range")
    scale = 1.0
    if mul is not None:
        c = [i for i in graph.ops[mul].inputs if i != m][0]
        scale = float(graph.ops[c].attrs["value"])
    operands = [Operand(index=i, op_id=j, name=graph.ops[j].name or f"op{j}", dtype=dts[j],
                        shape=shapes[j], last="vec", row_map="full")
                for i, j in enumerate((q_id, k_id))]
    outputs = [OutputSpec(index=0, op_id=sm, dtype=dts[sm], shape=shapes[sm], kind="full")]
    sk = SubKernel(family="attn", op_ids=list(ops), operands=operands, outputs=outputs,
                   rows=batch * M, cols=N, m=M, n=N, k=D, a_operand=0, b_operand=1)
    if DTYPE_SIZE[dts[sm]] != 2:
        raise LoweringError("attention scores are stored as bf16 or fp16")
    if M < 1 or N < 1:
        raise LoweringError("attention scores need at least one row and one column")
    o = dict(tune.get("attn") or {})
    bn = int(o.get("bn") or min(256, 64 * -(-N // 64)))
    if bn % 64 or not 64 <= bn <= 256:
        raise LoweringError(f"attention column block {bn} must be 64..256, a multiple of 64")
    dch = -(-D // 64)
    # epilogue warps: 4 per TMEM lane quarter when a tile has 4 column parts
    # of whole 32-column chunks, else 2
    # epilogue warps: 4 per TMEM lane quarter, each a quarter of every
    # tile's columns ("groups": 2 splits them into two groups taking
    # alternate tiles -- measured slower: each group then owns one of the two
    # accumulator buffers and waits for its next tile's MMA serially)
    groups = int(o.get("groups") or 1)
    epi = int(o.get("epi_warps") or (16 if (bn // 32) % (4 // groups) == 0 else 8))
    if epi not in (4, 8, 12, 16) or groups not in (1, 2) or (epi // 4) % groups:
        raise LoweringError(f"{epi} epilogue warps cannot form {groups} groups")
    parts = epi // 4 // groups
    if (bn // 32) % parts:
        raise LoweringError(f"{parts} column parts cannot split a {bn}-column block")
    # resident Q tile + K ring + per-warp staging tiles of 32 rows x (up to
    # 64) columns (two per warp up to 8 warps) + the (max, sum) exchange
    scols = 64 if (bn // parts) % 64 == 0 else 32
    out_bytes = epi * (2 if epi <= 8 else 1) * 32 * scols * 2
    q_bytes, stage, stat_bytes = dch * 128 * 128, bn * 128, 2 * epi * 32 * 8
    acc_bufs = 4 if 4 * bn <= 512 else 2                  # TMEM accumulator buffers
    fit = (ATTN_SMEM_LIMIT - 2048 - out_bytes - stat_bytes - q_bytes) // stage
    stages = int(o.get("stages") or max(2, min(8, fit)))
    smem = (q_bytes + stages * stage + out_bytes + stat_bytes + (2 * stages + 2 * acc_bufs + 7) * 8
            + 16 + 1024)
    if smem > ATTN_SMEM_LIMIT:
        raise LoweringError(f"attention tile needs {smem} bytes of shared memory")
    rows_aligned = (N * 2) % 16 == 0
    # a TMA store box of 32 rows stays inside its head when m % 32 == 0; with
    # one head the rows past m lie outside the tensor and are dropped
    tma_store = bool(o.get("tma_store", True)) and rows_aligned and (M % 32 == 0 or batch == 1)
    # of each 32 exponentials per pass, how many run on the FMA pipe
    poly = o.get("poly", ATTN_POLY)
    poly = [int(poly), int(poly)] if isinstance(poly, (int, float)) else [int(x) for x in poly]
    if len(poly) != 2 or not all(0 <= x <= 32 for x in poly):
        raise LoweringError(f"attention poly split {poly} must be two counts in 0..32")
    sk.config = {"bn": bn, "dch": dch, "stages": stages, "smem_bytes": smem,
                 "threads": 32 * (4 + epi), "epi_warps": epi, "groups": groups,
                 "scale": scale, "batch": int(batch), "rows_aligned": rows_aligned,
                 "tma_store": tma_store, "poly": poly, "store_cols": scols,
                 "sum16": bool(o.get("sum16", ATTN_SUM16)), "x2": bool(o.get("x2", ATTN_X2))}
    return sk


def _plan_gemm(graph, ops, ext, outs, shapes, dts, tune) -> SubKernel:
    mm = ops[0]
    a_id, b_id = graph.ops[mm].inputs
    # RMSNorm prologue: A = x / RMS(x) * w, computed as the GEMM stages x
    pro = rms_prologue(graph, mm, set(ops), set(outs))
    prologue = None
    if pro is not None and all(o in ops for o in pro):
        r_id, d_id, mul_id = pro
        x_id = graph.ops[d_id].inputs[0]
        w_id = [i for i in graph.ops[mul_id].inputs if i != d_id][0]
        prologue = {"eps": float(graph.ops[r_id].attrs.get("eps", 1e-6)), "w_op": w_id}
        a_id = x_id
        ops = [o for o in ops if o not in pro]
    # B given as TRANSPOSE(Bt) with Bt [N, K]: read K-major, no copy
    b_kmajor = graph.ops[b_id].op_type == OpType.TRANSPOSE and b_id in ops
    if b_kmajor:
        if b_id in outs:
            raise LoweringError("a transposed GEMM operand cannot also be an output")
        b_id = graph.ops[b_id].inputs[0]
        ops = [o for o in ops if graph.ops[o].op_type != OpType.TRANSPOSE]
    a_shape, b_shape = shapes[a_id], shapes[b_id]
    K, N = (int(b_shape[-1]), int(b_shape[-2])) if b_kmajor else (int(b_shape[-2]), int(b_shape[-1]))
    # B with leading dims: a batch of independent problems stacked in memory
    batch = prod(b_shape[:-2]) if len(b_shape) > 2 else 1
    M = int(a_shape[-2]) if batch > 1 else prod(a_shape[:-1])
    if min(M, K, N, batch) <= 0:
        raise LoweringError(f"MATMUL with an empty dimension (M={M}, K={K}, N={N}, batch={batch}) "
                            "has no sm_100a lowering")
    if batch > 1 and prologue is not None:
        raise LoweringError("the RMSNorm prologue takes an unbatched B")
    # fp32 operands run on the bf16 tensor cores as three bf16 planes each
    split3 = "float32" in (dts[a_id], dts[b_id])
    if split3 and prologue is not None:
        raise LoweringError("the RMSNorm prologue takes 16-bit GEMM operands")
    if (3 if split3 else 1) * max(batch * M, batch * K, batch * N) >= 2 ** 31:
        raise LoweringError("GEMM rows beyond the 32-bit TMA coordinate range")
    it = shapes[mm]
    for o in ops:
        it = broadcast_shapes(it, shapes[o])
    if prod(it[:-1]) != batch * M or it[-1] != N:
        raise LoweringError("the GEMM epilogue broadcasts beyond the product shape")
    operands = []
    a_idx = b_idx = None
    for j in ext:
        src = graph.ops[j]
        if src.op_type == OpType.CONSTANT:
            continue
        if j in (a_id, b_id) and not any(j in graph.ops[o].inputs for o in ops[1:]):
            last, row_map, terms = "vec", "full", ()
        elif prologue is not None and j == prologue["w_op"] \
                and not any(j in graph.ops[o].inputs for o in ops[1:]):
            last, row_map, terms = "vec", "zero", ()        # per-K weight of the prologue
        else:
            last, row_map, terms = classify_operand(shapes[j], it)
        operands.append(Operand(index=len(operands), op_id=j, name=src.name or f"op{j}",
                                dtype=dts[j], shape=shapes[j], last=last,
                                row_map=row_map, row_terms=terms))
        if j == a_id:
            a_idx = operands[-1].index
        if j == b_id:
            b_idx = operands[-1].index
    if a_id == b_id:
        b_idx = a_idx
    if not split3 and dts[a_id] != dts[b_id]:
        raise LoweringError("the tensor-core GEMM takes bf16 x bf16, fp16 x fp16 or fp32 operands")
    if prologue is not None:
        w_id = prologue["w_op"]
        w_shape = tuple(int(v) for v in shapes[w_id])
        if prod(w_shape) != K or w_shape[-1] != K or graph.ops[w_id].op_type == OpType.CONSTANT:
            raise LoweringError("the RMSNorm prologue needs a weight vector of length K")
        prologue["w"] = [o.index for o in operands if o.op_id == w_id][0]
        prologue["w_dtype"] = dts[w_id]
    outputs = []
    for o in outs:
        s = shapes[o]
        s_pad = (1,) * (len(it) - len(s)) + tuple(s)
        if s_pad != tuple(it):
            raise LoweringError("GEMM outputs must have the product shape")
        outputs.append(OutputSpec(index=len(outputs), op_id=o, dtype=dts[o], shape=s, kind="full"))
    epi_operands = [o for o in operands if o.index not in (a_idx, b_idx)
                    or any(o.op_id in graph.ops[x].inputs for x in ops[1:])]
    values, env = build_dag(graph, ops[1:], epi_operands, N, acc_op=mm)
    sk = SubKernel(family="gemm", op_ids=list(ops), operands=operands, outputs=outputs,
                   rows=M, cols=N, values=values, out_values=[env[o] for o in outs],
                   m=M, n=N, k=K, a_operand=a_idx, b_operand=b_idx)
    sk.precise = any(o.dtype == "float32" for o in outputs)
    needed = _needed(values, sk.out_values)
    if any(values[v].avail for v in needed):
        raise LoweringError("GEMM epilogues are elementwise only")
    from .gemm_config import choose_gemm_config
    gemm_tune = dict(tune.get("gemm") or {})
    if split3:
        # the one-SM engine with 128-column tiles: its epilogue warps sum the
        # promoted accumulator chunks, one 128-column row per thread
        gemm_tune.update(pair=False, bn=128)
    sk.config = choose_gemm_config(sk, gemm_tune, batch=batch,
                                   allow_pair=prologue is None and not split3,
                                   allow_streamk=prologue is None and not split3)
    sk.config["split3"] = split3
    sk.config["b_kmajor"] = bool(b_kmajor)
    sk.config["batch"] = int(batch)
    if prologue is not None:
        sk.config["prologue"] = {"kind": "rmsnorm", "eps": prologue["eps"], "w": prologue["w"],
                                 "w_dtype": prologue["w_dtype"]}
        sk.config["threads"] = 512
        # GemmLayout<..., PRO>: ready[S], rms_full[2], rms_empty[2], 1/rms [2][BM]
        sk.config["smem_bytes"] += (sk.config["stages"] + 4) * 8 + 2 * sk.config["bm"] * 4
    sk.config["needed"] = sorted(needed)
    return sk
