"""Code generator: fusion group -> hand-structured sm_100a CUDA source.

Drop-in for the reference's ``molten/codegen.py``: ``KernelConfig``
(``codegen.py:23-31``), ``GeneratedKernel`` (``codegen.py:34-47``),
``CodeGenerator(compute_capability, fp16).generate(graph, group)``
(``codegen.py:82-100``), the ``molten_fused_<ops>`` naming rule
(``codegen.py:380-387``) and ``compile_graph`` (``codegen.py:390-405``) keep
their signatures.

What it emits is new.  Each group is pattern-matched into a family:

* row patterns (RMSNorm, RMSNorm*SiLU(gate), softmax, any last-dim
  reduction followed by elementwise ops) -> register-resident row kernel;
* pure elementwise chains with broadcast operands -> vectorised chain kernel;
* MATMUL + elementwise epilogue -> tcgen05/TMEM GEMM with the epilogue
  applied on the TMEM -> register -> global path;

and a group the hardware cannot run as one kernel is split into consecutive
kernels of one module.  Sources are specialised for concrete shapes and
dtypes; symbolic dims use a stand-in size and the runtime re-specialises on
the first call with real tensors.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass, field
from typing import Optional

from .fusion import FusionEngine, FusionGroup
from .ir import DataflowGraph, Op, OpType
from .lowering import DTYPE_SIZE, GroupPlan, LoweringError, canon_dtype
from .plan import declared_shape, plan_group

ARCH = "sm_100a"


@dataclass
class KernelConfig:
    """Launch metadata.  The first seven fields are the reference's; the
    rest describe the sm_100a launch (grid policy, clusters, sub-kernels)."""
    block_size_x: int = 256
    block_size_y: int = 1
    vectorize: int = 4
    shared_mem_bytes: int = 0
    registers_per_thread: int = 32
    dtype: str = "float"
    use_half2: bool = True
    family: str = "ew"
    cluster_x: int = 1
    launches: list = field(default_factory=list)


@dataclass
class GeneratedKernel:
    name: str
    source: str
    config: KernelConfig
    num_args: int
    estimated_flops: int = 0
    estimated_memory_bytes: int = 0
    plan: Optional[GroupPlan] = None
    graph: Optional[DataflowGraph] = None
    group: Optional[FusionGroup] = None
    dtype: str = "float32"

    @property
    def arithmetic_intensity(self) -> float:
        if self.estimated_memory_bytes == 0:
            return 0.0
        return self.estimated_flops / self.estimated_memory_bytes

    @property
    def inputs(self) -> list:
        return list(self.plan.inputs) if self.plan else []


def make_name(ops: list) -> str:
    """``molten_fused_`` + the first four distinct op names, in group order."""
    parts = []
    for op in ops:
        n = op.op_type.name.lower()
        if n not in parts:
            parts.append(n)
    return "molten_fused_" + "_".join(parts[:4])


def launch_records(plan: GroupPlan, name: str) -> list:
    """Per sub-kernel launch policy (entry name, family, geometry)."""
    recs = []
    for i, sk in enumerate(plan.kernels):
        c = sk.config
        rec = {"entry": kernel_entry(name, i, len(plan.kernels)), "family": sk.family}
        if sk.family == "row" and c.get("engine") == "tma":
            rec.update(engine="tma", block=32 * (c["nc"] * c.get("tw", 1) + 1), stages=c["stages"],
                       smem=c["smem"])
        elif sk.family == "row":
            rec.update(engine="regs", block=c["block"], rpc=c["rpc"], cl=c["cl"], smem=0)
        elif sk.family == "ew":
            rec.update(block=c["block"], rpc=c["rpc"], upt=c["upt"], tiles=c["tiles"], smem=0)
        elif sk.family == "rope":
            rec.update(block=c["block"], vec=c["vec"], slots_per_row=c["spr"], smem=0)
        elif sk.family == "split3":
            rec.update(block=c["block"], vec=c["vec"], elements=c["total"], smem=0)
        elif sk.family == "causal":
            zp = c.get("zpersist", 0)
            rec.update(block=c["threads"], zero_tiles_per_row=c["zt"], zero_tile_cols=c["zcols"],
                       zero_ctas=zp, grid=sk.rows + (zp if zp else sk.rows * c["zt"]), smem=0)
        elif sk.family == "attn":
            rec.update(block=c["threads"], bm=128, bn=c["bn"], stages=c["stages"],
                       smem=c["smem_bytes"], tma_store=c["tma_store"],
                       store_cols=c["store_cols"], batch=c["batch"])
        else:
            rec.update(block=c["threads"], bm=c["bm"], bn=c["bn"], bk=c["bk"],
                       stages=c["stages"], smem=c.get("smem_bytes", 0),
                       cluster=2 if c.get("pair") else 1)
            if c.get("split3"):
                rec.update(split3=True)
            if c.get("streamk"):
                rec.update(streamk=True, grid=c["sk_ctas"],
                           work_floats=c["sk_tiles"] * c["sk_maxseg"] * c["bm"] * c["bn"],
                           tile_counters=c["sk_tiles"])
        recs.append(rec)
    return recs


def kernel_entry(name: str, i: int, n: int) -> str:
    return name if n == 1 else f"{name}_k{i}"


def estimate(plan: GroupPlan):
    """(flops, bytes) of the algorithmic work of one call."""
    flops = 0
    nbytes = 0
    for shp, dt in zip(plan.input_shapes, plan.input_dtypes):
        n = 1
        for d in shp:
            n *= d
        nbytes += n * DTYPE_SIZE[dt]
    for shp, dt in zip(plan.output_shapes, plan.output_dtypes):
        n = 1
        for d in shp:
            n *= d
        nbytes += n * DTYPE_SIZE[dt]
    for sk in plan.kernels:
        if sk.family == "gemm":
            flops += 2 * sk.m * sk.n * sk.k
        elif sk.family == "attn":
            flops += 2 * sk.config["batch"] * sk.m * sk.n * sk.k
        flops += sk.rows * sk.cols * max(1, len(sk.op_ids))
    return flops, nbytes


class CodeGenerator:
    """Emits one sm_100a CUDA module per fusion group.

    ``fp16=True`` selects fp16 I/O as in the reference; ``dtype`` (an
    addition) selects any of float32 / bfloat16 / float16 for every input
    whose dtype is not given explicitly.  ``tune`` overrides the planner's
    choices per family (``{"row": {...}, "ew": {...}, "gemm": {...}}``);
    ``tune["defines"]`` lists preprocessor definitions ("NAME" or
    "NAME=VALUE") placed at the top of the emitted module.
    """

    def __init__(self, compute_capability: int = 80, fp16: bool = False,
                 dtype: Optional[str] = None, tune: Optional[dict] = None):
        self.cc = compute_capability
        self.fp16 = fp16
        self.io_dtype = canon_dtype(dtype) if dtype else ("float16" if fp16 else "float32")
        self.dtype = "half" if self.io_dtype == "float16" else \
            ("bfloat16" if self.io_dtype == "bfloat16" else "float")
        self.tune = tune or {}

    def generate(self, graph: DataflowGraph, group: FusionGroup,
                 input_shapes: Optional[dict] = None,
                 input_dtypes: Optional[dict] = None) -> GeneratedKernel:
        ops = [graph.ops[i] for i in group.op_ids]
        name = make_name(ops)
        shapes, dtypes = self._spec(graph, group, input_shapes, input_dtypes)
        plan = plan_group(graph, group.op_ids, shapes, dtypes, name, self.tune)
        return self.generate_from_plan(plan, name, graph, group)

    def generate_from_plan(self, plan: GroupPlan, name: str, graph=None, group=None):
        from .emit import emit_ew, emit_row, emit_row_tma
        from .emit_gemm import emit_gemm, emit_split3
        from .emit_causal import emit_causal
        from .emit_rope import emit_rope
        from .emit_attn import emit_attn
        chunks = []
        ops_txt = " -> ".join(graph.ops[i].op_type.name for i in group.op_ids) if graph else ""
        chunks.append(f"// Molten auto-generated for {ARCH}: {name}")
        if ops_txt:
            chunks.append(f"// Fused ops: {ops_txt}")
        chunks.append("// input dtypes: " + json.dumps(plan.input_dtypes))
        for d in self.tune.get("defines") or ():
            if not re.fullmatch(r"[A-Za-z_][A-Za-z0-9_]*(=[A-Za-z0-9_.+\-]+)?", str(d)):
                raise LoweringError(f"tune define {d!r} is not NAME or NAME=VALUE")
            chunks.append("#define " + str(d).replace("=", " ", 1))
        smem = 0
        block_x, block_y, fam = 256, 1, "ew"
        for i, sk in enumerate(plan.kernels):
            entry = kernel_entry(name, i, len(plan.kernels))
            if sk.family == "row" and sk.config.get("engine") == "tma":
                chunks.append(emit_row_tma(sk, entry))
                smem = max(smem, sk.config["smem"])
                block_x = 32 * (sk.config["nc"] * sk.config.get("tw", 1) + 1)
            elif sk.family == "row":
                chunks.append(emit_row(sk, entry))
                c = sk.config
                smem = max(smem, 4)
                block_x = c["block"]
            elif sk.family == "ew":
                chunks.append(emit_ew(sk, entry))
                block_x = sk.config["block"]
            elif sk.family == "rope":
                chunks.append(emit_rope(sk, entry))
                block_x = sk.config["block"]
            elif sk.family == "split3":
                chunks.append(emit_split3(sk, entry))
            elif sk.family == "causal":
                chunks.append(emit_causal(sk, entry))
                smem = max(smem, 4)
                block_x = sk.config["threads"]
            elif sk.family == "attn":
                chunks.append(emit_attn(sk, entry))
                block_x, block_y = sk.config["threads"], 1
                smem = max(smem, sk.config["smem_bytes"])
            else:
                chunks.append(emit_gemm(sk, entry))
                block_x, block_y = 128, sk.config["threads"] // 128
                smem = max(smem, sk.config.get("smem_bytes", 0))
            fam = sk.family if fam != "gemm" else fam
        if any(sk.family == "gemm" for sk in plan.kernels):
            fam = "gemm"
        elif any(sk.family in ("row", "causal") for sk in plan.kernels):
            fam = "row"
        source = "\n".join(chunks)
        flops, nbytes = estimate(plan)
        cfg = KernelConfig(block_size_x=block_x, block_size_y=block_y,
                           vectorize=plan.kernels[0].config.get("vec", 8),
                           shared_mem_bytes=smem, dtype=self.dtype,
                           family=fam,
                           cluster_x=max(sk.config.get("cl", 2 if sk.config.get("pair") else 1)
                                         for sk in plan.kernels),
                           launches=launch_records(plan, name))
        return GeneratedKernel(name=name, source=source, config=cfg,
                               num_args=len(plan.inputs) + len(plan.outputs) + 1,
                               estimated_flops=flops, estimated_memory_bytes=nbytes,
                               plan=plan, graph=graph, group=group,
                               dtype=plan.output_dtypes[0] if plan.output_dtypes else self.io_dtype)

    def _spec(self, graph, group, input_shapes, input_dtypes):
        from .lowering import group_boundary
        ext, _, _ = group_boundary(graph, group.op_ids)
        declared = declared_graph_shapes(graph)
        shapes, dtypes = {}, {}
        for i in ext:
            op = graph.ops[i]
            if op.op_type == OpType.CONSTANT:
                continue
            if input_shapes and i in input_shapes:
                shapes[i] = tuple(input_shapes[i])
            elif i in declared:
                shapes[i] = declared[i]
            else:
                raise LoweringError(f"cannot infer the shape of op {i} ({op.op_type.name})")
            dtypes[i] = input_dtypes[i] if input_dtypes and i in input_dtypes else self.io_dtype
        return shapes, dtypes


def declared_graph_shapes(graph: DataflowGraph) -> dict:
    """Shapes of every op from the declared INPUT shapes (symbolic dims get a
    stand-in size); ops whose shape cannot be inferred are left out."""
    from .lowering import infer_shapes
    symbols: dict = {}
    shapes = {}
    for oid in graph.topological_order():
        op = graph.ops[oid]
        if op.op_type == OpType.INPUT:
            shapes[oid] = declared_shape(op, symbols)
        elif op.op_type == OpType.CONSTANT:
            shapes[oid] = ()
        elif op.op_type == OpType.OUTPUT:
            continue
        elif all(i in shapes for i in op.inputs):
            try:
                shapes.update(infer_shapes(graph, [oid], {i: shapes[i] for i in op.inputs}))
            except LoweringError:
                pass
    return shapes


def compile_graph(graph: DataflowGraph, compute_capability: int = 80,
                  fp16: bool = False, dtype: Optional[str] = None) -> list:
    """Fuse the graph and emit one GeneratedKernel per fusion group."""
    groups = FusionEngine().fuse(graph)
    gen = CodeGenerator(compute_capability, fp16=fp16, dtype=dtype)
    return [gen.generate(graph, g) for g in groups]
