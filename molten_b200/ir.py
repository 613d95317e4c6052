"""Dataflow IR: the graph a user builds and the fusion engine partitions.

Drop-in for the reference's ``molten/ir.py``: the same ``OpType`` members in
the same order (``molten/ir.py:20-66``), the same ``TensorShape``/``Op``
fields (``ir.py:69-103``) and the same ``DataflowGraph`` builders and analysis
methods (``ir.py:106-236``).  Additions, all optional keyword arguments or new
helpers so that reference callers are unaffected:

* ``rms_norm(..., eps=1e-6)`` records ``eps`` on the RMS op (the reference
  hard-codes 1e-6 in its kernels, ``codegen.py:286``).
* ``clamp(x, lo, hi)`` stores the bounds in ``attrs["min"]``/``attrs["max"]``
  (the reference has a CLAMP op type but no semantics for it).
* ``causal_mask(period, offset)`` adds a CONSTANT whose value is generated
  from indices: 0 where ``col <= (row mod period) + offset``, ``-inf`` above.
* small builders for the remaining unary ops (``gelu``, ``silu`` ...).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Optional


class OpType(Enum):
    # elementwise
    ADD = auto()
    SUB = auto()
    MUL = auto()
    DIV = auto()
    NEG = auto()
    SQRT = auto()
    RSQRT = auto()
    EXP = auto()
    LOG = auto()
    TANH = auto()
    SIGMOID = auto()
    GELU = auto()
    SILU = auto()
    RELU = auto()
    ABS = auto()
    CLAMP = auto()
    # row reductions
    SUM = auto()
    MEAN = auto()
    MAX = auto()
    MIN = auto()
    NORM = auto()
    RMS = auto()
    # contractions
    MATMUL = auto()
    DOT = auto()
    OUTER = auto()
    # attention primitives
    SOFTMAX = auto()
    ROTATE = auto()
    # data movement
    TRANSPOSE = auto()
    RESHAPE = auto()
    SLICE = auto()
    CONCAT = auto()
    BROADCAST = auto()
    # graph boundary
    INPUT = auto()
    OUTPUT = auto()
    CONSTANT = auto()


ELEMENTWISE_OPS = frozenset({
    OpType.ADD, OpType.SUB, OpType.MUL, OpType.DIV,
    OpType.NEG, OpType.SQRT, OpType.RSQRT, OpType.EXP,
    OpType.LOG, OpType.TANH, OpType.SIGMOID, OpType.GELU,
    OpType.SILU, OpType.RELU, OpType.ABS, OpType.CLAMP,
})

REDUCTION_OPS = frozenset({
    OpType.SUM, OpType.MEAN, OpType.MAX, OpType.MIN,
    OpType.NORM, OpType.RMS, OpType.SOFTMAX,
})

BOUNDARY_OPS = frozenset({OpType.INPUT, OpType.OUTPUT, OpType.CONSTANT})


@dataclass
class TensorShape:
    """Shape with optional symbolic (string) dimensions."""
    dims: list

    def __repr__(self):
        return "(" + ", ".join(str(d) for d in self.dims) + ")"

    @property
    def ndim(self) -> int:
        return len(self.dims)

    @property
    def is_fully_known(self) -> bool:
        return all(isinstance(d, int) for d in self.dims)


@dataclass
class Op:
    """One node of the dataflow graph."""
    id: int
    op_type: OpType
    name: str = ""
    inputs: list = field(default_factory=list)
    shape: Optional[TensorShape] = None
    dtype: str = "float16"
    attrs: dict = field(default_factory=dict)
    fusable: bool = True
    memory_bound: bool = False
    reduction_dim: Optional[int] = None

    def __repr__(self):
        return f"Op({self.id}: {self.op_type.name} '{self.name}' {self.shape})"


class DataflowGraph:
    """A DAG of ``Op`` nodes keyed by integer id (ids are insertion order)."""

    def __init__(self, name: str = "unnamed"):
        self.name = name
        self.ops: dict[int, Op] = {}
        self._next_id = 0
        self._outputs: list[int] = []

    # ------------------------------------------------------------------ build
    def add_op(self, op_type: OpType, inputs: list = None, name: str = "",
               shape: Optional[TensorShape] = None, dtype: str = "float16",
               **attrs) -> int:
        op_id = self._next_id
        self._next_id += 1
        self.ops[op_id] = Op(id=op_id, op_type=op_type, name=name,
                             inputs=list(inputs or []), shape=shape,
                             dtype=dtype, attrs=attrs)
        return op_id

    def add_input(self, name: str, shape: TensorShape,
                  dtype: str = "float16") -> int:
        return self.add_op(OpType.INPUT, name=name, shape=shape, dtype=dtype)

    def add_output(self, input_id: int, name: str = "output") -> int:
        out_id = self.add_op(OpType.OUTPUT, [input_id], name=name,
                             shape=self.ops[input_id].shape)
        self._outputs.append(out_id)
        return out_id

    def add_constant(self, name: str, value: float) -> int:
        return self.add_op(OpType.CONSTANT, name=name, value=value)

    # ------------------------------------------------------------- builders
    def add(self, a: int, b: int, name: str = "") -> int:
        return self.add_op(OpType.ADD, [a, b], name)

    def sub(self, a: int, b: int, name: str = "") -> int:
        return self.add_op(OpType.SUB, [a, b], name)

    def mul(self, a: int, b: int, name: str = "") -> int:
        return self.add_op(OpType.MUL, [a, b], name)

    def div(self, a: int, b: int, name: str = "") -> int:
        return self.add_op(OpType.DIV, [a, b], name)

    def matmul(self, a: int, b: int, name: str = "") -> int:
        return self.add_op(OpType.MATMUL, [a, b], name)

    def softmax(self, x: int, dim: int = -1, name: str = "") -> int:
        op_id = self.add_op(OpType.SOFTMAX, [x], name)
        self.ops[op_id].reduction_dim = dim
        return op_id

    def rms_norm(self, x: int, weight: int, name: str = "",
                 eps: float = 1e-6) -> int:
        """x / rms(x) * weight, expanded to RMS -> DIV -> MUL."""
        rms_id = self.add_op(OpType.RMS, [x], f"{name}_rms", eps=eps)
        div_id = self.div(x, rms_id, f"{name}_div")
        return self.mul(div_id, weight, f"{name}_scale")

    def rope(self, x: int, freqs: int, name: str = "", sin: Optional[int] = None,
             style: Optional[str] = None) -> int:
        """ROTATE: rotary position embedding of x [..., seq, heads, head_dim].

        ``rope(x, freqs)`` is the reference's builder (``ir.py:175-176``);
        its table layout is not specified there, so here ``freqs`` is
        [seq, head_dim] holding each pair's (cos, sin) interleaved.  With
        ``sin`` given, ``freqs`` is the cos table and both are
        [seq, head_dim/2] -- the form of ``benchmarks/ops.py:24-35``.
        ``style``: "interleaved" pairs (2i, 2i+1) as in ops.py (default) or
        "half" pairs (i, i + head_dim/2).  The result has x's dtype."""
        inputs = [x, freqs] + ([sin] if sin is not None else [])
        attrs = {"style": style} if style else {}
        return self.add_op(OpType.ROTATE, inputs, name, **attrs)

    def transpose(self, x: int, name: str = "") -> int:
        """TRANSPOSE of the last two dims (a matrix [N, K] -> [K, N]).  As
        a MATMUL's B operand it costs nothing: the GEMM reads the original
        rows K-major."""
        return self.add_op(OpType.TRANSPOSE, [x], name)

    def unary(self, op_type: OpType, x: int, name: str = "", **attrs) -> int:
        return self.add_op(op_type, [x], name, **attrs)

    def gelu(self, x: int, name: str = "") -> int:
        return self.unary(OpType.GELU, x, name)

    def silu(self, x: int, name: str = "") -> int:
        return self.unary(OpType.SILU, x, name)

    def sigmoid(self, x: int, name: str = "") -> int:
        return self.unary(OpType.SIGMOID, x, name)

    def relu(self, x: int, name: str = "") -> int:
        return self.unary(OpType.RELU, x, name)

    def exp(self, x: int, name: str = "") -> int:
        return self.unary(OpType.EXP, x, name)

    def clamp(self, x: int, lo: Optional[float] = None,
              hi: Optional[float] = None, name: str = "") -> int:
        return self.add_op(OpType.CLAMP, [x], name, min=lo, max=hi)

    def causal_mask(self, period: Optional[int] = None, offset: int = 0,
                    name: str = "causal_mask") -> int:
        """Index-generated additive mask: 0 on/below the diagonal, -inf above.

        Element (row, col) of the mask is ``-inf`` iff
        ``col > (row mod period) + offset``; ``period=None`` means the number
        of columns of the tensor it is added to.
        """
        return self.add_op(OpType.CONSTANT, name=name, kind="causal_mask",
                           period=period, offset=offset, value=None)

    # -------------------------------------------------------------- analysis
    def inputs(self) -> list:
        return [op for op in self.ops.values() if op.op_type == OpType.INPUT]

    def outputs(self) -> list:
        return [op for op in self.ops.values() if op.op_type == OpType.OUTPUT]

    def consumers(self, op_id: int) -> list:
        return [oid for oid, op in self.ops.items() if op_id in op.inputs]

    def producers(self, op_id: int) -> list:
        return self.ops[op_id].inputs

    def topological_order(self) -> list:
        """Depth-first post-order over op ids, visiting roots by id."""
        seen: set = set()
        order: list = []
        for root in self.ops:
            if root in seen:
                continue
            # iterative DFS so that deep chains do not hit the recursion limit
            stack = [(root, 0)]
            seen.add(root)
            while stack:
                node, i = stack[-1]
                ins = self.ops[node].inputs
                if i < len(ins):
                    stack[-1] = (node, i + 1)
                    nxt = ins[i]
                    if nxt not in seen:
                        seen.add(nxt)
                        stack.append((nxt, 0))
                else:
                    stack.pop()
                    order.append(node)
        return order

    def is_elementwise(self, op_id: int) -> bool:
        return self.ops[op_id].op_type in ELEMENTWISE_OPS

    def is_reduction(self, op_id: int) -> bool:
        return self.ops[op_id].op_type in REDUCTION_OPS

    def __repr__(self):
        lines = [f"DataflowGraph '{self.name}' ({len(self.ops)} ops):"]
        lines += [f"  {self.ops[i]}" for i in self.topological_order()]
        return "\n".join(lines)
