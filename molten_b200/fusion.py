"""Fusion engine: partitions a DataflowGraph into groups, one kernel each.

Behaviour is kept identical to the reference's ``molten/fusion.py`` because it
decides which pattern the code generator sees:

* the six rules of ``FusionGroup.can_add`` (``fusion.py:38-69``):
  1. elementwise after elementwise fuses, 2. elementwise after a reduction
  fuses, 3. a reduction joins a group without one, 4. two reductions share a
  group only when their ``reduction_dim`` is equal (and not None),
  5. a matmul joins a group that has no matmul (epilogue fusion),
  6. never two matmuls in one group; anything else is allowed;
* the greedy pass of ``FusionEngine.fuse`` (``fusion.py:83-138``): walk the
  topological order, skip INPUT/OUTPUT/CONSTANT, join the largest producer
  group that accepts the op (first one wins ties), else open a new group;
* ``_merge_small_groups`` (``fusion.py:140-158``): a one-op, matmul-free group
  is appended to the previous kept group when that group accepts its op.  This
  can place an op before its producer in ``op_ids``; consumers that need an
  execution order re-sort the ids topologically.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from .ir import BOUNDARY_OPS, DataflowGraph, Op, OpType


@dataclass
class FusionGroup:
    """Ops that become a single kernel."""
    group_id: int
    op_ids: list = field(default_factory=list)
    has_matmul: bool = False
    has_reduction: bool = False
    reduction_dim: Optional[int] = None

    @property
    def size(self) -> int:
        return len(self.op_ids)

    def can_add(self, op: Op, graph: DataflowGraph) -> bool:
        elementwise = graph.is_elementwise(op.id)
        reduction = graph.is_reduction(op.id)
        if op.op_type == OpType.MATMUL:
            return not self.has_matmul                       # rules 5 and 6
        if elementwise:
            return True                                      # rules 1 and 2
        if reduction and self.has_reduction:                 # rule 4
            return (op.reduction_dim is not None
                    and op.reduction_dim == self.reduction_dim)
        return True                                          # rule 3 / default

    def _absorb(self, op: Op, graph: DataflowGraph) -> None:
        self.op_ids.append(op.id)
        if graph.is_reduction(op.id):
            self.has_reduction = True
            self.reduction_dim = op.reduction_dim
        if op.op_type == OpType.MATMUL:
            self.has_matmul = True


class FusionEngine:
    """Greedy partitioner; group ids keep counting across ``fuse`` calls."""

    def __init__(self):
        self._group_counter = 0

    def fuse(self, graph: DataflowGraph) -> list:
        owner: dict = {}          # op id -> group id
        groups: dict = {}         # group id -> FusionGroup (insertion order)
        for op_id in graph.topological_order():
            op = graph.ops[op_id]
            if op.op_type in BOUNDARY_OPS:
                continue
            target = None
            for producer in op.inputs:
                gid = owner.get(producer)
                if gid is None:
                    continue
                cand = groups[gid]
                if cand.can_add(op, graph) and (target is None or cand.size > target.size):
                    target = cand
            if target is None:
                target = FusionGroup(group_id=self._group_counter)
                self._group_counter += 1
                groups[target.group_id] = target
            target._absorb(op, graph)
            owner[op_id] = target.group_id
        return self._merge_small_groups(list(groups.values()), graph)

    def _merge_small_groups(self, groups: list, graph: DataflowGraph) -> list:
        if len(groups) <= 1:
            return groups
        kept = [groups[0]]
        for grp in groups[1:]:
            last = kept[-1]
            if grp.size == 1 and not grp.has_matmul:
                op = graph.ops[grp.op_ids[0]]
                if last.can_add(op, graph):
                    last.op_ids.extend(grp.op_ids)
                    # the reference sets only the flag here, not the dim
                    last.has_reduction = last.has_reduction or grp.has_reduction
                    continue
            kept.append(grp)
        return kept

    def report(self, graph: DataflowGraph, groups: list) -> str:
        lines = [f"Fusion Report for '{graph.name}':",
                 f"  Total ops: {len(graph.ops)}",
                 f"  Fusion groups (kernels): {len(groups)}",
                 f"  Fusion ratio: {len(graph.ops) / max(len(groups), 1):.1f}x",
                 ""]
        for grp in groups:
            names = " → ".join(graph.ops[i].op_type.name for i in grp.op_ids)
            kind = "matmul" if grp.has_matmul else "elementwise"
            if grp.has_reduction:
                kind += "+reduction"
            lines.append(f"  Kernel {grp.group_id}: [{names}] ({kind})")
        return "\n".join(lines)
