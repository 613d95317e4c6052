"""Data-parallel sharding of the fused path over the GPUs of one node.

Row patterns (RMSNorm, RMSNorm*SiLU, softmax, chains) are split by token
rows: rank r owns a contiguous block of rows, per-column operands (weights,
bias vectors) are replicated, and the kernel is told the block's global row
index (``row_offset``) so index-generated masks and row-broadcast operands
stay correct.  The GEMM epilogue is split by output columns: rank r owns
C[:, n0:n1] = epilogue(A @ B[:, n0:n1] + bias[n0:n1]), A replicated.
Neither split exchanges data, so there is no collective on the hot path;
one process drives one GPU (torchrun), and ``torch.distributed`` is used
only for the barrier and the max-over-ranks timing reduction.
"""

from __future__ import annotations


def row_shards(rows: int, world: int) -> list:
    """Contiguous, balanced [start, stop) row blocks, one per rank."""
    if world < 1:
        raise ValueError("world size must be >= 1")
    base, extra = divmod(rows, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def col_shards(n: int, world: int, align: int = 64) -> list:
    """[start, stop) output-column blocks, boundaries on multiples of
    ``align`` (whole GEMM tiles) when the width allows it."""
    if world < 1:
        raise ValueError("world size must be >= 1")
    units = n // align
    if units >= world and n % align == 0:
        out, start = [], 0
        base, extra = divmod(units, world)
        for r in range(world):
            u = base + (1 if r < extra else 0)
            out.append((start * align, (start + u) * align))
            start += u
        return out
    return row_shards(n, world)


def shard_rows(t, start: int, stop: int):
    """Rows [start, stop) of a tensor flattened to [rows, cols] (a view)."""
    return t.reshape(-1, t.shape[-1])[start:stop]


def run_row_sharded(compiled, inputs: list, rank: int, world: int, row_inputs: set):
    """Run a compiled row / elementwise kernel on this rank's row block.

    ``row_inputs`` are the positions of inputs that carry one row per
    output row (they are sliced); all others are replicated.
    """
    rows = None
    for i, t in enumerate(inputs):
        if i in row_inputs:
            r = t.reshape(-1, t.shape[-1]).shape[0]
            rows = r if rows is None else rows
            if r != rows:
                raise ValueError("row-sharded inputs disagree on the row count")
    start, stop = row_shards(rows, world)[rank]
    local = [shard_rows(t, start, stop) if i in row_inputs else t for i, t in enumerate(inputs)]
    return compiled(*local, row_offset=start), (start, stop)
