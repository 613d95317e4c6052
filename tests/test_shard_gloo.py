"""Multi-process sharding on CPU (gloo, world size 2).

Row patterns are split by contiguous row blocks with the block's global row
offset; the GEMM epilogue by output-column blocks.  Each rank evaluates its
shard with the CPU oracle through the product's host-side helpers
(molten_b200.shard); rank 0 gathers the shards and checks them against the
whole-tensor evaluation bit for bit (rows and columns are independent)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from molten_b200 import graphs
from molten_b200.shard import col_shards, row_shards, run_row_sharded
from oracle import graph_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _out(g):
    return g.ops[g._outputs[0]].inputs[0]


def _worker(rank, world, port, results):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        rng = np.random.default_rng(0)
        # causal softmax, 9 rows: the mask depends on the global row index
        x = (3 * rng.standard_normal((9, 64))).astype(np.float32)

        def oracle_kernel(xs, row_offset=0):
            g = graphs.softmax(tuple(xs.shape), causal=True)
            return orc.evaluate(g, {"logits": xs.numpy()}, row_offset=row_offset)[("f32", _out(g))]

        part, (start, stop) = run_row_sharded(oracle_kernel, [torch.from_numpy(x)], rank, world, {0})
        parts = [None] * world
        dist.all_gather_object(parts, (start, stop, part))
        # GEMM + bias + GELU, output columns split on 64-column tiles
        A = rng.standard_normal((16, 32)).astype(np.float32)
        B = (rng.standard_normal((32, 256)) / 6).astype(np.float32)
        bias = (0.02 * rng.standard_normal(256)).astype(np.float32)
        n0, n1 = col_shards(256, world)[rank]
        gs = graphs.gemm_bias_gelu(16, 32, n1 - n0, dtype="float32")
        cpart = orc.evaluate(gs, {"A": A, "B": np.ascontiguousarray(B[:, n0:n1]),
                                  "bias": bias[n0:n1]})[("f32", _out(gs))]
        cparts = [None] * world
        dist.all_gather_object(cparts, (n0, n1, cpart))
        if rank == 0:
            g = graphs.softmax((9, 64), causal=True)
            whole = orc.evaluate(g, {"logits": x})[("f32", _out(g))]
            rows = np.concatenate([p for _, _, p in sorted(parts, key=lambda t: t[0])])
            gw = graphs.gemm_bias_gelu(16, 32, 256, dtype="float32")
            cw = orc.evaluate(gw, {"A": A, "B": B, "bias": bias})[("f32", _out(gw))]
            cols = np.concatenate([p for _, _, p in sorted(cparts, key=lambda t: t[0])], axis=1)
            results.put((bool(np.array_equal(rows, whole)), bool(np.array_equal(cols, cw)),
                         [(a, b) for a, b, _ in parts], [(a, b) for a, b, _ in cparts]))
    finally:
        dist.destroy_process_group()


def test_row_and_column_shards_reassemble_on_two_ranks():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    rows_ok, cols_ok, row_blocks, col_blocks = results.get(timeout=10)
    assert rows_ok and cols_ok
    assert sorted(row_blocks) == [(0, 5), (5, 9)]
    assert sorted(col_blocks) == [(0, 128), (128, 256)]


def test_shard_helpers():
    assert row_shards(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert row_shards(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    assert col_shards(14336, 8) == [(i * 1792, (i + 1) * 1792) for i in range(8)]
    assert col_shards(100, 3, align=64) == row_shards(100, 3)
    with pytest.raises(ValueError):
        row_shards(4, 0)
