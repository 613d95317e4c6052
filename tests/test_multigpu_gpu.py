"""Row- and column-sharded launches on two GPUs, one process per GPU.

Each process runs its shard through the C ABI on its own device (rows with
their global row offset, or a column block of B for the GEMM); the shards,
copied to the host, must equal a single-GPU launch over the whole input bit
for bit.  No collective is involved: the shards are independent."""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _np(t):
    """Host copy that survives the worker's exit (plain numpy, pickled by value)."""
    t = t.detach().cpu()
    return t.view(torch.int16).numpy().copy() if t.dtype == torch.bfloat16 else t.numpy().copy()


def _rows_worker(rank, world, q):
    from molten_b200 import graphs, workloads
    from molten_b200.codegen import compile_graph
    from molten_b200.runtime import MoltenRuntime
    from molten_b200.shard import row_shards
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    w = workloads.scaled(workloads.WORKLOADS["rmsnorm_silu_bf16_8192x3584"], rows=1000)
    xs = workloads.make_inputs(w, seed=11, device="cpu")
    start, stop = row_shards(1000, world)[rank]
    local = [xs[0][start:stop].to(dev), xs[1].to(dev), xs[2][start:stop].to(dev)]
    g = graphs.rmsnorm_silu_gate(stop - start, 3584)
    ck = MoltenRuntime().compile(compile_graph(g, dtype="bfloat16")[0])
    out = ck(*local, row_offset=start)
    sm = 3 * torch.randn(96, 256, generator=torch.Generator().manual_seed(3))
    s0, s1 = row_shards(96, world)[rank]
    gs = graphs.softmax((s1 - s0, 256), causal=True)
    cks = MoltenRuntime().compile(compile_graph(gs)[0])
    sout = cks(sm[s0:s1].to(dev), row_offset=s0)
    torch.cuda.synchronize()
    q.put((rank, start, _np(out), s0, _np(sout)))


def _gemm_worker(rank, world, q):
    from molten_b200 import graphs
    from molten_b200.codegen import compile_graph
    from molten_b200.runtime import MoltenRuntime
    from molten_b200.shard import col_shards
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    gen = torch.Generator().manual_seed(5)
    A = torch.randn(1100, 256, generator=gen).to(torch.bfloat16)
    B = (torch.randn(256, 1024, generator=gen) / 16).to(torch.bfloat16)
    bias = (0.02 * torch.randn(1024, generator=gen)).to(torch.bfloat16)
    n0, n1 = col_shards(1024, world)[rank]
    g = graphs.gemm_bias_gelu(1100, 256, n1 - n0)
    (kern,) = compile_graph(g, dtype="bfloat16")
    assert kern.plan.kernels[0].config["pair"]          # SM-pair clusters on every rank
    ck = MoltenRuntime().compile(kern)
    out = ck(A.to(dev), B[:, n0:n1].contiguous().to(dev), bias[n0:n1].contiguous().to(dev))
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(rank) == 0
    q.put((rank, n0, _np(out)))


def _run(target, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    return sorted(got, key=lambda t: t[0])


@pytest.fixture(scope="module")
def world():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    return 2


def test_row_shards_on_two_gpus_match_one_launch(world):
    from molten_b200 import graphs, workloads
    from molten_b200.codegen import compile_graph
    from molten_b200.runtime import MoltenRuntime
    parts = _run(_rows_worker, world)
    w = workloads.scaled(workloads.WORKLOADS["rmsnorm_silu_bf16_8192x3584"], rows=1000)
    xs = [t.to("cuda:0") for t in workloads.make_inputs(w, seed=11, device="cpu")]
    rt = MoltenRuntime()
    whole = rt.compile(compile_graph(graphs.rmsnorm_silu_gate(1000, 3584), dtype="bfloat16")[0])(*xs)
    sm = 3 * torch.randn(96, 256, generator=torch.Generator().manual_seed(3))
    swhole = rt.compile(compile_graph(graphs.softmax((96, 256), causal=True))[0])(sm.to("cuda:0"))
    torch.cuda.synchronize()
    import numpy as np
    assert np.array_equal(np.concatenate([p[2] for p in parts]), _np(whole))
    assert np.array_equal(np.concatenate([p[4] for p in parts]), _np(swhole))


def test_gemm_column_shards_on_two_gpus_match_one_launch(world):
    from molten_b200 import graphs
    from molten_b200.codegen import compile_graph
    from molten_b200.runtime import MoltenRuntime
    parts = _run(_gemm_worker, world)
    gen = torch.Generator().manual_seed(5)
    A = torch.randn(1100, 256, generator=gen).to(torch.bfloat16)
    B = (torch.randn(256, 1024, generator=gen) / 16).to(torch.bfloat16)
    bias = (0.02 * torch.randn(1024, generator=gen)).to(torch.bfloat16)
    ck = MoltenRuntime().compile(compile_graph(graphs.gemm_bias_gelu(1100, 256, 1024),
                                               dtype="bfloat16")[0])
    whole = ck(A.cuda(), B.cuda(), bias.cuda())
    torch.cuda.synchronize()
    import numpy as np
    assert np.array_equal(np.concatenate([p[2] for p in parts], axis=1), _np(whole))
