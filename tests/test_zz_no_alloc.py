"""The allocation-free entry point, molten_scores_softmax_bf16_noalloc.

Some callers cannot allocate device memory while they run: a stream that is
being captured into a CUDA graph (an allocation would break the capture), a
host whose device heap belongs to another framework's allocator, a loop that
must not allocate after start-up.  For them the library offers one entry
point that keeps its fp32 intermediate (the Q @ K scores between the GEMM and
the row softmax) in a fixed device array instead of asking for memory.

Checked here through the C ABI: two calls in a row match the oracle (the CPU
restatement of the reference's softmax(matmul) semantics) and the regular
path -- the generated GEMM + row-softmax kernels launched with molten_launch,
whose intermediate comes from the caller's allocator -- within the bf16
parity bar of the other GPU tests; no bounded wait ran out (the status bits
molten_read_status reports); and a call larger than the array is refused
before anything is launched.  This file runs last so that a failure here
cannot hide the results of the other tests.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from molten_b200 import _capi
from molten_b200.codegen import compile_graph
from molten_b200.ir import DataflowGraph, TensorShape
from molten_b200.runtime import MoltenRuntime
from oracle import graph_oracle as orc
from tests._golden import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def scores_graph(m, kd, n):
    g = DataflowGraph("scores")
    q = g.add_input("q", TensorShape([m, kd]), dtype="bfloat16")
    k = g.add_input("k", TensorShape([kd, n]), dtype="bfloat16")
    g.add_output(g.softmax(g.matmul(q, k)))
    return g


def test_noalloc_scores_match_the_regular_path():
    lib = _capi.load_library()
    rt = MoltenRuntime()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    for m, kd, n, seed in [(256, 128, 512, 1), (300, 64, 1024, 2)]:
        gen = torch.Generator(device=DEV)
        gen.manual_seed(seed)
        q = torch.randn(m, kd, generator=gen, device=DEV).to(torch.bfloat16)
        k = (torch.randn(kd, n, generator=gen, device=DEV) / kd ** 0.5).to(torch.bfloat16)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
        rc = lib.molten_scores_softmax_bf16_noalloc(
            ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
            ctypes.c_void_p(out.data_ptr()), m, n, kd, ctypes.c_void_p(stream))
        assert rc == 0, _capi.last_error()
        g = scores_graph(m, kd, n)
        ck = rt.compile(compile_graph(g, dtype="bfloat16")[0])
        ref = ck(q, k)
        torch.cuda.synchronize()
        assert MoltenRuntime.read_status(0) == 0, "a bounded wait ran out"
        got = out.float().cpu().numpy()
        assert_close(got, ref.float().cpu().numpy(), "bfloat16",
                     f"no-alloc scores {m}x{kd}x{n} vs the regular path")
        bits = {nm: t.cpu().view(torch.int16).numpy().view(np.uint16) for nm, t in (("q", q), ("k", k))}
        res = orc.evaluate(g, bits)
        assert_close(got, res[("f32", g.ops[g._outputs[0]].inputs[0])], "bfloat16",
                     f"no-alloc scores {m}x{kd}x{n} vs the oracle")


def test_noalloc_scores_refuse_sizes_beyond_the_array():
    lib = _capi.load_library()
    q = torch.empty(4096, 64, dtype=torch.bfloat16, device=DEV)
    k = torch.empty(64, 4096, dtype=torch.bfloat16, device=DEV)
    out = torch.empty(4096, 4096, dtype=torch.bfloat16, device=DEV)
    rc = lib.molten_scores_softmax_bf16_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), 4096, 4096, 64, None)
    assert rc == 1 and "exceeds the allocation-free limit" in _capi.last_error()
