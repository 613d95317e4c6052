"""The reference's own hand-written CUDA kernels, run on the same B200.

benchmarks/reference_kernels.cu is the only GPU code the reference ships for
this path: fused RMSNorm (:12-50) and fused RMSNorm*SiLU*gate (:104-144),
fp32 only, one 256-thread CTA per row, launched on the default stream.
oracle/build_ref.py compiles it for sm_100a into oracle/_ref/ (in the build
container, where the reference checkout is; the library travels with the
repository).  Here, on the same seeded inputs:

* the reference's kernels match the oracle (fp32 bar): a second pin of the
  oracle, by the reference's own GPU code;
* both the reference's kernels and this library's are timed with CUDA
  events over 50 calls queued back to back on the GPU, inputs and outputs
  rotated over more than 2x L2, and the table is printed (run with -s).
"""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from molten_b200 import graphs
from molten_b200.codegen import compile_graph
from molten_b200.runtime import MoltenRuntime
from oracle import build_ref
from oracle import graph_oracle as orc
from tests._golden import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
L2_BYTES = 126 * 1024 * 1024

# (kind, rows, cols): the benchmark's fp32 RMSNorm, the RMSNorm*SiLU rows at
# hidden 3584 in fp32 (the reference kernels take fp32 only), and the
# paper's decode / prefill / long shapes at hidden 5120
CONFIGS = [
    ("rmsnorm", 2048, 5120),
    ("rmsnorm", 1, 5120),
    ("rmsnorm", 8192, 5120),
    ("rmsnorm_silu_gate", 1, 3584),
    ("rmsnorm_silu_gate", 2048, 3584),
    ("rmsnorm_silu_gate", 8192, 3584),
    ("rmsnorm_silu_gate", 2048, 5120),
]


@pytest.fixture(scope="module")
def ref():
    mod = build_ref.load_library()
    if mod is None:
        pytest.skip("oracle/_ref has no build of the reference's kernels")
    return mod


def _inputs(kind, rows, cols, seed):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    x = torch.randn(rows, cols, generator=gen, device=DEV)
    w = 1 + 0.1 * torch.randn(cols, generator=gen, device=DEV)
    if kind == "rmsnorm":
        return [x, w]
    return [x, w, torch.randn(rows, cols, generator=gen, device=DEV)]


def _ref_call(ref, kind, xs):
    if kind == "rmsnorm":
        return ref.fused_rmsnorm(xs[0], xs[1], 1e-6)
    return ref.fused_rmsnorm_silu_gate(xs[0], xs[1], xs[2], 1e-6)


def _time(fn, sets, reps=50):
    """Mean device µs per call over `reps` calls rotating over `sets`.

    The calls are queued behind a GPU sleep long enough for the host to
    enqueue all of them, so the events time the kernels back to back and
    not the host's per-call cost (the reference's kernels launch on the
    legacy default stream, which a CUDA graph capture would reject)."""
    for i in range(5):
        fn(i % len(sets))
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(40_000_000)          # ~20 ms at the B200's clocks
    a.record()
    for i in range(reps):
        fn(i % len(sets))
    b.record()
    torch.cuda.synchronize()
    return 1e3 * a.elapsed_time(b) / reps


@pytest.mark.parametrize("kind,rows,cols", CONFIGS)
def test_reference_kernels_match_the_oracle_and_are_timed(ref, kind, rows, cols):
    g = graphs.rmsnorm(rows, cols) if kind == "rmsnorm" else \
        graphs.rmsnorm_silu_gate(rows, cols, dtype="float32")
    xs = _inputs(kind, rows, cols, seed=rows + cols)
    theirs = _ref_call(ref, kind, xs)
    ck = MoltenRuntime().compile(compile_graph(g, dtype="float32")[0])
    ours = ck(*xs)
    torch.cuda.synchronize()
    pick = np.unique(np.concatenate([[0, rows - 1], np.random.default_rng(0).integers(0, rows, 32)]))
    sub = [t[torch.as_tensor(pick, device=DEV)].cpu().numpy() if t.dim() == 2 else t.cpu().numpy()
           for t in xs]
    sg = graphs.rmsnorm(len(pick), cols) if kind == "rmsnorm" else \
        graphs.rmsnorm_silu_gate(len(pick), cols, dtype="float32")
    names = ["x", "w"] if kind == "rmsnorm" else ["x", "w", "gate"]
    res = orc.evaluate(sg, dict(zip(names, sub)))[("f32", sg.ops[sg._outputs[0]].inputs[0])]
    idx = torch.as_tensor(pick, device=DEV)
    assert_close(theirs[idx].cpu().numpy(), res, "float32", f"reference kernel {kind} {rows}x{cols}")
    assert_close(ours[idx].cpu().numpy(), res, "float32", f"molten {kind} {rows}x{cols}")

    io = sum(t.numel() * 4 for t in xs) + rows * cols * 4
    nsets = max(1, min(64, -(-2 * L2_BYTES // io)))
    sets = [xs] + [[t.clone() for t in xs] for _ in range(nsets - 1)]
    outs = [torch.empty_like(ours) for _ in sets]
    t_ref = _time(lambda i: _ref_call(ref, kind, sets[i]), sets)
    t_ours = _time(lambda i: ck(*sets[i], out=outs[i]), sets)
    assert MoltenRuntime.read_status(0) == 0
    line = {"kernel": kind, "rows": rows, "cols": cols, "dtype": "f32", "bytes": io,
            "reference_us": round(t_ref, 2), "molten_us": round(t_ours, 2),
            "speedup": round(t_ref / t_ours, 2),
            "reference_gbs": round(io / t_ref / 1e3, 1), "molten_gbs": round(io / t_ours / 1e3, 1),
            "sets": nsets, "timing": "50 calls queued behind a GPU sleep, CUDA events"}
    print("reference-vs-molten " + json.dumps(line))
    path = os.environ.get("MOLTEN_REFERENCE_TIMING")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(line) + "\n")
