"""The bounded-wait contract of the tcgen05 GEMM, exercised on the GPU.

Every mbarrier wait in the GEMM engine gives up after MOLTEN_WAIT_NS; the
CTA then sets a bit in the status word, stops issuing, drains its own
copies, frees its TMEM and returns, so the context stays usable.  Here a
single-tile GEMM is built with a 20 ms wait limit and the test-only switch
MOLTEN_TEST_SKIP_KSTEP, under which the TMA producer leaves one k-step of
the tile unissued: the MMA issuer's wait for that stage runs out (a barrier
that nothing completes), and so does the epilogue's wait for the
accumulator.  The test checks that the launch returns, that the status word
carries those bits, and that a normal launch of the same GEMM right after it
in the same process is correct.  No fault, trap or unbounded wait is
involved: the failure is a copy that is never issued.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from molten_b200 import graphs
from molten_b200.build import build_cubin
from molten_b200.codegen import CodeGenerator
from molten_b200.fusion import FusionEngine
from molten_b200.runtime import MoltenRuntime, _Spec
from oracle import graph_oracle as orc
from tests._golden import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

# molten::GemmStatus bits (molten/gemm_sm100.cuh)
TIMEOUT_FULL, TIMEOUT_ACC = 1, 4


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_gemm_wait_runs_out_and_the_next_launch_is_correct():
    m, k, n = 128, 256, 128                       # one 128 x 128 tile, 4 k-steps
    g = graphs.gemm_bias_gelu(m, k, n)
    kern = CodeGenerator(dtype="bfloat16", tune={"gemm": {"pair": False, "streamk": False}}) \
        .generate(g, FusionEngine().fuse(g)[0])
    (sk,) = kern.plan.kernels
    assert sk.family == "gemm" and not sk.config["pair"] and not sk.config["streamk"]
    gen = torch.Generator(device=DEV)
    gen.manual_seed(7)
    A = torch.randn(m, k, generator=gen, device=DEV).to(torch.bfloat16)
    B = (torch.randn(k, n, generator=gen, device=DEV) / k ** 0.5).to(torch.bfloat16)
    bias = (0.02 * torch.randn(n, generator=gen, device=DEV)).to(torch.bfloat16)

    MoltenRuntime.read_status(0, reset=True)      # start from a clear word
    broken = _Spec(kern, build_cubin(kern.source, kern.name + "_skipk2", extra_flags=[
        "-DMOLTEN_WAIT_NS=20000000ull", "-DMOLTEN_TEST_SKIP_KSTEP=2"]))
    broken.run([A, B, bias], None, None, 0)
    torch.cuda.synchronize()                      # the launch returned
    status = MoltenRuntime.read_status(0, reset=True)
    assert status & TIMEOUT_FULL, f"status {status:#x}: the MMA's wait should have run out"
    assert status & TIMEOUT_ACC, f"status {status:#x}: the epilogue's wait should have run out"
    assert MoltenRuntime.read_status(0) == 0      # reset cleared it

    ck = MoltenRuntime().compile(kern)
    out = ck(A, B, bias)
    torch.cuda.synchronize()
    assert MoltenRuntime.read_status(0) == 0
    res = orc.evaluate(g, {"A": _bits(A), "B": _bits(B), "bias": _bits(bias)})
    assert_close(out.float().cpu().numpy(), res[("f32", g.ops[g._outputs[0]].inputs[0])],
                 "bfloat16", "GEMM after a timed-out launch")


def test_debug_mode_raises_at_the_call(monkeypatch):
    """MOLTEN_DEBUG: the call whose bounded wait ran out raises, with the
    status bits in the message, and leaves the word clear for the next call."""
    from molten_b200 import _capi, runtime
    m, k, n = 128, 256, 128
    g = graphs.gemm_bias_gelu(m, k, n)
    kern = CodeGenerator(dtype="bfloat16", tune={"gemm": {"pair": False, "streamk": False}}) \
        .generate(g, FusionEngine().fuse(g)[0])
    A = torch.randn(m, k, device=DEV).to(torch.bfloat16)
    B = (torch.randn(k, n, device=DEV) / k ** 0.5).to(torch.bfloat16)
    bias = torch.zeros(n, device=DEV).to(torch.bfloat16)
    MoltenRuntime.read_status(0, reset=True)
    monkeypatch.setattr(runtime, "DEBUG", True)
    broken = _Spec(kern, build_cubin(kern.source, kern.name + "_skipk2", extra_flags=[
        "-DMOLTEN_WAIT_NS=20000000ull", "-DMOLTEN_TEST_SKIP_KSTEP=2"]))
    with pytest.raises(_capi.MoltenError, match="bounded wait ran out"):
        broken.run([A, B, bias], None, None, 0)
    assert MoltenRuntime.read_status(0) == 0
    out = MoltenRuntime().compile(kern)(A, B, bias)      # a good call passes the check
    assert out.shape == (m, n)
