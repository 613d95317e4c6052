"""The CPU oracle, pinned against the reference's own evaluation.

tests/golden/*.npz hold the reference's results (benchmarks/ops.py run on
seeded inputs, made by tests/golden/make_golden.py).  The oracle must
reproduce them: fp32 within a few ulp, and the once-rounded 16-bit outputs
bit for bit except where the fp32 value sits on a rounding boundary."""
import numpy as np
import pytest

from oracle import graph_oracle as orc
from tests._golden import CASES, assert_close, bf16_ulp_diff, graph_for, input_dtype, load


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference(case):
    meta, inputs, ref_f32, ref_out = load(case)
    g = graph_for(meta, inputs)
    res = orc.evaluate(g, inputs)
    out_id = g.ops[g._outputs[0]].inputs[0]
    got = res[("f32", out_id)]
    assert got.shape == ref_f32.shape
    err = np.abs(got.astype(np.float64) - ref_f32)
    scale = np.abs(ref_f32).astype(np.float64)
    # fp32: a few ulp of each value (plus ulps of the row scale for sums)
    assert np.all(err <= 4e-7 * scale + 1e-7 * scale.max()), f"max err {err.max()}"
    dt = meta["out_dtype"]
    assert res[("dtype", out_id)] == dt
    if dt == "bfloat16":
        ulps = bf16_ulp_diff(res[out_id], ref_out)
        assert ulps.max() <= 1
        assert np.mean(ulps > 0) < 0.01
    else:
        np.testing.assert_allclose(res[out_id], ref_out, rtol=1e-6, atol=1e-7 * scale.max())


def test_bf16_roundtrip_and_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, np.inf, -np.inf, 0.0, 3.0e38],
                 dtype=np.float32)
    bits = orc.f32_to_bf16_bits(x)
    back = orc.bf16_bits_to_f32(bits)
    # 1 + 2^-8 is a tie -> rounds to even (1.0); 1 + 1.5*2^-8 rounds up
    assert back[0] == 1.0 and back[1] == 1.0 and back[2] == np.float32(1.0078125)
    assert back[3] == -2.5 and np.isinf(back[4]) and np.isinf(back[5]) and back[6] == 0.0
    nan = orc.f32_to_bf16_bits(np.array([np.nan], dtype=np.float32))
    assert np.isnan(orc.bf16_bits_to_f32(nan))[0]


def test_causal_mask_definition():
    m = orc.causal_mask((2, 3), 3, None, 0)
    # row index is the flat row modulo the period (default: cols)
    expect = np.array([[0, -np.inf, -np.inf], [0, 0, -np.inf], [0, 0, 0]] * 2, dtype=np.float32)
    np.testing.assert_array_equal(m.reshape(6, 3), expect)
    m = orc.causal_mask((4,), 8, None, 2, row_offset=1)
    assert np.isinf(m[0, 4]) and m[0, 3] == 0


def test_oracle_row_independence():
    """Rows are independent: evaluating row blocks (with their global row
    offset for the mask) equals evaluating the whole tensor."""
    meta, inputs, ref_f32, _ = load("softmax_f32_causal")
    g = graph_for(meta, inputs)
    whole = orc.evaluate(g, inputs)
    oid = g.ops[g._outputs[0]].inputs[0]
    x = inputs["logits"]
    from molten_b200 import graphs
    parts = []
    for start, stop in ((0, 2), (2, 5), (5, 6)):
        gs = graphs.softmax((stop - start, x.shape[1]), causal=True)
        r = orc.evaluate(gs, {"logits": x[start:stop]}, row_offset=start)
        parts.append(r[("f32", gs.ops[gs._outputs[0]].inputs[0])])
    np.testing.assert_array_equal(np.concatenate(parts), whole[("f32", oid)])


def test_assert_close_catches_a_planted_error():
    meta, inputs, ref_f32, _ = load("rmsnorm_silu_bf16_r3")
    g = graph_for(meta, inputs)
    res = orc.evaluate(g, inputs)
    oid = g.ops[g._outputs[0]].inputs[0]
    good = orc.bf16_bits_to_f32(res[oid])
    assert_close(good, ref_f32, "bfloat16")
    bad = good.copy()
    i = np.unravel_index(np.argmax(np.abs(bad)), bad.shape)
    bad[i] *= 1.03             # a 3% error in one element (planted in the oracle's output)
    with pytest.raises(AssertionError):
        assert_close(bad, ref_f32, "bfloat16")
