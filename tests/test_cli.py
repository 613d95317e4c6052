"""The command line (``molten compile | benchmark | info``, reference
``molten/cli.py:19-120``): the reference's graph-JSON schema, --fp16 (a
TypeError in the reference), --dtype, --build, and the JSON round trip."""
import json

import pytest

from molten_b200 import cli, graphs
from molten_b200.ir import OpType

# the reference's schema: ops by position, no shapes or dtypes
RMSNORM_JSON = {
    "name": "rmsnorm",
    "ops": [
        {"type": "INPUT", "name": "x"},
        {"type": "INPUT", "name": "w"},
        {"type": "RMS", "inputs": [0], "name": "rms"},
        {"type": "DIV", "inputs": [0, 2], "name": "normed"},
        {"type": "MUL", "inputs": [3, 1], "name": "out"},
        {"type": "OUTPUT", "inputs": [4], "name": "y"},
    ],
}


def _write(tmp_path, data, name="g.json"):
    p = tmp_path / name
    p.write_text(json.dumps(data))
    return p


def test_graph_from_reference_json():
    g = cli.graph_from_json(RMSNORM_JSON)
    assert [g.ops[i].op_type for i in sorted(g.ops)] == [
        OpType.INPUT, OpType.INPUT, OpType.RMS, OpType.DIV, OpType.MUL, OpType.OUTPUT]
    assert g._outputs == [5] and g.ops[3].inputs == [0, 2]


def test_bad_json_is_rejected():
    with pytest.raises(ValueError):
        cli.graph_from_json({"ops": [{"type": "NOPE"}]})
    with pytest.raises(ValueError):
        cli.graph_from_json({"ops": [{"type": "RMS", "inputs": [3]}]})


def test_compile_fp16_writes_kernels(tmp_path, capsys):
    out = tmp_path / "out"
    assert cli.main(["compile", str(_write(tmp_path, RMSNORM_JSON)), "-o", str(out), "--fp16"]) == 0
    cus = list(out.glob("molten_fused_*.cu"))
    assert len(cus) == 1
    src = cus[0].read_text()
    assert "const f16*" in src and "f16* __restrict__ out0" in src
    assert (out / "molten_generated.h").exists() and (out / "molten" / "row_engine.cuh").exists()
    assert "Generated 1 kernel(s)" in capsys.readouterr().out


def test_compile_with_shapes_attrs_and_build(tmp_path):
    g = graphs.softmax((64, 2048), dtype="bfloat16", causal=True)
    data = cli.graph_to_json(g)
    assert cli.graph_to_json(cli.graph_from_json(data)) == data
    out = tmp_path / "out"
    rc = cli.main(["compile", str(_write(tmp_path, data)), "-o", str(out),
                   "--dtype", "bfloat16", "--build"])
    assert rc == 0
    cubins = list(out.glob("molten_fused_*.cubin"))
    assert len(cubins) == 1 and cubins[0].stat().st_size > 1000
    src = next(out.glob("molten_fused_*.cu")).read_text()
    assert "constexpr long long COLS = 2048LL" in src and "mlim" in src


def test_missing_graph_file(tmp_path, capsys):
    assert cli.main(["compile", str(tmp_path / "nope.json")]) == 1
    assert "not found" in capsys.readouterr().out


def test_benchmark_generates_and_info(tmp_path, capsys):
    assert cli.main(["benchmark", "--dim", "1024", "--seq", "16", "-o", str(tmp_path)]) == 0
    assert "molten_fused_rms_div_mul" in capsys.readouterr().out
    assert cli.main(["info"]) == 0
    assert "sm_100a" in capsys.readouterr().out
