"""CUDA emission for the split causal row softmax.

softmax(x + causal_mask) over long rows (``benchmarks/ops.py:45-47`` with
the additive mask of ``DataflowGraph.causal_mask``) as one kernel of row
CTAs for the visible logits and zero-tile CTAs for the masked rest: the
module instantiates ``molten/causal_softmax.cuh`` with the element type,
the row length, the mask's period and offset and the zero-tile geometry as
compile-time constants.
"""

from __future__ import annotations

from .lowering import DTYPE_CTYPE, SubKernel


def emit_causal(sk: SubKernel, name: str) -> str:
    c = sk.config
    ct = DTYPE_CTYPE[sk.operands[0].dtype]
    precise = "true" if c["precise"] else "false"
    L = []
    w = L.append
    w(f"// Molten sm_100a causal softmax: {name}")
    w(f"// out[{sk.rows}, {sk.cols}] = softmax(x + mask), mask -inf for col > "
      f"(row mod {c['period']}) + {c['offset']}; " +
      (f"{c['zt']} zero tiles of {c['zcols']} columns per row" if c["zt"] else
       "each row CTA stores its own zeros"))
    w("#include \"molten/causal_softmax.cuh\"")
    w("")
    w("using namespace molten;")
    w("")
    w(f"extern \"C\" __global__ void __launch_bounds__({c['threads']}) "
      f"{name}(const __grid_constant__ RowArgs args) {{")
    w("  pdl_enter();")
    w(f"  causal_softmax_cta<{ct}, {c['threads']}, {sk.cols}LL, {c['period']}LL, {c['offset']}LL, "
      f"{c['zt']}, {c['zcols']}LL, {precise}, {'true' if c.get('interleave') else 'false'}, "
      f"{'true' if c.get('w32') else 'false'}, {int(c.get('zpersist', 0))}>(args);")
    w("}")
    return "\n".join(L) + "\n"
