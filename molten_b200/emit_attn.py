"""CUDA emission for the fused attention-score sub-kernel.

softmax(Q @ K^T * scale) over the last dim (``benchmarks/ops.py:55-59``)
as one kernel: the module instantiates the engine of
``molten/attn_sm100.cuh`` with the tile shape, the input and output types,
the store path and C2 = scale * log2(e) as compile-time constants.
"""

from __future__ import annotations

import math

from .emit import c_float
from .lowering import DTYPE_CTYPE, SubKernel


def emit_attn(sk: SubKernel, name: str) -> str:
    c = sk.config
    q = sk.operands[0]
    f16in = "true" if q.dtype == "float16" else "false"
    ot = DTYPE_CTYPE[sk.outputs[0].dtype]
    c2 = c["scale"] * math.log2(math.e)
    L = []
    w = L.append
    w(f"// Molten sm_100a fused attention scores: {name}")
    w(f"// P[{c['batch']} x {sk.m}, {sk.n}] = softmax(Q K^T * {c['scale']!r}), d = {sk.k}; "
      f"column block {c['bn']}, {c['stages']} stages, "
      f"{'TMA' if c['tma_store'] else 'direct'} stores")
    w("#include \"molten/attn_sm100.cuh\"")
    w("")
    w("using namespace molten;")
    w("")
    w(f"typedef AttnLayout<{c['bn']}, {c['dch']}, {c['stages']}, {c['epi_warps']}, {c['groups']}> "
      f"Layout_{name};")
    w(f"static_assert(Layout_{name}::SMEM_BYTES <= {c['smem_bytes']}, "
      f"\"the launch's dynamic shared memory holds the layout\");")
    w(f"static_assert(Layout_{name}::THREADS == {c['threads']}, \"block size\");")
    w("")
    w(f"extern \"C\" __global__ void __launch_bounds__({c['threads']}, 1) "
      f"{name}(const __grid_constant__ AttnArgs args) {{")
    w("  extern __shared__ __align__(1024) uint8_t smem_raw[];")
    w(f"  const AttnShared sh = attn_carve<Layout_{name}>(smem_raw);")
    w(f"  attn_init<Layout_{name}>(sh, args);     // mbarriers + TMEM allocation")
    w("  pdl_enter();                            // no global access before this")
    w("  __syncthreads();")
    w(f"  attn_roles<Layout_{name}, {f16in}, {ot}, {'true' if c['tma_store'] else 'false'}, "
      f"{'true' if c['rows_aligned'] else 'false'}, {c['poly'][0]}, {c['poly'][1]}, "
      f"{'true' if c['sum16'] else 'false'}, {'true' if c['x2'] else 'false'}>"
      f"(sh, args, {c_float(c2)});")
    w("  __syncthreads();")
    w(f"  attn_teardown<Layout_{name}>(sh);       // TMEM release")
    w("}")
    return "\n".join(L) + "\n"
