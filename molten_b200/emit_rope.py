"""CUDA C++ emission for the RoPE (ROTATE) sub-kernel.

Semantics of ``benchmarks/ops.py:24-35``: x [..., seq, heads, head_dim]
viewed as rows of head_dim elements; row r sits at position
p = ((row_offset + r) / heads) % seq; each pair (x0, x1) becomes
(x0 cos - x1 sin, x0 sin + x1 cos) with cos, sin = table[p, pair].

Pairs are (2i, 2i+1) ("interleaved", as in ops.py) or (i, i + head_dim/2)
("half").  Tables are cos and sin [seq, head_dim/2], or one packed
[seq, head_dim] table of (cos, sin) per pair.  fp32 arithmetic, one
rounding to x's dtype.

One thread handles one 16-byte slot of x per grid-stride step (VEC
elements, VEC/2 pairs; with "half" the slot and its partner slot in the
second half, VEC pairs): one vector load of x (two for "half"), vector
loads of the pair's table entries (cached: every head of a position reads
the same table row), one (two) vector store(s).  ``scalar`` kernels, for
pointers that are not 16-byte aligned, move single elements.
"""

from __future__ import annotations

from .lowering import DTYPE_CTYPE, SubKernel


def emit_rope(sk: SubKernel, name: str) -> str:
    c = sk.config
    VEC, SCALAR, STYLE, PACKED = c["vec"], c["scalar"], c["style"], c["packed"]
    D, SEQ, HEADS, SPR = sk.cols, c["seq"], c["heads"], c["spr"]
    XT = DTYPE_CTYPE[sk.operands[0].dtype]
    T1 = DTYPE_CTYPE[sk.operands[1].dtype]
    T2 = DTYPE_CTYPE[sk.operands[2].dtype] if not PACKED else T1
    OT = DTYPE_CTYPE[sk.outputs[0].dtype]
    half = STYLE == "half"
    L = []
    w = L.append
    w(f"// Molten sm_100a RoPE kernel: {name}")
    w(f"// x [.., {SEQ}, {HEADS}, {D}] {sk.operands[0].dtype}; "
      f"{'packed (cos, sin) table' if PACKED else 'cos/sin tables'} "
      f"{sk.operands[1].dtype}; {STYLE} pairs")
    w("#include \"molten/row_engine.cuh\"")
    w("")
    w("using namespace molten;")
    w("")
    minb = c.get("min_blocks", 0)
    lb = f"{c['block']}, {minb}" if minb else f"{c['block']}"
    w(f"extern \"C\" __global__ void __launch_bounds__({lb}) "
      f"{name}(const __grid_constant__ RowArgs args) {{")
    w("  pdl_enter();")
    w(f"  constexpr int VEC = {VEC}, SPR = {SPR};")
    w(f"  constexpr long long D = {D}LL, SEQ = {SEQ}LL, HEADS = {HEADS}LL;")
    w(f"  const {XT}* __restrict__ x = static_cast<const {XT}*>(args.in[0]);")
    w(f"  const {T1}* __restrict__ t1 = static_cast<const {T1}*>(args.in[1]);")
    if not PACKED:
        w(f"  const {T2}* __restrict__ t2 = static_cast<const {T2}*>(args.in[2]);")
    w(f"  {OT}* __restrict__ out = static_cast<{OT}*>(args.out[0]);")
    w("  const long long total = args.rows * SPR;")
    w("  const long long stride = (long long)gridDim.x * blockDim.x;")
    w("  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; "
      "i += stride) {")
    w("    const long long row = i / SPR;")
    w("    const int j = (int)(i - row * SPR);")
    w("    const long long pos = ((args.row_offset + row) / HEADS) % SEQ;")
    w("    const long long xo = row * D + (long long)j * VEC;")
    # ---- gather the slot's elements and its pairs' cos / sin as fp32
    if half:
        npair = VEC
        w(f"    float a[VEC], b[VEC], cs[VEC], sn[VEC];      // pairs (a[e], b[e])")
        if SCALAR:
            w("#pragma unroll")
            w("    for (int e = 0; e < VEC; ++e) {")
            w("      a[e] = to_f32(x[xo + e]);")
            w("      b[e] = to_f32(x[xo + D / 2 + e]);")
            w("    }")
        else:
            w(f"    {{ const Slot<{XT}, VEC> s = load_slot<kLoadStream, {XT}, VEC>(x + xo);")
            w("#pragma unroll")
            w("      for (int e = 0; e < VEC; ++e) a[e] = to_f32(s.v[e]); }")
            w(f"    {{ const Slot<{XT}, VEC> s = load_slot<kLoadStream, {XT}, VEC>(x + xo + D / 2);")
            w("#pragma unroll")
            w("      for (int e = 0; e < VEC; ++e) b[e] = to_f32(s.v[e]); }")
        pair0 = "(long long)j * VEC"
    else:
        npair = max(1, VEC // 2)
        w(f"    float a[VEC / 2], b[VEC / 2], cs[VEC / 2], sn[VEC / 2];   // pairs (a[p], b[p])")
        if SCALAR:
            w("#pragma unroll")
            w("    for (int p = 0; p < VEC / 2; ++p) {")
            w("      a[p] = to_f32(x[xo + 2 * p]);")
            w("      b[p] = to_f32(x[xo + 2 * p + 1]);")
            w("    }")
        else:
            w(f"    {{ const Slot<{XT}, VEC> s = load_slot<kLoadStream, {XT}, VEC>(x + xo);")
            w("#pragma unroll")
            w("      for (int p = 0; p < VEC / 2; ++p) { a[p] = to_f32(s.v[2 * p]); "
              "b[p] = to_f32(s.v[2 * p + 1]); } }")
        pair0 = "(long long)j * (VEC / 2)"
    NP = "VEC" if half else "VEC / 2"
    w(f"    const long long p0 = {pair0};                  // first pair of this thread")
    if PACKED:
        # (cos, sin) of pair q at t1[pos * D + 2 q], t1[pos * D + 2 q + 1]
        if SCALAR:
            w("#pragma unroll")
            w(f"    for (int p = 0; p < {NP}; ++p) {{")
            w("      cs[p] = to_f32(t1[pos * D + 2 * (p0 + p)]);")
            w("      sn[p] = to_f32(t1[pos * D + 2 * (p0 + p) + 1]);")
            w("    }")
        else:
            w(f"    {{ const Slot<{T1}, 2 * ({NP})> s = "
              f"load_slot<kLoadDefault, {T1}, 2 * ({NP})>(t1 + pos * D + 2 * p0);")
            w("#pragma unroll")
            w(f"      for (int p = 0; p < {NP}; ++p) {{ cs[p] = to_f32(s.v[2 * p]); "
              "sn[p] = to_f32(s.v[2 * p + 1]); } }")
    else:
        if SCALAR:
            w("#pragma unroll")
            w(f"    for (int p = 0; p < {NP}; ++p) {{")
            w("      cs[p] = to_f32(t1[pos * (D / 2) + p0 + p]);")
            w("      sn[p] = to_f32(t2[pos * (D / 2) + p0 + p]);")
            w("    }")
        else:
            w(f"    {{ const Slot<{T1}, {NP}> s = "
              f"load_slot<kLoadDefault, {T1}, {NP}>(t1 + pos * (D / 2) + p0);")
            w("#pragma unroll")
            w(f"      for (int p = 0; p < {NP}; ++p) cs[p] = to_f32(s.v[p]); }}")
            w(f"    {{ const Slot<{T2}, {NP}> s = "
              f"load_slot<kLoadDefault, {T2}, {NP}>(t2 + pos * (D / 2) + p0);")
            w("#pragma unroll")
            w(f"      for (int p = 0; p < {NP}; ++p) sn[p] = to_f32(s.v[p]); }}")
    # ---- rotate and store
    if half:
        w("    float o1[VEC], o2[VEC];")
        w("#pragma unroll")
        w("    for (int e = 0; e < VEC; ++e) {")
        w("      o1[e] = a[e] * cs[e] - b[e] * sn[e];")
        w("      o2[e] = a[e] * sn[e] + b[e] * cs[e];")
        w("    }")
        if SCALAR:
            w("#pragma unroll")
            w("    for (int e = 0; e < VEC; ++e) {")
            w(f"      out[xo + e] = from_f32<{OT}>(o1[e]);")
            w(f"      out[xo + D / 2 + e] = from_f32<{OT}>(o2[e]);")
            w("    }")
        else:
            w(f"    Slot<{OT}, VEC> s1, s2;")
            w(f"    pack_slot<{OT}, VEC>(s1, o1);")
            w(f"    pack_slot<{OT}, VEC>(s2, o2);")
            w(f"    store_slot<kStoreDefault, {OT}, VEC>(out + xo, s1);")
            w(f"    store_slot<kStoreDefault, {OT}, VEC>(out + xo + D / 2, s2);")
    else:
        w("    float o[VEC];")
        w("#pragma unroll")
        w("    for (int p = 0; p < VEC / 2; ++p) {")
        w("      o[2 * p] = a[p] * cs[p] - b[p] * sn[p];")
        w("      o[2 * p + 1] = a[p] * sn[p] + b[p] * cs[p];")
        w("    }")
        if SCALAR:
            w("#pragma unroll")
            w(f"    for (int e = 0; e < VEC; ++e) out[xo + e] = from_f32<{OT}>(o[e]);")
        else:
            w(f"    Slot<{OT}, VEC> so;")
            w(f"    pack_slot<{OT}, VEC>(so, o);")
            w(f"    store_slot<kStoreDefault, {OT}, VEC>(out + xo, so);")
    w("  }")
    w("}")
    del npair
    return "\n".join(L) + "\n"


def rope_table_slot(config: dict) -> int:
    """Table elements one thread reads per table in vector mode."""
    vec = config["vec"]
    npair = vec if config["style"] == "half" else vec // 2
    return 2 * npair if config["packed"] else npair
