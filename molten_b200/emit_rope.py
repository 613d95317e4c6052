"""CUDA C++ emission for the RoPE (ROTATE) sub-kernel.

Semantics of ``benchmarks/ops.py:24-35``: x [..., seq, heads, head_dim]
viewed as rows of head_dim elements; row r sits at position
p = ((row_offset + r) / heads) % seq; each pair (x0, x1) becomes
(x0 cos - x1 sin, x0 sin + x1 cos) with cos, sin = table[p, pair].

Pairs are (2i, 2i+1) ("interleaved", as in ops.py) or (i, i + head_dim/2)
("half").  Tables are cos and sin [seq, head_dim/2], or one packed
[seq, head_dim] table of (cos, sin) per pair.  fp32 arithmetic, one
rounding to x's dtype.

Vector form: per grid-stride step a thread takes UPT items one block apart,
an item being one 16-byte slot of x (VEC elements, VEC/2 pairs; with
"half" the slot and its partner slot in the second half, VEC pairs); it
issues all the items' x loads and table loads (cached: every head of a
position reads the same table row) before rotating and storing any, so
UPT loads per operand are in flight per thread.  The ``scalar`` form, for
pointers that are not 16-byte aligned, moves one pair per thread per step
with element accesses.
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
    if not SCALAR:
        _emit_vector_body(w, c, XT, T1, T2, OT, half, PACKED)
        w("}")
        return "\n".join(L) + "\n"
    # scalar form: one pair per thread per step, element accesses only
    w("  const long long stride = (long long)gridDim.x * blockDim.x;")
    w("  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; "
      "i += stride) {")
    w("    const long long row = i / SPR;")
    w("    const int j = (int)(i - row * SPR);")
    w("    const long long pos = ((args.row_offset + row) / HEADS) % SEQ;")
    if half:
        # pair j: elements j and j + D/2 (VEC == 1)
        w("    const long long ia = row * D + j, ib = ia + D / 2;")
    else:
        # pair j: elements 2j and 2j + 1 (VEC == 2)
        w("    const long long ia = row * D + 2LL * j, ib = ia + 1;")
    w("    const float a = to_f32(x[ia]), b = to_f32(x[ib]);")
    if PACKED:
        w("    const float cs = to_f32(t1[pos * D + 2LL * j]);")
        w("    const float sn = to_f32(t1[pos * D + 2LL * j + 1]);")
    else:
        w("    const float cs = to_f32(t1[pos * (D / 2) + j]);")
        w("    const float sn = to_f32(t2[pos * (D / 2) + j]);")
    w(f"    out[ia] = from_f32<{OT}>(a * cs - b * sn);")
    w(f"    out[ib] = from_f32<{OT}>(a * sn + b * cs);")
    w("  }")
    w("}")
    return "\n".join(L) + "\n"


def _emit_vector_body(w, c, XT, T1, T2, OT, half: bool, packed: bool):
    """Vector form: each thread takes UPT items (x slots) spaced one block
    apart per grid-stride step; all their x and table loads are issued
    before any rotation or store, so UPT 16-byte loads per operand are in
    flight per thread."""
    UPT = c.get("upt", 2)
    NP = "VEC" if half else "VEC / 2"                  # pairs per item
    NT = f"2 * ({NP})" if packed else NP              # table entries per item and table
    w(f"  constexpr int UPT = {UPT};")
    w("  const long long step = (long long)gridDim.x * blockDim.x * UPT;")
    w("  for (long long base = (long long)blockIdx.x * blockDim.x * UPT + threadIdx.x; "
      "base < total; base += step) {")
    w(f"    Slot<{XT}, VEC> xa[UPT];")
    if half:
        w(f"    Slot<{XT}, VEC> xb[UPT];")
    w(f"    Slot<{T1}, {NT}> ta[UPT];")
    if not packed:
        w(f"    Slot<{T2}, {NT}> tb[UPT];")
    w("    long long xo[UPT];")
    w("#pragma unroll")
    w("    for (int u = 0; u < UPT; ++u) {             // loads")
    w("      const long long i = base + (long long)u * blockDim.x;")
    w("      xo[u] = -1;")
    w("      if (i >= total) continue;")
    w("      const long long row = i / SPR;")
    w("      const int j = (int)(i - row * SPR);")
    w("      const long long pos = ((args.row_offset + row) / HEADS) % SEQ;")
    w("      xo[u] = row * D + (long long)j * VEC;")
    w(f"      const long long p0 = (long long)j * ({NP});")
    w(f"      xa[u] = load_slot<kLoadStream, {XT}, VEC>(x + xo[u]);")
    if half:
        w(f"      xb[u] = load_slot<kLoadStream, {XT}, VEC>(x + xo[u] + D / 2);")
    if packed:
        w(f"      ta[u] = load_slot<kLoadDefault, {T1}, {NT}>(t1 + pos * D + 2 * p0);")
    else:
        w(f"      ta[u] = load_slot<kLoadDefault, {T1}, {NT}>(t1 + pos * (D / 2) + p0);")
        w(f"      tb[u] = load_slot<kLoadDefault, {T2}, {NT}>(t2 + pos * (D / 2) + p0);")
    w("    }")
    w("#pragma unroll")
    w("    for (int u = 0; u < UPT; ++u) {             // rotate, round once, store")
    w("      if (xo[u] < 0) continue;")
    w(f"      float cs[{NP}], sn[{NP}];")
    w("#pragma unroll")
    w(f"      for (int p = 0; p < {NP}; ++p) {{")
    if packed:
        w("        cs[p] = to_f32(ta[u].v[2 * p]);")
        w("        sn[p] = to_f32(ta[u].v[2 * p + 1]);")
    else:
        w("        cs[p] = to_f32(ta[u].v[p]);")
        w("        sn[p] = to_f32(tb[u].v[p]);")
    w("      }")
    if half:
        w("      float o1[VEC], o2[VEC];")
        w("#pragma unroll")
        w("      for (int e = 0; e < VEC; ++e) {")
        w("        const float a = to_f32(xa[u].v[e]), b = to_f32(xb[u].v[e]);")
        w("        o1[e] = a * cs[e] - b * sn[e];")
        w("        o2[e] = a * sn[e] + b * cs[e];")
        w("      }")
        w(f"      Slot<{OT}, VEC> s1, s2;")
        w(f"      pack_slot<{OT}, VEC>(s1, o1);")
        w(f"      pack_slot<{OT}, VEC>(s2, o2);")
        w(f"      store_slot<kStoreDefault, {OT}, VEC>(out + xo[u], s1);")
        w(f"      store_slot<kStoreDefault, {OT}, VEC>(out + xo[u] + D / 2, s2);")
    else:
        w("      float o[VEC];")
        w("#pragma unroll")
        w("      for (int p = 0; p < VEC / 2; ++p) {")
        w("        const float a = to_f32(xa[u].v[2 * p]), b = to_f32(xa[u].v[2 * p + 1]);")
        w("        o[2 * p] = a * cs[p] - b * sn[p];")
        w("        o[2 * p + 1] = a * sn[p] + b * cs[p];")
        w("      }")
        w(f"      Slot<{OT}, VEC> so;")
        w(f"      pack_slot<{OT}, VEC>(so, o);")
        w(f"      store_slot<kStoreDefault, {OT}, VEC>(out + xo[u], so);")
    w("    }")
    w("  }")


def rope_table_slot(config: dict) -> int:
    """Table elements one thread reads per table in vector mode."""
    vec = config["vec"]
    npair = vec if config["style"] == "half" else vec // 2
    return 2 * npair if config["packed"] else npair
