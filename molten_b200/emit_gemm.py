"""CUDA emission for the MATMUL + elementwise-epilogue family.

The emitted module instantiates the tcgen05 engine of
``molten/gemm_sm100.cuh`` with a generated epilogue functor: the epilogue
warps read 32 fp32 accumulator columns of one output row from TMEM, and the
functor applies the fused ops (bias add, GELU, ...) in fp32, rounds once and
stores 16 bytes at a time.
"""

from __future__ import annotations

from .emit import _mask_period, _row_index_expr, c_float, value_expr
from .lowering import DTYPE_CTYPE, DTYPE_SIZE, LoweringError, SubKernel


def emit_gemm(sk: SubKernel, name: str) -> str:
    cfg = sk.config
    BM, BN, BK, ST = cfg["bm"], cfg["bn"], cfg["bk"], cfg["stages"]
    a = sk.operands[sk.a_operand]
    split3 = "true" if cfg.get("split3") else "false"
    # fp32 operands reach the tensor cores as bf16 planes
    f16in = "true" if a.dtype == "float16" and not cfg.get("split3") else "false"
    values = sk.values
    needed = set(cfg["needed"])
    L = []
    w = L.append
    pair = bool(cfg.get("pair"))
    w(f"// Molten sm_100a tcgen05 GEMM + epilogue: {name}")
    w(f"// C[{sk.m}, {sk.n}] = epilogue(A[{sk.m}, {sk.k}] @ B[{sk.k}, {sk.n}]); "
      f"tile {BM}x{BN}x{BK}, {ST} stages" + ("; SM pair (cta_group::2)" if pair else ""))
    if cfg.get("split3"):
        w("// fp32 operands as three bf16 planes each (bf16x3: six products per k-block)")
    streamk = bool(cfg.get("streamk"))
    w("#include \"molten/gemm2_sm100.cuh\"" if pair else
      ("#include \"molten/gemm_sk_sm100.cuh\"" if streamk else "#include \"molten/gemm_sm100.cuh\""))
    w("")
    w("using namespace molten;")
    w("")
    w("namespace {")
    w(f"constexpr int TILE_M = {BM}, TILE_N = {BN}, TILE_K = {BK}, STAGES = {ST};")
    pro = cfg.get("prologue")
    if pair:
        if pro:
            raise LoweringError("the SM-pair GEMM has no RMSNorm prologue")
        w(f"typedef Gemm2Layout<TILE_N, STAGES, {cfg.get('group_m', 16)}> Layout_{name};")
        w(f"static_assert(Layout_{name}::SMEM_BYTES <= {cfg['smem_bytes']}, \"shared memory\");")
    else:
        w(f"typedef GemmLayout<TILE_M, TILE_N, TILE_K, STAGES, {cfg.get('group_m', 16)}, "
          f"{'true' if pro else 'false'}> Layout_{name};")
    if pro:
        wt = DTYPE_CTYPE[pro["w_dtype"]]
        w(f"// RMSNorm prologue: A = x / sqrt(mean(x^2) + eps) * w, normalised as it is staged")
        w(f"struct Prologue_{name} {{")
        w("  static constexpr bool ENABLED = true;")
        w(f"  static constexpr float EPS = {c_float(pro['eps'])};")
        w("  // w[k0 .. k0 + 31] (k0 a multiple of 8; 0 beyond K, which is a multiple of 8)")
        w("  __device__ __forceinline__ static void w32(const GemmArgs& args, long long k0, float (&w)[32]) {")
        w(f"    const {wt}* p = static_cast<const {wt}*>(args.in[{pro['w']}]);")
        w("#pragma unroll")
        w("    for (int q = 0; q < 4; ++q) {")
        w(f"      Slot<{wt}, 8> s;")
        w(f"      if (k0 + 8 * q < args.k) s = load_slot<kLoadDefault, {wt}, 8>(p + k0 + 8 * q);")
        w("      else {")
        w("#pragma unroll")
        w(f"        for (int e = 0; e < 8; ++e) s.v[e] = from_f32<{wt}>(0.0f);")
        w("      }")
        w("#pragma unroll")
        w("      for (int e = 0; e < 8; ++e) w[8 * q + e] = to_f32(s.v[e]);")
        w("    }")
        w("  }")
        w("};")
    w(f"struct Epilogue_{name} {{")
    w("  // C[row, col0 .. col0 + 31] from the fp32 accumulators of one TMEM row")
    w("  __device__ __forceinline__ static void apply(const GemmArgs& args, long long row,")
    w("                                               long long col0, const float (&acc)[32]) {")
    w(f"    constexpr long long N = {sk.n}LL;")
    w("    const long long grow = args.row_offset + row;")
    w("    (void)grow;")
    # row-level leaves
    for vid in sorted(needed):
        v = values[vid]
        if v.op == "load" and v.kind == "row":
            o = sk.operands[v.attrs["operand"]]
            ct = DTYPE_CTYPE[o.dtype]
            idx = _row_index_expr(o, "row", "grow")
            w(f"    const float v{vid} = load_scalar(static_cast<const {ct}*>(args.in[{o.index}]) + {idx});")
        if v.op == "mask":
            period = _mask_period(v, sk.n)
            off = int(v.attrs.get("offset", 0))
            w(f"    const int mlim{vid} = clamp_col_limit((grow % {period}LL) + ({off}LL));")
    for vid in sorted(needed):
        v = values[vid]
        if v.kind in ("row", "const") and v.op not in ("load", "const"):
            args = [_leaf(sk, x) for x in v.args]
            w(f"    const float v{vid} = {value_expr(v, args, True)};")
    vec_ops = sorted({values[v].attrs["operand"] for v in needed
                      if values[v].op == "load" and values[v].kind == "elem"})
    # 16-byte chunk accesses need every row of every row-indexed operand and
    # output to start on a 16-byte boundary; otherwise (and for the last,
    # partial chunk of a row) elements are moved one at a time
    strides = [DTYPE_SIZE[o.dtype] for o in sk.outputs]
    strides += [DTYPE_SIZE[sk.operands[i].dtype] for i in vec_ops
                if sk.operands[i].row_map != "zero"]
    vec_ok = all((sk.n * e) % 16 == 0 for e in strides)
    w(f"    constexpr bool ROWS_ALIGNED = {'true' if vec_ok else 'false'};")
    w("#pragma unroll")
    w("    for (int q = 0; q < 4; ++q) {")
    w("      const long long c = col0 + 8 * q;")
    w("      if (c >= N) break;")
    w("      const bool whole = ROWS_ALIGNED && c + 8 <= N;")
    w("      const int valid = (int)(N - c < 8 ? N - c : 8);")
    for i in vec_ops:
        o = sk.operands[i]
        ct = DTYPE_CTYPE[o.dtype]
        idx = _row_index_expr(o, "row", "grow")
        w(f"      const {ct}* src{i} = static_cast<const {ct}*>(args.in[{i}]) + {idx} * N + c;")
        w(f"      Slot<{ct}, 8> sl{i};")
        w(f"      if (whole) {{ sl{i} = load_slot<kLoadDefault, {ct}, 8>(src{i}); }}")
        w("      else {")
        w("#pragma unroll")
        w(f"        for (int e = 0; e < 8; ++e) sl{i}.v[e] = e < valid ? src{i}[e] : from_f32<{ct}>(0.0f);")
        w("      }")
    for o in sk.outputs:
        w(f"      float f{o.index}[8];")
    w("#pragma unroll")
    w("      for (int e = 0; e < 8; ++e) {")
    if any(values[v].op == "mask" for v in needed):
        w("        const int col = (int)c + e;")
    for vid in sorted(needed):
        v = values[vid]
        if v.kind != "elem" or v.op in ("load", "acc"):
            continue
        if v.op == "mask":
            w(f"        const float v{vid} = (col > mlim{vid}) ? (-INFINITY) : 0.0f;")
            continue
        args = [_leaf(sk, x) for x in v.args]
        w(f"        const float v{vid} = {value_expr(v, args, sk.precise)};")
    for o in sk.outputs:
        w(f"        f{o.index}[e] = {_leaf(sk, sk.out_values[o.index])};")
    w("      }")
    for o in sk.outputs:
        ct = DTYPE_CTYPE[o.dtype]
        w(f"      {ct}* dst{o.index} = static_cast<{ct}*>(args.out[{o.index}]) + row * N + c;")
        w(f"      if (whole) {{ Slot<{ct}, 8> o{o.index}; pack_slot<{ct}, 8>(o{o.index}, f{o.index}); "
          f"store_slot<kStoreDefault, {ct}, 8>(dst{o.index}, o{o.index}); }}")
        w("      else {")
        w("#pragma unroll")
        w(f"        for (int e = 0; e < 8; ++e) if (e < valid) dst{o.index}[e] = from_f32<{ct}>(f{o.index}[e]);")
        w("      }")
    w("    }")
    w("  }")
    w("};")
    w("}  // namespace")
    w("")
    w(f"extern \"C\" __global__ void __launch_bounds__({cfg['threads']}, 1) "
      f"{name}(const __grid_constant__ GemmArgs args) {{")
    w("  extern __shared__ __align__(1024) uint8_t smem_raw[];")
    if pair:
        kmaj = "true" if cfg.get("b_kmajor") else "false"
        w(f"  const GemmShared sh = gemm2_carve<Layout_{name}>(smem_raw);")
        w(f"  gemm2_init<Layout_{name}>(sh, args);    // mbarriers, pair TMEM allocation, pair barrier")
        w("  pdl_enter();                            // no global access before this")
        w(f"  gemm2_roles<Layout_{name}, {f16in}, Epilogue_{name}, {kmaj}, {split3}>(sh, args);")
        w("  __syncthreads();")
        w(f"  gemm2_teardown<Layout_{name}>(sh);      // pair barrier, pair TMEM release")
        w("}")
        return "\n".join(L) + "\n"
    w(f"  const GemmShared sh = gemm_carve<Layout_{name}>(smem_raw);")
    if streamk:
        kmaj = "true" if cfg.get("b_kmajor") else "false"
        w(f"  gemm_sk_init<Layout_{name}>(sh, args);  // mbarriers + TMEM allocation")
        w("  pdl_enter();                            // no global access before this")
        w("  __syncthreads();")
        w(f"  gemm_sk_roles<Layout_{name}, {f16in}, Epilogue_{name}, {kmaj}, {cfg['sk_maxseg']}, "
          f"{cfg.get('sk_splits', 0)}>(sh, args);")
        w("  __syncthreads();")
        w(f"  gemm_teardown<Layout_{name}>(sh);       // TMEM release")
        w("}")
        return "\n".join(L) + "\n"
    w(f"  gemm_init<Layout_{name}>(sh, args);     // mbarriers + TMEM allocation")
    w("  pdl_enter();                            // no global access before this")
    w("  __syncthreads();")
    kmaj = "true" if cfg.get("b_kmajor") else "false"
    pro_t = f"Prologue_{name}" if pro else "NoPrologue"
    w(f"  gemm_roles<Layout_{name}, {f16in}, Epilogue_{name}, {kmaj}, {pro_t}, {split3}>(sh, args);")
    w("  __syncthreads();")
    w(f"  gemm_teardown<Layout_{name}>(sh);       // TMEM release")
    w("}")
    return "\n".join(L) + "\n"


def emit_split3(sk: SubKernel, name: str) -> str:
    """Kernel writing a GEMM operand as three stacked bf16 planes
    (x ~ x0 + x1 + x2, molten::split3_value): grid-stride over VEC-element
    slots, one read of the operand and three 16-byte plane stores per slot."""
    cfg = sk.config
    src = sk.operands[0]
    ct = DTYPE_CTYPE[src.dtype]
    total, vec = cfg["total"], cfg["vec"]
    L = []
    w = L.append
    w(f"// Molten sm_100a: {name} -- operand {src.name!r} {list(src.shape)} {src.dtype} "
      f"-> bf16 planes [3, {total}]")
    w("#include \"molten/gemm_sm100.cuh\"")
    w("#include \"molten/row_engine.cuh\"")
    w("")
    w("using namespace molten;")
    w("")
    w(f"extern \"C\" __global__ void __launch_bounds__({cfg['block']}) "
      f"{name}(const __grid_constant__ RowArgs args) {{")
    w("  pdl_enter();")
    w(f"  constexpr long long TOTAL = {total}LL;")
    w(f"  constexpr int VEC = {vec};")
    w(f"  const {ct}* __restrict__ x = static_cast<const {ct}*>(args.in[0]);")
    w("  bf16* __restrict__ p = static_cast<bf16*>(args.out[0]);")
    w("  const long long step = (long long)gridDim.x * blockDim.x;")
    w("  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < TOTAL / VEC; "
      "i += step) {")
    w(f"    const Slot<{ct}, VEC> v = load_slot<kLoadStream, {ct}, VEC>(x + i * VEC);")
    w("    Slot<bf16, VEC> s0, s1, s2;")
    w("#pragma unroll")
    w("    for (int e = 0; e < VEC; ++e) split3_value(to_f32(v.v[e]), s0.v[e], s1.v[e], s2.v[e]);")
    w("    store_slot<kStoreDefault, bf16, VEC>(p + i * VEC, s0);")
    w("    store_slot<kStoreDefault, bf16, VEC>(p + TOTAL + i * VEC, s1);")
    w("    store_slot<kStoreDefault, bf16, VEC>(p + 2 * TOTAL + i * VEC, s2);")
    w("  }")
    w("}")
    return "\n".join(L) + "\n"


def _leaf(sk: SubKernel, vid: int) -> str:
    v = sk.values[vid]
    if v.op == "const" and v.kind == "const":
        return c_float(v.attrs["value"])
    if v.op == "acc":
        return "acc[8 * q + e]"
    if v.op == "load" and v.kind == "elem":
        return f"to_f32(sl{v.attrs['operand']}.v[e])"
    return f"v{vid}"
