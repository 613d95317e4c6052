"""CUDA C++ emission for the row and elementwise families.

Each sub-kernel becomes one ``extern "C" __global__`` function built on
``molten/row_engine.cuh``.  Shapes (cols), dtypes, the op DAG, constants and
the launch geometry are baked in as constexpr; rows and pointers are runtime
kernel arguments (``molten::RowArgs``).
"""

from __future__ import annotations

import math

import numpy as np

from .lowering import DTYPE_CTYPE, LoweringError, SubKernel, Value
from .plan import pass_closures


def c_float(x: float) -> str:
    """Exact fp32 literal for x (rounded to fp32 first)."""
    f = float(np.float32(x))
    if math.isnan(f):
        return "NAN"
    if math.isinf(f):
        return "INFINITY" if f > 0 else "(-INFINITY)"
    if f == 0.0:
        return "-0.0f" if math.copysign(1.0, f) < 0 else "0.0f"
    if f == int(f) and abs(f) < 1e7:
        return f"{int(f)}.0f"
    return f"{f.hex()}f /* {f!r} */"


def value_expr(v: Value, a, precise: bool) -> str:
    """C expression for value v given the spelled arguments a."""
    P = "true" if precise else "false"
    op = v.op
    if op == "add":
        return f"({a[0]} + {a[1]})"
    if op == "sub":
        return f"({a[0]} - {a[1]})"
    if op == "mul":
        return f"({a[0]} * {a[1]})"
    if op == "div":
        return f"({a[0]} / {a[1]})" if precise else f"__fdividef({a[0]}, {a[1]})"
    if op == "rcp":
        return f"(1.0f / {a[0]})"
    if op == "neg":
        return f"(-{a[0]})"
    if op == "sqrt":
        return f"sqrtf({a[0]})"
    if op == "rsqrt":
        return f"rsqrtf({a[0]})"
    if op == "exp":
        return f"expf({a[0]})" if precise else f"__expf({a[0]})"
    if op == "log":
        return f"logf({a[0]})" if precise else f"__logf({a[0]})"
    if op == "tanh":
        return f"tanhf({a[0]})" if precise else f"m_tanh<false>({a[0]})"
    if op == "sigmoid":
        return f"m_sigmoid<{P}>({a[0]})"
    if op == "silu":
        return f"m_silu<{P}>({a[0]})"
    if op == "gelu":
        return f"m_gelu_tanh<{P}>({a[0]})"
    if op == "relu":
        return f"fmaxf({a[0]}, 0.0f)"
    if op == "abs":
        return f"fabsf({a[0]})"
    if op == "clamp":
        e = a[0]
        lo, hi = v.attrs.get("min"), v.attrs.get("max")
        if lo is not None:
            e = f"fmaxf({e}, {c_float(lo)})"
        if hi is not None:
            e = f"fminf({e}, {c_float(hi)})"
        return e
    raise LoweringError(f"no expression for {op}")


_RED_INIT = {"rsum": "0.0f", "rmax": "(-INFINITY)", "rmin": "INFINITY"}
_RED_OP = {"rsum": "OpSum", "rmax": "OpMax", "rmin": "OpMin"}
_RED_COMBINE = {"rsum": "{a} += {x};", "rmax": "{a} = fmaxf({a}, {x});",
                "rmin": "{a} = fminf({a}, {x});"}
_LOAD_HINT = {True: "kLoadStream", False: "kLoadDefault"}


def _ctype(dtype: str) -> str:
    return DTYPE_CTYPE[dtype]


def _row_index_expr(opd, local: str, glob: str) -> str:
    if opd.row_map == "full":
        return local
    if opd.row_map == "zero":
        return "0LL"
    terms = []
    for div, mod, stride in opd.row_terms:
        t = glob if div == 1 else f"({glob} / {div}LL)"
        t = f"({t} % {mod}LL)"
        if stride != 1:
            t = f"{t} * {stride}LL"
        terms.append(t)
    return "(" + " + ".join(terms) + ")" if terms else "0LL"


def _mask_period(v: Value, cols: int) -> int:
    p = v.attrs.get("period")
    return int(p) if p else int(cols)


class _Emitter:
    def __init__(self, sk: SubKernel, name: str):
        self.sk = sk
        self.name = name
        self.values = sk.values
        self.cfg = sk.config
        self.needed = set(self.cfg["needed"])
        self.lines = []

    def w(self, s=""):
        self.lines.append(s)

    # --------------------------------------------------------- leaf spelling
    def leaf(self, vid: int, in_loop: bool, prefetched: set, mat_ready: set,
             loaded_now: set) -> str:
        v = self.values[vid]
        if v.kind == "const" and v.op == "const":
            return c_float(v.attrs["value"])
        if v.kind in ("row", "const"):
            return f"v{vid}"
        if vid in mat_ready:
            if v.op == "softmax":
                return f"(m{vid}[k][e] * sc{vid})"
            return f"m{vid}[k][e]"
        if v.op == "load":
            i = v.attrs["operand"]
            if i in prefetched:
                return f"to_f32(s{i}[k].v[e])"
            return f"to_f32(sl{i}.v[e])"
        if v.op == "acc":
            return "acc[e]"
        return f"v{vid}"

    def elem_statements(self, targets, prefetched, mat_ready, indent):
        """Emit statements for the elem values in ``targets`` (closure),
        in topological order, inside the (k, e) loop."""
        out = []
        for vid in sorted(targets):
            v = self.values[vid]
            if v.kind != "elem" or vid in mat_ready:
                continue
            if v.op in ("load", "acc", "softmax"):
                continue
            if v.op == "mask":
                period = _mask_period(v, self.sk.cols)
                out.append(f"{indent}const float v{vid} = (col > mlim{vid}) ? (-INFINITY) : 0.0f;")
                continue
            args = [self.leaf(a, True, prefetched, mat_ready, set()) for a in v.args]
            out.append(f"{indent}const float v{vid} = {value_expr(v, args, self.sk.precise)};")
        return out

    def row_statement(self, vid, prefetched) -> str:
        # once per row: always the precise form
        v = self.values[vid]
        args = [self.leaf(a, False, prefetched, set(), set()) for a in v.args]
        return f"const float v{vid} = {value_expr(v, args, True)};"

    def header(self, kind: str):
        sk = self.sk
        ops = " -> ".join(v for v in self.cfg.get("op_names", []))
        self.w(f"// Molten sm_100a {kind} kernel: {self.name}")
        if ops:
            self.w(f"// Fused ops: {ops}")
        self.w(f"// cols = {sk.cols}; inputs: " + ", ".join(
            f"{o.name}[{o.dtype} {o.last}/{o.row_map}]" for o in sk.operands))
        self.w("#include \"molten/row_engine.cuh\"")
        self.w("")

    def pointers(self, lrow: str, grow: str, ok: str, vec_slots: bool = True):
        sk = self.sk
        for opd in sk.operands:
            ct = _ctype(opd.dtype)
            idx = _row_index_expr(opd, f"({ok} ? {lrow} : 0LL)", grow)
            stride = "COLS" if opd.last == "vec" else "1LL"
            self.w(f"  const {ct}* __restrict__ in{opd.index} = "
                   f"static_cast<const {ct}*>(args.in[{opd.index}]) + {idx} * {stride};")
        for out in sk.outputs:
            ct = _ctype(out.dtype)
            stride = "COLS" if out.kind == "full" else "1LL"
            self.w(f"  {ct}* __restrict__ out{out.index} = "
                   f"static_cast<{ct}*>(args.out[{out.index}]) + ({ok} ? {lrow} : 0LL) * {stride};")

    def row_leaves(self, prefetched):
        """Row-kind loads and mask limits (computed once per row)."""
        sk = self.sk
        for vid in sorted(self.needed):
            v = self.values[vid]
            if v.op == "load" and v.kind == "row":
                i = v.attrs["operand"]
                self.w(f"  const float v{vid} = rok ? load_scalar(in{i}) : 0.0f;")
            if v.op == "mask":
                period = _mask_period(v, sk.cols)
                off = int(v.attrs.get("offset", 0))
                self.w(f"  const int mlim{vid} = clamp_col_limit((grow % {period}LL) + ({off}LL));")


def emit_row(sk: SubKernel, name: str) -> str:
    """Register-resident row kernel.

    Default form: one team of TPC threads (in CL CTAs of a cluster) per row,
    RPC teams per CTA, one launch-wide pass over the rows.

    ``config["stream"] = S > 0``: a persistent form for long rows.  The grid
    is sized to what is resident; each team walks rows ``base0 + i * step``
    and every thread copies its own slots of the next S-1 rows into shared
    memory with cp.async (one commit group per row), so HBM reads stay in
    flight through the current row's reductions, barriers and stores.
    Row-invariant operands are loaded once.  With a cluster, partials are
    pushed into the peers' shared memory (st.async completing on the
    receiver's mbarrier) instead of a barrier.cluster round, whose release
    fence would wait for the previous row's output stores.  Exchange areas
    alternate with the row's parity: a peer pushes row n+2's partials into an
    area only after this CTA's row n+1 push, which follows its reads of row
    n's values there.
    """
    e = _Emitter(sk, name)
    cfg = sk.config
    VEC, NV, TPC, RPC, CL = cfg["vec"], cfg["nv"], cfg["tpc"], cfg["rpc"], cfg["cl"]
    stream = int(cfg.get("stream", 0) or 0)
    prefetch = set(cfg["prefetch"])
    materialize = {int(v): int(p) for v, p in cfg["materialize"]}
    values = sk.values
    needed = e.needed
    closures = pass_closures(values, sk, needed, materialize)
    # reductions per pass, in id order
    reds = {p: [] for p in range(sk.passes)}
    for vid in sorted(needed):
        v = values[vid]
        if v.op in ("rsum", "rmax", "rmin"):
            reds[v.avail - 1].append(vid)
    smx = smx_of(values, needed, sk.passes)
    # one exchange area per reduce call (two sets in the stream form)
    n_calls = sum(len({values[r].op for r in rs}) for rs in reds.values())
    n_calls += sum(len(v) for v in smx.values())
    n_calls = max(n_calls, 1)
    max_nr = max([len(rs) for rs in reds.values()] + [2 if any(smx.values()) else 1]) or 1
    n_areas = n_calls * (2 if stream else 1)
    masked_only = _causal_masked_only_operands(sk, closures, reds, smx, materialize)

    e.header("row")
    e.w("using namespace molten;")
    e.w("")
    minb = cfg.get("min_blocks", 0)
    lb = f"{TPC * RPC}, {minb}" if minb else f"{TPC * RPC}"
    e.w(f"extern \"C\" __global__ void __launch_bounds__({lb}) "
        f"{name}(const __grid_constant__ RowArgs args) {{")
    e.w("  pdl_enter();")
    e.w(f"  constexpr int VEC = {VEC}, NV = {NV}, TPC = {TPC}, RPC = {RPC}, CL = {CL};")
    e.w(f"  constexpr long long COLS = {sk.cols}LL;")
    e.w(f"  constexpr int NVEC = {cfg['nvec']};")
    e.w("  typedef RowTeam<TPC, RPC, CL> Team;")
    e.w(f"  __shared__ float red_smem[Team::smem_floats({max_nr}, {n_areas}) > 0 ? "
        f"Team::smem_floats({max_nr}, {n_areas}) : 1];")
    e.w("  const Team tm(args.rows, 0);")
    # the causal pass may hand masked row tails to the TMA engine (bulk zero
    # stores): its shared zero buffer goes here, its drain before the end
    zmark = len(e.lines)
    e.zero_tail = bool(cfg.get("zero_tail")) and CL == 1 and RPC == 1 and TPC >= 256
    e.zero_tail_used = False
    body = dict(closures=closures, reds=reds, smx=smx, materialize=materialize,
                prefetch=prefetch, masked_only=masked_only)
    if not stream:
        push = CL > 1
        if push:
            _emit_exchange_setup(e, n_areas, max_nr)
            e.w("  constexpr uint32_t xph = 0u;            // one row per team: phase 0 only")
        e.w("  const long long lrow = tm.row;")
        e.w("  const long long grow = args.row_offset + lrow;")
        e.w("  const bool rok = tm.row_ok;")
        e.w("  (void)grow;")
        _emit_row_body(e, staged=[], area=lambda c: f"{c}", done_early=not push, push=push,
                       wait_exchange=push, **body)
        if push:
            _emit_exchange_teardown(e)
        else:
            e.w("  tm.cluster_done_wait();")
        _finish_zero_tail(e, zmark)
        e.w("}")
        return "\n".join(e.lines) + "\n"

    staged = [i for i in sorted(prefetch) if sk.operands[i].row_map != "zero"]
    hoisted = [i for i in sorted(prefetch) if i not in staged]
    if not staged:
        raise LoweringError("the stream form needs a row-indexed streamed operand")
    bulk = bool(cfg.get("bulk"))
    e.w(f"  constexpr int STAGES = {stream}, NSTAGED = {len(staged)};")
    if bulk:
        offs = cfg["bulk_offsets"]
        e.w(f"  constexpr uint32_t STAGE_BYTES = {cfg['stage_bytes']}u;   // whole rows, 128-byte aligned")
        e.w("  constexpr uint32_t " + ", ".join(f"OFF{p} = {o}u" for p, o in enumerate(offs)) + ";")
        e.w("  extern __shared__ __align__(128) uint8_t stage_smem[];")
        e.w("  __shared__ __align__(8) unsigned long long sbar[STAGES];")
        e.w("  __shared__ int sabort;")
        e.w("  const uint32_t sbase = shared_addr(stage_smem);")
        e.w("  if (threadIdx.x == 0) {")
        e.w("    for (int s = 0; s < STAGES; ++s) xch_init(shared_addr(&sbar[s]));")
        e.w("    sabort = 0;")
        e.w("    xch_init_fence();")
        e.w("  }")
        e.w("  __syncthreads();")
    else:
        e.w("  constexpr uint32_t STAGE_BYTES = NSTAGED * NV * (TPC * RPC) * 16u;")
        e.w("  extern __shared__ __align__(16) uint8_t stage_smem[];")
        e.w("  const uint32_t lanes = shared_addr(stage_smem) + threadIdx.x * 16u;")
    e.w("  const long long step = (long long)(gridDim.x / CL) * RPC;")
    e.w("  const long long base0 = (long long)(blockIdx.x / CL) * RPC;")
    for i in hoisted:
        # row-invariant streamed operand: loaded once for every row
        opd = sk.operands[i]
        ct = _ctype(opd.dtype)
        e.w(f"  Slot<{ct}, VEC> s{i}[NV];")
        e.w("  {")
        e.w(f"    const {ct}* __restrict__ src = static_cast<const {ct}*>(args.in[{i}]);")
        e.w("#pragma unroll")
        e.w("    for (int k = 0; k < NV; ++k) {")
        e.w("      const int j = tm.slot(k);")
        e.w(f"      if (j < NVEC) s{i}[k] = load_slot<kLoadDefault, {ct}, VEC>(src + j * VEC);")
        e.w("    }")
        e.w("  }")
    push = CL > 1
    if push:
        _emit_exchange_setup(e, n_areas, max_nr)
    stage_row = _emit_bulk_row if bulk else _emit_stage_row
    e.w("#pragma unroll 1")
    e.w("  for (int s = 0; s < STAGES - 1; ++s) {")
    stage_row(e, staged, masked_only, "base0 + s * step + tm.team", "s", "    ")
    if not bulk:
        e.w("    cp_async_commit();")
    e.w("  }")
    if push:
        e.w("  cluster_wait();")
    e.w("  int st = 0;")
    e.w("  uint32_t use = 0;")
    e.w("#pragma unroll 1")
    e.w("  for (long long base = base0; base < args.rows; base += step) {")
    e.w("    const uint32_t par = use & 1u, xph = (use >> 1) & 1u;   // area set, barrier phase")
    e.w("    (void)par; (void)xph;")
    e.w("    // the row STAGES-1 ahead goes into the stage read one row ago")
    stage_row(e, staged, masked_only, "base + (STAGES - 1) * step + tm.team",
              "(st == 0 ? STAGES - 1 : st - 1)", "    ")
    if bulk:
        # every thread read that stage before the previous row's reduction
        # barrier, which all threads have passed: it is free to refill
        e.w("    xch_wait(shared_addr(&sbar[st]), (use / STAGES) & 1u, &sabort);   // row `base` landed")
    else:
        e.w("    cp_async_commit();")
        e.w("    cp_async_wait<STAGES - 1>();        // this thread's copies of row `base` landed")
    e.w("    const long long lrow = base + tm.team;")
    e.w("    const long long grow = args.row_offset + lrow;")
    e.w("    const bool rok = lrow < args.rows;")
    e.w("    (void)grow;")
    mark = len(e.lines)
    _emit_row_body(e, staged=staged, area=lambda c: f"{c} + (int)par * {n_calls}",
                   done_early=False, push=push, **body)
    e.lines[mark:] = [ln if ln.startswith("#") else "  " + ln for ln in e.lines[mark:]]
    e.w("    st = (st + 1 == STAGES) ? 0 : st + 1;")
    e.w("    ++use;")
    e.w("  }")
    if bulk:
        e.w("  if (threadIdx.x == 0 && sabort && args.status) atomicOr(args.status, kRowTimeoutStage);")
    else:
        e.w("  cp_async_wait<0>();")
    if push:
        _emit_exchange_teardown(e)
    _finish_zero_tail(e, zmark)
    e.w("}")
    return "\n".join(e.lines) + "\n"


ZERO_TAIL_BYTES = 16384      # shared zero buffer the bulk zero stores read


def _finish_zero_tail(e: "_Emitter", zmark: int):
    """When the causal pass used bulk zero stores: the zero buffer (filled
    and fenced for the TMA engine before any row) at ``zmark``, and the
    issuing thread's drain of its bulk groups before the kernel ends."""
    if not e.zero_tail_used:
        return
    e.lines[zmark:zmark] = [
        f"  constexpr uint32_t ZBYTES = {ZERO_TAIL_BYTES}u;",
        "  __shared__ __align__(128) uint4 zbuf[ZBYTES / 16];",
        "  zero_shared_for_bulk(zbuf, ZBYTES);     // zeros the bulk zero-tail stores read",
        "  __syncthreads();",
        "  const uint32_t zsrc = shared_addr(zbuf);",
    ]
    e.w("  if (threadIdx.x == 0) bulk_zero_drain();   // this thread's bulk zero stores are done")


def _emit_exchange_setup(e: _Emitter, n_areas: int, max_nr: int):
    """Shared state of the push exchange (cluster kernels): one mbarrier per
    exchange area, initialised by thread 0 and published to the cluster by a
    release arrive; the matching cluster_wait() comes before the first
    push."""
    e.w("  // cluster partials are pushed (st.async + mbarrier), not exchanged")
    e.w("  // behind a barrier.cluster round")
    e.w(f"  constexpr int NAREAS = {n_areas}, XNR = {max_nr};")
    e.w("  __shared__ float xslots[NAREAS * RPC * CL * XNR];")
    e.w("  __shared__ __align__(8) unsigned long long xbar[NAREAS];")
    e.w("  __shared__ int xabort;")
    e.w("  if (threadIdx.x == 0) {")
    e.w("    for (int a = 0; a < NAREAS; ++a) xch_init(shared_addr(&xbar[a]));")
    e.w("    xabort = 0;")
    e.w("    xch_init_fence();")
    e.w("  }")
    e.w("  cluster_arrive();          // every peer's barriers exist before the first push")
    e.w("  const ClusterExchange xch{xslots, shared_addr(xbar), XNR, &xabort};")


def _emit_exchange_teardown(e: _Emitter):
    """Report a timed-out exchange wait; keep every CTA of the cluster alive
    until all have finished (a relaxed barrier: it hands over no data)."""
    e.w("  if (threadIdx.x == 0 && xabort && args.status) atomicOr(args.status, kRowTimeoutExchange);")
    e.w("  cluster_arrive_relaxed();")
    e.w("  cluster_wait();")


def _emit_bulk_row(e: _Emitter, staged, masked_only, row_expr: str, stage_expr: str, indent: str):
    """Thread 0 arms stage ``stage_expr``'s mbarrier with the byte count of
    local row ``row_expr`` (if it exists) and copies each staged operand's
    row with one bulk copy; a causal softmax's operand is copied only up to
    its last visible slot."""
    sk = e.sk

    def w(s):
        e.w(indent + s)

    w("if (threadIdx.x == 0) {")
    w(f"  const long long fr = {row_expr};")
    w("  if (fr < args.rows) {")
    w("    const long long fg = args.row_offset + fr;")
    w("    (void)fg;")
    w(f"    const uint32_t bar = shared_addr(&sbar[{stage_expr}]);")
    w(f"    const uint32_t dst = sbase + (uint32_t)({stage_expr}) * STAGE_BYTES;")
    terms = []
    for p, i in enumerate(staged):
        opd = sk.operands[i]
        ct = _ctype(opd.dtype)
        row_bytes = sk.cols * (2 if opd.dtype != "float32" else 4)
        w(f"    const {ct}* src{p} = static_cast<const {ct}*>(args.in[{i}]) + "
          f"{_row_index_expr(opd, 'fr', 'fg')} * COLS;")
        if i in masked_only:
            mk = masked_only[i]
            v = e.values[mk]
            period = _mask_period(v, sk.cols)
            off = int(v.attrs.get("offset", 0))
            w(f"    const int fl{p} = clamp_col_limit((fg % {period}LL) + ({off}LL));")
            # visible slots 0 .. fl / VEC, 16 bytes each
            w(f"    const uint32_t nb{p} = fl{p} < 0 ? 0u : "
              f"(uint32_t)min((long long){row_bytes}, ((long long)fl{p} / VEC + 1) * 16LL);")
        else:
            w(f"    const uint32_t nb{p} = {row_bytes}u;")
        terms.append(f"nb{p}")
    w(f"    xch_arm(bar, {' + '.join(terms)});")
    for p, i in enumerate(staged):
        w(f"    if (nb{p}) bulk_row_g2s(dst + OFF{p}, src{p}, nb{p}, bar);")
    w("  }")
    w("}")


def _emit_stage_row(e: _Emitter, staged, masked_only, row_expr: str, stage_expr: str, indent: str):
    """cp.async this thread's slots of local row ``row_expr`` (if it exists)
    into stage ``stage_expr``: staged operand p, slot k at lane offset
    ((p * NV + k) * BLOCK) * 16.  Slots a causal softmax never reads are not
    copied."""
    sk = e.sk

    def w(s):
        e.w(indent + s)

    w("{")
    w(f"  const long long fr = {row_expr};")
    w("  if (fr < args.rows) {")
    w("    const long long fg = args.row_offset + fr;")
    w("    (void)fg;")
    for mk in sorted({masked_only[i] for i in staged if i in masked_only}):
        v = e.values[mk]
        period = _mask_period(v, sk.cols)
        off = int(v.attrs.get("offset", 0))
        w(f"    const int fl{mk} = clamp_col_limit((fg % {period}LL) + ({off}LL));")
    for i in staged:
        opd = sk.operands[i]
        ct = _ctype(opd.dtype)
        # one base per row; slot k is a constant stride further
        w(f"    const {ct}* __restrict__ src{i} = static_cast<const {ct}*>(args.in[{i}]) + "
          f"({_row_index_expr(opd, 'fr', 'fg')} * COLS + (long long)tm.slot(0) * VEC);")
    w(f"    const uint32_t dst = lanes + (uint32_t)({stage_expr}) * STAGE_BYTES;")
    e.w("#pragma unroll")
    w("    for (int k = 0; k < NV; ++k) {")
    w("      const int j = tm.slot(k);")
    w("      if (j < NVEC) {")
    for p, i in enumerate(staged):
        cp = (f"cp_async16(dst + (uint32_t)(({p} * NV + k) * (TPC * RPC) * 16), "
              f"src{i} + k * (TPC * CL * VEC));")
        if i in masked_only:
            w(f"        if (j * VEC <= fl{masked_only[i]}) {cp}")
        else:
            w(f"        {cp}")
    w("      }")
    w("    }")
    w("  }")
    w("}")


def _emit_row_body(e: _Emitter, closures, reds, smx, materialize, prefetch, masked_only, staged,
                   area, done_early: bool, push: bool = False, wait_exchange: bool = False):
    """Everything a team does for its current row (``lrow``/``grow``/``rok``
    in scope): pointers, per-row leaves, the streamed slots (global loads, or
    shared-memory reads of the staged copies), the reduction passes and the
    outputs."""
    sk = e.sk
    values = sk.values
    needed = e.needed
    e.pointers("lrow", "grow", "rok")
    e.row_leaves(prefetch)
    emitted_rows = set()

    def emit_rows_at(p):
        for vid in sorted(needed):
            v = values[vid]
            if v.kind in ("row", "const") and v.avail == p and vid not in emitted_rows \
                    and v.op not in ("load", "const", "rsum", "rmax", "rmin"):
                e.w("  " + e.row_statement(vid, prefetch))
                emitted_rows.add(vid)

    emit_rows_at(0)
    # the row-streamed operands: into registers (row-invariant ones of the
    # stream form are already there)
    per_row = [i for i in sorted(prefetch) if not staged or i in staged]
    for i in per_row:
        e.w(f"  Slot<{_ctype(sk.operands[i].dtype)}, VEC> s{i}[NV];")
    if per_row:
        e.w("#pragma unroll")
        e.w("  for (int k = 0; k < NV; ++k) {")
        e.w("    const int j = tm.slot(k);")
        e.w("    if (rok && j < NVEC) {")
        for i in per_row:
            opd = sk.operands[i]
            ct = _ctype(opd.dtype)
            if staged and sk.config.get("bulk"):
                p = staged.index(i)
                load = (f"s{i}[k] = lds_slot16<{ct}, VEC>(sbase + (uint32_t)(st * STAGE_BYTES + "
                        f"OFF{p} + j * 16));")
            elif staged:
                p = staged.index(i)
                load = (f"s{i}[k] = lds_slot16<{ct}, VEC>(lanes + (uint32_t)(st * STAGE_BYTES + "
                        f"({p} * NV + k) * (TPC * RPC) * 16));")
            else:
                hint = _LOAD_HINT[opd.row_map == "full"]
                load = f"s{i}[k] = load_slot<{hint}, {ct}, VEC>(in{i} + j * VEC);"
            if i in masked_only:
                # only the causal softmax reads it: columns above the
                # row's limit are never needed, so they are not loaded
                e.w(f"      if (j * VEC <= mlim{masked_only[i]}) {load}")
            else:
                e.w(f"      {load}")
        e.w("    }")
        e.w("  }")
    if wait_exchange:
        e.w("  cluster_wait();          // peers' exchange barriers are initialised")
    for vid in sorted(materialize):
        e.w(f"  float m{vid}[NV][VEC];")
    mat_ready = set()
    call = 0
    early_zero, skip_lim = (), None        # outputs stored early in their masked slots
    for p in range(sk.passes):
        rs = reds[p]
        e.w(f"  // ---- pass {p}: " + ", ".join(f"{values[r].op}(v{values[r].args[0]})"
                                             for r in rs + smx[p]))
        for r in rs:
            e.w(f"  float v{r} = {_RED_INIT[values[r].op]};")
        targets = set(closures[p])
        to_mat = {m for m, pm in materialize.items() if pm == p and values[m].op != "softmax"}
        causal = None
        if len(smx[p]) == 1 and not rs and not to_mat:
            causal = _causal_softmax_parts(values, smx[p][0], targets)
        if causal is not None:
            full = [o for o in sk.outputs if o.kind == "full"]
            # only where the row's reduction crosses warps (shared memory /
            # cluster rounds that the zero stores can overlap); a one-warp
            # row measured slower with them (bf16 x2048 causal 70.9 -> 75.4 us)
            team = sk.config["tpc"] * sk.config.get("cl", 1)
            if (p == sk.passes - 1 and full and team > 32
                    and all(sk.out_values[o.index] == smx[p][0] for o in full)):
                early_zero = full
                skip_lim = f"mlim{causal[1]}"
            _emit_causal_softmax_pass(e, sk, smx[p][0], causal, targets, prefetch, mat_ready,
                                      early_zero)
        else:
            if smx[p]:
                _emit_softmax_local_max(e, sk, smx[p], targets, prefetch, mat_ready)
            e.w("#pragma unroll")
            e.w("  for (int k = 0; k < NV; ++k) {")
            e.w("    const int j = tm.slot(k);")
            e.w("    if (!(rok && j < NVEC)) continue;")
            _emit_nonprefetched_loads(e, targets, prefetch, "    ")
            e.w("#pragma unroll")
            e.w("    for (int e = 0; e < VEC; ++e) {")
            if any(values[t].op == "mask" for t in targets):
                e.w("      const int col = (int)(j * VEC) + e;")
            for st in e.elem_statements(targets, prefetch, mat_ready, "      "):
                e.w(st)
            for m in sorted(to_mat):
                e.w(f"      m{m}[k][e] = v{m};")
            for v in smx[p]:
                # step 2: exponentials relative to the thread's max, kept in registers
                x = e.leaf(values[v].args[0], True, prefetch, mat_ready, set())
                e.w(f"      {{ const float ev = {_softmax_exp(sk, v, x)}; m{v}[k][e] = ev; ls{v} += ev; }}")
            for r in rs:
                x = e.leaf(values[r].args[0], True, prefetch, mat_ready, set())
                e.w("      " + _RED_COMBINE[values[r].op].format(a=f"v{r}", x=x))
            e.w("    }")
            e.w("  }")
        mat_ready |= to_mat
        for v in smx[p]:
            # step 3: one pair reduction per row; scale = e^(m_thread - M) / S
            e.w(f"  float gm{v} = lm{v}, gs{v} = ls{v};")
            if push:
                e.w(f"  tm.reduce_softmax_push(gm{v}, gs{v}, red_smem, xch, {area(call)}, xph);")
            else:
                e.w(f"  tm.reduce_softmax(gm{v}, gs{v}, red_smem, {area(call)});")
            # (once per thread and row: CUDA's expf for fp32 outputs)
            scale_exp = (f"expf(lm{v} - gm{v})" if sk.precise
                         else f"fast_exp2((lm{v} - gm{v}) * MOLTEN_LOG2E)")
            e.w(f"  const float sc{v} = (gs{v} > 0.0f) ? ((lm{v} == (-INFINITY)) ? 0.0f : "
                f"{scale_exp} / gs{v}) : NAN;")
            call += 1
            mat_ready.add(v)
        by_op = {}
        for r in rs:
            by_op.setdefault(values[r].op, []).append(r)
        for op, group in by_op.items():
            nr = len(group)
            e.w("  {")
            e.w(f"    float red[{nr}] = {{" + ", ".join(f"v{r}" for r in group) + "};")
            if push:
                e.w(f"    tm.reduce_push<{nr}>(red, {_RED_OP[op]}{{}}, red_smem, xch, {area(call)}, xph);")
            else:
                e.w(f"    tm.reduce<{nr}>(red, {_RED_OP[op]}{{}}, red_smem, {area(call)});")
            for i, r in enumerate(group):
                e.w(f"    v{r} = red[{i}];")
            e.w("  }")
            call += 1
        emit_rows_at(p + 1)
    if done_early:
        e.w("  tm.cluster_done_arrive();")
    # ---- final pass: outputs
    fin = set(closures[sk.passes])
    full_outs = [o for o in sk.outputs if o.kind == "full"]

    def output_loop(packer, ind):
        e.w("#pragma unroll")
        e.w(f"{ind}for (int k = 0; k < NV; ++k) {{")
        e.w(f"{ind}  const int j = tm.slot(k);")
        e.w(f"{ind}  if (!(rok && j < NVEC)) continue;")
        if skip_lim:
            e.w(f"{ind}  if (j * VEC > {skip_lim}) continue;         // stored before the reductions")
        _emit_nonprefetched_loads(e, fin, prefetch, ind + "  ")
        for o in full_outs:
            e.w(f"{ind}  float f{o.index}[VEC];")
        e.w("#pragma unroll")
        e.w(f"{ind}  for (int e = 0; e < VEC; ++e) {{")
        if any(values[t].op == "mask" for t in fin):
            e.w(f"{ind}    const int col = (int)(j * VEC) + e;")
        for st in e.elem_statements(fin, prefetch, mat_ready, ind + "    "):
            e.w(st)
        for o in full_outs:
            src = e.leaf(sk.out_values[o.index], True, prefetch, mat_ready, set())
            e.w(f"{ind}    f{o.index}[e] = {src};")
        e.w(f"{ind}  }}")
        for o in full_outs:
            ct = _ctype(o.dtype)
            e.w(f"{ind}  Slot<{ct}, VEC> o{o.index}; {packer}<{ct}, VEC>(o{o.index}, f{o.index});")
            e.w(f"{ind}  store_slot<kStoreDefault, {ct}, VEC>(out{o.index} + j * VEC, o{o.index});")
        e.w(f"{ind}}}")

    if full_outs:
        e.w("  // ---- final pass: outputs")
        output_loop("pack_slot", "  ")
    for o in sk.outputs:
        if o.kind == "row":
            src = e.leaf(sk.out_values[o.index], False, prefetch, set(), set())
            e.w(f"  if (rok && tm.t == 0 && tm.rank == 0) store_scalar(out{o.index}, {src});")


def _emit_nonprefetched_loads(e: _Emitter, targets, prefetch, indent):
    sk = e.sk
    used = set()
    for t in targets:
        v = e.values[t]
        if v.op == "load" and v.kind == "elem" and v.attrs["operand"] not in prefetch:
            used.add(v.attrs["operand"])
        for a in v.args:
            va = e.values[a]
            if va.op == "load" and va.kind == "elem" and va.attrs["operand"] not in prefetch:
                used.add(va.attrs["operand"])
    for i in sorted(used):
        opd = sk.operands[i]
        ct = _ctype(opd.dtype)
        e.w(f"{indent}const Slot<{ct}, VEC> sl{i} = load_slot<kLoadDefault, {ct}, VEC>(in{i} + j * VEC);")


def emit_ew(sk: SubKernel, name: str) -> str:
    """Pure elementwise kernel: grid.x = column tiles, grid.y strides over
    blocks of RPC * UPT rows; per-column operands are loaded once per thread
    and reused for every row it visits."""
    e = _Emitter(sk, name)
    cfg = sk.config
    VEC, NV, TPC, RPC, UPT = cfg["vec"], cfg["nv"], cfg["tpc"], cfg["rpc"], cfg["upt"]
    values = sk.values
    needed = e.needed
    e.header("elementwise")
    e.w("using namespace molten;")
    e.w("")
    minb = cfg.get("min_blocks", 0)
    lb = f"{TPC * RPC}, {minb}" if minb else f"{TPC * RPC}"
    e.w(f"extern \"C\" __global__ void __launch_bounds__({lb}) "
        f"{name}(const __grid_constant__ RowArgs args) {{")
    e.w("  pdl_enter();")
    e.w(f"  constexpr int VEC = {VEC}, NV = {NV}, TPC = {TPC}, RPC = {RPC}, UPT = {UPT};")
    e.w(f"  constexpr long long COLS = {sk.cols}LL, NVEC = {cfg['nvec']}LL;")
    e.w("  const int t = threadIdx.x % TPC, team = threadIdx.x / TPC;")
    e.w("  const long long tile0 = (long long)blockIdx.x * (TPC * NV);")
    # per-column operands: hoisted loads
    col_ops = [o for o in sk.operands if o.last == "vec" and o.row_map == "zero"]
    row_ops = [o for o in sk.operands if o.last == "vec" and o.row_map != "zero"]
    bc_ops = [o for o in sk.operands if o.last == "bcast"]
    for o in col_ops:
        ct = _ctype(o.dtype)
        e.w(f"  Slot<{ct}, VEC> c{o.index}[NV];")
        e.w("#pragma unroll")
        e.w("  for (int k = 0; k < NV; ++k) {")
        e.w("    const long long j = tile0 + t + (long long)k * TPC;")
        e.w(f"    if (j < NVEC) c{o.index}[k] = load_slot<kLoadDefault, {ct}, VEC>"
            f"(static_cast<const {ct}*>(args.in[{o.index}]) + j * VEC);")
        e.w("  }")
    e.w("  for (long long rb = blockIdx.y; rb * (RPC * UPT) < args.rows; rb += gridDim.y) {")
    # row loads for all UPT rows first
    for o in row_ops:
        ct = _ctype(o.dtype)
        e.w(f"    Slot<{ct}, VEC> s{o.index}[UPT][NV];")
    e.w("#pragma unroll")
    e.w("    for (int u = 0; u < UPT; ++u) {")
    e.w("      const long long lrow = rb * (RPC * UPT) + (long long)u * RPC + team;")
    e.w("      const long long grow = args.row_offset + lrow;")
    e.w("      (void)grow;")
    e.w("      if (lrow >= args.rows) continue;")
    e.w("#pragma unroll")
    e.w("      for (int k = 0; k < NV; ++k) {")
    e.w("        const long long j = tile0 + t + (long long)k * TPC;")
    e.w("        if (j >= NVEC) continue;")
    for o in row_ops:
        ct = _ctype(o.dtype)
        idx = _row_index_expr(o, "lrow", "grow")
        hint = _LOAD_HINT[o.row_map == "full"]
        e.w(f"        s{o.index}[u][k] = load_slot<{hint}, {ct}, VEC>(static_cast<const {ct}*>"
            f"(args.in[{o.index}]) + {idx} * COLS + j * VEC);")
    e.w("      }")
    e.w("    }")
    e.w("#pragma unroll")
    e.w("    for (int u = 0; u < UPT; ++u) {")
    e.w("      const long long lrow = rb * (RPC * UPT) + (long long)u * RPC + team;")
    e.w("      const long long grow = args.row_offset + lrow;")
    e.w("      (void)grow;")
    e.w("      if (lrow >= args.rows) continue;")
    for o in bc_ops:
        ct = _ctype(o.dtype)
        idx = _row_index_expr(o, "lrow", "grow")
        for vid in sorted(needed):
            v = values[vid]
            if v.op == "load" and v.attrs["operand"] == o.index:
                e.w(f"      const float v{vid} = load_scalar(static_cast<const {ct}*>"
                    f"(args.in[{o.index}]) + {idx});")
    for vid in sorted(needed):
        v = values[vid]
        if v.op == "mask":
            period = _mask_period(v, sk.cols)
            off = int(v.attrs.get("offset", 0))
            e.w(f"      const int mlim{vid} = clamp_col_limit((grow % {period}LL) + ({off}LL));")
    for vid in sorted(needed):
        v = values[vid]
        if v.kind in ("row", "const") and v.op not in ("load", "const"):
            args = [_ew_leaf(e, a) for a in v.args]
            e.w(f"      const float v{vid} = {value_expr(v, args, True)};")
    e.w("#pragma unroll")
    e.w("      for (int k = 0; k < NV; ++k) {")
    e.w("        const long long j = tile0 + t + (long long)k * TPC;")
    e.w("        if (j >= NVEC) continue;")
    for o in sk.outputs:
        e.w(f"        float f{o.index}[VEC];")
    e.w("#pragma unroll")
    e.w("        for (int e = 0; e < VEC; ++e) {")
    if any(values[t].op == "mask" for t in needed):
        e.w("          const int col = (int)(j * VEC) + e;")
    for vid in sorted(needed):
        v = values[vid]
        if v.kind != "elem" or v.op in ("load",):
            continue
        if v.op == "mask":
            e.w(f"          const float v{vid} = (col > mlim{vid}) ? (-INFINITY) : 0.0f;")
            continue
        args = [_ew_leaf(e, a) for a in v.args]
        e.w(f"          const float v{vid} = {value_expr(v, args, sk.precise)};")
    for o in sk.outputs:
        e.w(f"          f{o.index}[e] = {_ew_leaf(e, sk.out_values[o.index])};")
    e.w("        }")
    for o in sk.outputs:
        ct = _ctype(o.dtype)
        e.w(f"        Slot<{ct}, VEC> o{o.index}; pack_slot<{ct}, VEC>(o{o.index}, f{o.index});")
        e.w(f"        store_slot<kStoreDefault, {ct}, VEC>(static_cast<{ct}*>(args.out[{o.index}]) "
            f"+ lrow * COLS + j * VEC, o{o.index});")
    e.w("      }")
    e.w("    }")
    e.w("  }")
    e.w("}")
    return "\n".join(e.lines) + "\n"


def _ew_leaf(e: _Emitter, vid: int) -> str:
    v = e.values[vid]
    if v.kind == "const" and v.op == "const":
        return c_float(v.attrs["value"])
    if v.op == "load" and v.kind == "elem":
        o = e.sk.operands[v.attrs["operand"]]
        if o.row_map == "zero":
            return f"to_f32(c{o.index}[k].v[e])"
        return f"to_f32(s{o.index}[u][k].v[e])"
    return f"v{vid}"


def emit_row_tma(sk: SubKernel, name: str) -> str:
    """Row kernel on the TMA-staged engine (molten/row_tma.cuh): rows of the
    row-indexed operands stream through a shared-memory ring; one consumer
    warp per row; reductions are warp shuffles."""
    cfg = sk.config
    VEC, NV, NC, ST = cfg["vec"], cfg["nv"], cfg["nc"], cfg["stages"]
    TW = int(cfg.get("tw", 1))                     # warps per row (a team)
    staged = list(cfg["staged"])                   # operand indices, stage order
    offs = dict(zip(staged, cfg["stage_offsets"]))
    consts = list(cfg.get("consts", ()))           # per-column operands, copied once
    coffs = dict(zip(consts, cfg.get("const_offsets", ())))
    CB = cfg.get("const_bytes", 0)
    values = sk.values
    needed = set(cfg["needed"])
    materialize = {int(v): int(p) for v, p in cfg["materialize"]}
    closures = pass_closures(values, sk, needed, materialize)
    reds = {p: [] for p in range(sk.passes)}
    for vid in sorted(needed):
        v = values[vid]
        if v.op in ("rsum", "rmax", "rmin"):
            reds[v.avail - 1].append(vid)
    L = []
    w = L.append
    w(f"// Molten sm_100a TMA-staged row kernel: {name}")
    w(f"// cols = {sk.cols}; inputs: " + ", ".join(
        f"{o.name}[{o.dtype} {o.last}/{o.row_map}]" for o in sk.operands))
    w("#include \"molten/row_tma.cuh\"")
    w("")
    w("using namespace molten;")
    w("")
    # largest number of values one team reduction combines
    nred = max([len([r for r in reds[p] if values[r].op == op])
                for p in reds for op in ("rsum", "rmax", "rmin")] + [1])
    w(f"extern \"C\" __global__ void __launch_bounds__({32 * (NC * TW + 1)}, 1) "
      f"{name}(const __grid_constant__ RowArgs args) {{")
    w("  pdl_enter();")
    w(f"  constexpr int VEC = {VEC}, NV = {NV}, NC = {NC}, STAGES = {ST}, "
      f"STAGE_BYTES = {cfg['stage_bytes']};")
    if TW > 1:
        w(f"  constexpr int TW = {TW}, NRED = {nred};")
    w(f"  constexpr long long COLS = {sk.cols}LL, NVEC = {cfg['nvec']}LL;")
    w(f"  constexpr uint32_t ROW_BYTES = {cfg['row_bytes']}u;")
    w("  extern __shared__ __align__(128) uint8_t smem_raw[];")
    w(f"  const auto ring = row_ring_carve<STAGES, STAGE_BYTES, {CB}>(smem_raw);")
    if TW > 1:
        w("  __shared__ float team_red[NC * 2 * TW * NRED];")
        w("  __shared__ __align__(8) uint64_t team_bar[NC * 2];")
        w("  row_ring_init(ring, STAGES, TW);")
        w("  team_bars_init(smem_u32(team_bar), NC, TW);")
    else:
        w("  row_ring_init(ring, STAGES);")
    w("  __syncthreads();")
    w("  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;")
    w("  const long long G = gridDim.x;")
    w("  const long long nloc = args.rows > (long long)blockIdx.x ? "
      "(args.rows - 1 - blockIdx.x) / G + 1 : 0;")
    w("  if (warp == 0) {")
    w("    if (lane == 0) {")
    w("      long long issued = 0;")
    if consts:
        w(f"      mbar_expect_tx(ring.consts_full(), {sum(sk.cols * DTYPE_SIZE_OF[sk.operands[i].dtype] for i in consts)}u);")
        for i in consts:
            o = sk.operands[i]
            ct = _ctype(o.dtype)
            w(f"      bulk_g2s(ring.consts() + {coffs[i]}u, args.in[{i}], "
              f"{sk.cols * DTYPE_SIZE_OF[o.dtype]}u, ring.consts_full());")
    w("      for (long long j = 0; j < nloc && !*ring.abort_flag; ++j) {")
    w("        const int s = (int)(j % STAGES);")
    w("        const uint32_t ph = (uint32_t)((j / STAGES) & 1);")
    w("        if (!mbar_wait(ring.empty(s), ph ^ 1u)) {")
    w("          row_ring_fail(ring.abort_flag, args.status, kRowTimeoutEmpty);")
    w("          break;")
    w("        }")
    w("        const long long lrow = (long long)blockIdx.x + j * G;")
    w("        const long long grow = args.row_offset + lrow;")
    w("        (void)grow;")
    w("        mbar_expect_tx(ring.full(s), ROW_BYTES);")
    for i in staged:
        o = sk.operands[i]
        ct = _ctype(o.dtype)
        idx = _row_index_expr(o, "lrow", "grow")
        w(f"        bulk_g2s(ring.stage(s) + {offs[i]}u, "
          f"static_cast<const {ct}*>(args.in[{i}]) + {idx} * COLS, "
          f"{sk.cols * DTYPE_SIZE_OF[o.dtype]}u, ring.full(s));")
    w("        ++issued;")
    w("      }")
    w("      if (*ring.abort_flag) {")
    w("        for (long long i = issued - 1; i >= 0 && i >= issued - STAGES; --i) {")
    w("          if (!mbar_wait(ring.full((int)(i % STAGES)), (uint32_t)((i / STAGES) & 1)) && args.status)")
    w("            atomicOr(args.status, kRowTimeoutDrain);")
    w("        }")
    w("      }")
    w("    }")
    w("  } else {")
    if consts:
        w("    if (!__all_sync(0xffffffffu, mbar_wait(ring.consts_full(), 0u) ? 1 : 0)) {")
        w("      if (lane == 0) row_ring_fail(ring.abort_flag, args.status, kRowTimeoutFull);")
        w("      return;")
        w("    }")
        w("    const uint32_t cb = ring.consts();")
    if TW > 1:
        w("    const int team = (warp - 1) / TW, tw = (warp - 1) % TW, tl = tw * 32 + lane;")
        w("    TeamRed tr{team_red + team * (2 * TW * NRED), smem_u32(team_bar) + 16u * team, 0u};")
        w("    for (long long j = team; j < nloc; j += NC) {")
    else:
        w("    for (long long j = warp - 1; j < nloc; j += NC) {")
    w("      const int s = (int)(j % STAGES);")
    w("      const bool got = mbar_wait(ring.full(s), (uint32_t)((j / STAGES) & 1));")
    w("      if (!__all_sync(0xffffffffu, got ? 1 : 0)) {")
    w("        if (lane == 0) row_ring_fail(ring.abort_flag, args.status, kRowTimeoutFull);")
    w("        break;")
    w("      }")
    w("      const uint32_t sb = ring.stage(s);")
    w("      (void)sb;")
    w("      const long long lrow = (long long)blockIdx.x + j * G;")
    w("      const long long grow = args.row_offset + lrow;")
    w("      (void)grow;")
    # non-staged operand pointers and outputs
    for o in sk.operands:
        if o.index in staged or o.index in consts:
            continue
        ct = _ctype(o.dtype)
        idx = _row_index_expr(o, "lrow", "grow")
        stride = "COLS" if o.last == "vec" else "1LL"
        w(f"      const {ct}* __restrict__ in{o.index} = static_cast<const {ct}*>(args.in[{o.index}]) "
          f"+ {idx} * {stride};")
    for out in sk.outputs:
        ct = _ctype(out.dtype)
        stride = "COLS" if out.kind == "full" else "1LL"
        w(f"      {ct}* __restrict__ out{out.index} = static_cast<{ct}*>(args.out[{out.index}]) "
          f"+ lrow * {stride};")
    for vid in sorted(needed):
        v = values[vid]
        if v.op == "load" and v.kind == "row":
            w(f"      const float v{vid} = load_scalar(in{v.attrs['operand']});")
        if v.op == "mask":
            period = _mask_period(v, sk.cols)
            off = int(v.attrs.get("offset", 0))
            w(f"      const int mlim{vid} = clamp_col_limit((grow % {period}LL) + ({off}LL));")
    emitted = set()

    def rows_at(p):
        for vid in sorted(needed):
            v = values[vid]
            if v.kind in ("row", "const") and v.avail == p and vid not in emitted \
                    and v.op not in ("load", "const", "rsum", "rmax", "rmin"):
                args = [_tma_leaf(sk, a, staged, set()) for a in v.args]
                w(f"      const float v{vid} = {value_expr(v, args, True)};")
                emitted.add(vid)

    rows_at(0)
    for vid in sorted(materialize):
        w(f"      float m{vid}[NV][VEC];")
    mat_ready = set()

    def slot_loop(targets, body_extra, tail=None, outs=()):
        w("#pragma unroll")
        w("      for (int k = 0; k < NV; ++k) {")
        if TW > 1:
            w("        const long long j = tl + 32LL * TW * k;")
        else:
            w("        const long long j = lane + 32LL * k;")
        w("        if (j >= NVEC) break;")
        used_staged, used_glob = set(), set()
        for t in targets:
            vt = values[t]
            for x in [t] + list(vt.args):
                vx = values[x]
                if vx.op == "load" and vx.kind == "elem" and x not in mat_ready:
                    (used_staged if vx.attrs["operand"] in staged else used_glob).add(vx.attrs["operand"])
        for i in sorted(used_staged):
            o = sk.operands[i]
            ct = _ctype(o.dtype)
            off = offs[i]
            w(f"        const Slot<{ct}, VEC> st{i} = lds_slot<{ct}, VEC>(sb + {off}u + "
              f"(uint32_t)(j * (VEC * {DTYPE_SIZE_OF[o.dtype]})));")
        for i in sorted(used_glob):
            o = sk.operands[i]
            ct = _ctype(o.dtype)
            if i in consts:
                w(f"        const Slot<{ct}, VEC> sl{i} = lds_slot<{ct}, VEC>(cb + {coffs[i]}u + "
                  f"(uint32_t)(j * (VEC * {DTYPE_SIZE_OF[o.dtype]})));")
            else:
                w(f"        const Slot<{ct}, VEC> sl{i} = load_slot<kLoadDefault, {ct}, VEC>(in{i} + j * VEC);")
        for o in outs:
            w(f"        float f{o.index}[VEC];")
        w("#pragma unroll")
        w("        for (int e = 0; e < VEC; ++e) {")
        if any(values[t].op == "mask" for t in targets):
            w("          const int col = (int)(j * VEC) + e;")
        for vid in sorted(targets):
            v = values[vid]
            if v.kind != "elem" or vid in mat_ready or v.op == "load":
                continue
            if v.op == "mask":
                w(f"          const float v{vid} = (col > mlim{vid}) ? (-INFINITY) : 0.0f;")
                continue
            args = [_tma_leaf(sk, a, staged, mat_ready) for a in v.args]
            w(f"          const float v{vid} = {value_expr(v, args, sk.precise)};")
        body_extra()
        w("        }")
        if tail:
            tail()
        w("      }")

    for p in range(sk.passes):
        rs = reds[p]
        for r in rs:
            w(f"      float v{r} = {_RED_INIT[values[r].op]};")
        targets = set(closures[p])
        to_mat = {m for m, pm in materialize.items() if pm == p}

        def extra(rs=rs, to_mat=to_mat):
            for m in sorted(to_mat):
                w(f"          m{m}[k][e] = v{m};")
            for r in rs:
                x = _tma_leaf(sk, values[r].args[0], staged, mat_ready)
                w("          " + _RED_COMBINE[values[r].op].format(a=f"v{r}", x=x))

        slot_loop(targets, extra)
        mat_ready |= to_mat
        by_op = {}
        for r in rs:
            by_op.setdefault(values[r].op, []).append(r)
        for op, grp in by_op.items():
            fn = {"rsum": "warp_allreduce_sum", "rmax": "warp_allreduce_max",
                  "rmin": "warp_allreduce_min"}[op]
            w("      {")
            w(f"        float red[{len(grp)}] = {{" + ", ".join(f"v{r}" for r in grp) + "};")
            if TW > 1:
                opn = {"rsum": 0, "rmax": 1, "rmin": 2}[op]
                w(f"        if (!team_allreduce<{opn}, {len(grp)}, TW>(red, tr, tw, lane)) {{")
                w("          if (lane == 0) row_ring_fail(ring.abort_flag, args.status, kRowTimeoutTeam);")
                w("          break;")
                w("        }")
            else:
                w(f"        {fn}<{len(grp)}>(red);")
            for i, r in enumerate(grp):
                w(f"        v{r} = red[{i}];")
            w("      }")
        rows_at(p + 1)
    fin = set(closures[sk.passes])
    full_outs = [o for o in sk.outputs if o.kind == "full"]

    def fin_extra():
        for o in full_outs:
            w(f"          f{o.index}[e] = {_tma_leaf(sk, sk.out_values[o.index], staged, mat_ready)};")

    def fin_tail():
        for o in full_outs:
            ct = _ctype(o.dtype)
            w(f"        Slot<{ct}, VEC> o{o.index}; pack_slot<{ct}, VEC>(o{o.index}, f{o.index});")
            w(f"        store_slot<kStoreDefault, {ct}, VEC>(out{o.index} + j * VEC, o{o.index});")

    if full_outs:
        slot_loop(fin, fin_extra, fin_tail, full_outs)
    for o in sk.outputs:
        if o.kind == "row":
            w(f"      if ({'tl' if TW > 1 else 'lane'} == 0) store_scalar(out{o.index}, "
              f"{_tma_leaf(sk, sk.out_values[o.index], staged, mat_ready)});")
    w("      __syncwarp();")
    w("      if (lane == 0) mbar_arrive(ring.empty(s));")
    w("      if (__any_sync(0xffffffffu, *ring.abort_flag ? 1 : 0)) break;")
    w("    }")
    w("  }")
    w("}")
    return "\n".join(L) + "\n"


DTYPE_SIZE_OF = {"float32": 4, "bfloat16": 2, "float16": 2}


def _tma_leaf(sk: SubKernel, vid: int, staged, mat_ready) -> str:
    v = sk.values[vid]
    if v.kind == "const" and v.op == "const":
        return c_float(v.attrs["value"])
    if v.kind in ("row", "const"):
        return f"v{vid}"
    if vid in mat_ready:
        return f"m{vid}[k][e]"
    if v.op == "load":
        i = v.attrs["operand"]
        return f"to_f32(st{i}.v[e])" if i in staged else f"to_f32(sl{i}.v[e])"
    return f"v{vid}"


def _closure_within(values, root, allowed) -> set:
    """Elem values among ``allowed`` that ``root`` depends on (inclusive)."""
    out, stack = set(), [root]
    while stack:
        v = stack.pop()
        if v in out or v not in allowed:
            continue
        out.add(v)
        stack.extend(values[v].args)
    return out


def _softmax_exp(sk: SubKernel, v: int, x: str) -> str:
    """e^(x - m_thread) on the EX2 unit.  16-bit outputs: one FFMA + EX2,
    2^(x log2e - m log2e).  fp32 outputs: the difference first, then one
    multiply and EX2, 2^((x - m) log2e): the argument t = (x - m) log2e is
    then off by at most |t| 2^-23 (two roundings), so e^(x - m) is within
    |t| 2^-23 ln 2 + 2 ulp of its value -- below 1.7e-6 relative where
    e^(x - m) > e^-14 (and below the 1e-6 * max absolute term of the fp32
    parity bar elsewhere); results below 2^-126 flush to zero.  (expf was
    7% slower on fp32 4096 x 32768 rows and 3% on causal rows, at 1.0e-6
    measured relative difference.)"""
    if sk.precise:
        return f"fast_exp2(({x} - lz{v}) * MOLTEN_LOG2E)"
    return f"fast_exp2(fmaf({x}, MOLTEN_LOG2E, lzs{v}))"


def _emit_softmax_thread_max_decl(e: _Emitter, sk: SubKernel, vs):
    for v in vs:
        e.w(f"  float lm{v} = (-INFINITY), ls{v} = 0.0f;")


def _emit_softmax_max_tail(e: _Emitter, sk: SubKernel, vs):
    for v in vs:
        e.w(f"  const float lz{v} = (lm{v} == (-INFINITY)) ? 0.0f : lm{v};")
        if not sk.precise:
            e.w(f"  const float lzs{v} = -lz{v} * MOLTEN_LOG2E;")


def _emit_softmax_local_max(e: _Emitter, sk: SubKernel, vs, targets, prefetch, mat_ready):
    """Online softmax, step 1: this thread's max of each softmax input."""
    values = sk.values
    VEC = sk.config["vec"]
    _emit_softmax_thread_max_decl(e, sk, vs)
    xs_targets = set()
    for v in vs:
        xs_targets |= _closure_within(values, values[v].args[0], targets)
    e.w("#pragma unroll")
    e.w("  for (int k = 0; k < NV; ++k) {")
    e.w("    const int j = tm.slot(k);")
    e.w("    if (!(rok && j < NVEC)) continue;")
    packed = [v for v in vs if _packed_max_operand(sk, values[values[v].args[0]], prefetch, VEC)]
    for v in packed:
        i = values[values[v].args[0]].attrs["operand"]
        e.w(f"    lm{v} = slot_max16(s{i}[k], lm{v});      // two elements per max")
    rest = [v for v in vs if v not in packed]
    if rest:
        _emit_nonprefetched_loads(e, xs_targets, prefetch, "    ")
        e.w("#pragma unroll")
        e.w("    for (int e = 0; e < VEC; ++e) {")
        if any(values[t].op == "mask" for t in xs_targets):
            e.w("      const int col = (int)(j * VEC) + e;")
        for st in e.elem_statements(xs_targets, prefetch, mat_ready, "      "):
            e.w(st)
        for v in rest:
            x = e.leaf(values[v].args[0], True, prefetch, mat_ready, set())
            e.w(f"      lm{v} = fmaxf(lm{v}, {x});")
        e.w("    }")
    e.w("  }")
    _emit_softmax_max_tail(e, sk, vs)


def _causal_softmax_parts(values, v: int, targets):
    """(a, mask) when the softmax input is ADD(a, causal mask) and a does not
    depend on the mask; None otherwise."""
    x = values[values[v].args[0]]
    if x.op != "add":
        return None
    a, b = x.args
    if values[b].op == "mask" and values[a].op != "mask":
        pair = (a, b)
    elif values[a].op == "mask" and values[b].op != "mask":
        pair = (b, a)
    else:
        return None
    if pair[1] in _closure_within(values, pair[0], set(range(len(values)))):
        return None
    return pair


def _emit_causal_softmax_pass(e: _Emitter, sk: SubKernel, v: int, parts, targets, prefetch,
                              mat_ready, early_zero=()):
    """Softmax of a + causal mask, classifying each slot once: columns
    c0 .. c0+VEC-1 all above the row's limit (exponentials are 0, nothing is
    computed), all at or below it (no mask arithmetic), or straddling it (the
    one boundary slot of the row, checked per element).  ``early_zero``:
    outputs that are this softmax itself -- their fully masked slots are 0
    whatever the row's statistics, so they are stored here, before the
    row's reductions, and the output pass skips them."""
    values = sk.values
    VEC = sk.config["vec"]
    a, mk = parts
    a_targets = _closure_within(values, a, targets)
    lim = f"mlim{mk}"
    # bulk zero tail: the row's fully masked slots (columns from the first
    # slot above the limit to the end) are written by the TMA engine from a
    # shared zero buffer, issued by the row's one team leader; threads skip
    # them.  Needs 16-byte slots covering the row exactly and a 16-byte
    # aligned output row (checked per row; otherwise the threads store them)
    zt = None
    if (early_zero and getattr(e, "zero_tail", False) and sk.cols % VEC == 0
            and all(DTYPE_SIZE_OF[o.dtype] * VEC == 16 for o in early_zero)):
        zt = f"zt{v}"
        align = " | ".join(f"reinterpret_cast<uintptr_t>(out{o.index})" for o in early_zero)
        e.w(f"  const bool {zt} = rok && ((({align}) & 15u) == 0);")
        e.w(f"  if ({zt} && threadIdx.x == 0) {{")
        e.w(f"    const long long z0 = ({lim} < 0) ? 0LL : ((long long)({lim} / VEC) + 1) * VEC;")
        for o in early_zero:
            e.w(f"    if (z0 < COLS) bulk_zero_tail(out{o.index} + z0, (COLS - z0) * "
                f"(long long)sizeof(*out{o.index}), zsrc, ZBYTES);")
        e.w("  }")
        e.zero_tail_used = True
    _emit_softmax_thread_max_decl(e, sk, [v])
    packed = _packed_max_operand(sk, values[a], prefetch, VEC)

    def a_stmts(indent):
        for st in e.elem_statements(a_targets, prefetch, mat_ready, indent):
            e.w(st)

    x = e.leaf(a, True, prefetch, mat_ready, set())
    # step 1: thread max over the visible columns
    e.w("#pragma unroll")
    e.w("  for (int k = 0; k < NV; ++k) {")
    e.w("    const int j = tm.slot(k);")
    e.w("    if (!(rok && j < NVEC)) continue;")
    e.w("    const int c0 = j * VEC;")
    e.w(f"    if (c0 > {lim}) continue;                       // slot fully masked")
    _emit_nonprefetched_loads(e, a_targets, prefetch, "    ")
    if packed:
        i = values[a].attrs["operand"]
        e.w(f"    if (c0 + VEC - 1 <= {lim}) {{ lm{v} = slot_max16(s{i}[k], lm{v}); continue; }}")
    else:
        e.w(f"    if (c0 + VEC - 1 <= {lim}) {{")
        e.w("#pragma unroll")
        e.w("      for (int e = 0; e < VEC; ++e) {")
        a_stmts("        ")
        e.w(f"        lm{v} = fmaxf(lm{v}, {x});")
        e.w("      }")
        e.w("      continue;")
        e.w("    }")
    e.w("#pragma unroll")
    e.w("    for (int e = 0; e < VEC; ++e) {")
    a_stmts("      ")
    e.w(f"      if (c0 + e <= {lim}) lm{v} = fmaxf(lm{v}, {x});")
    e.w("    }")
    e.w("  }")
    _emit_softmax_max_tail(e, sk, [v])
    # step 2: exponentials of the visible columns, zeros above the limit
    ex = _softmax_exp(sk, v, x)
    e.w("#pragma unroll")
    e.w("  for (int k = 0; k < NV; ++k) {")
    e.w("    const int j = tm.slot(k);")
    e.w("    if (!(rok && j < NVEC)) continue;")
    e.w("    const int c0 = j * VEC;")
    e.w(f"    if (c0 > {lim}) {{")
    e.w("#pragma unroll")
    e.w(f"      for (int e = 0; e < VEC; ++e) m{v}[k][e] = 0.0f;")
    for o in early_zero:
        store = f"store_zero_slot<kStoreDefault, {_ctype(o.dtype)}, VEC>(out{o.index} + j * VEC);"
        e.w(f"      if (!{zt}) {store}" if zt else f"      {store}")
    e.w("      continue;")
    e.w("    }")
    _emit_nonprefetched_loads(e, a_targets, prefetch, "    ")
    e.w(f"    const bool whole = c0 + VEC - 1 <= {lim};")
    e.w("#pragma unroll")
    e.w("    for (int e = 0; e < VEC; ++e) {")
    a_stmts("      ")
    e.w(f"      const float ev = (whole || c0 + e <= {lim}) ? {ex} : 0.0f;")
    e.w(f"      m{v}[k][e] = ev;")
    e.w(f"      ls{v} += ev;")
    e.w("    }")
    e.w("  }")


def _packed_max_operand(sk: SubKernel, xv: Value, prefetch, vec: int) -> bool:
    """The softmax input is a prefetched 16-bit operand itself: its row max
    can be taken on packed pairs of raw elements."""
    if xv.op != "load" or xv.kind != "elem":
        return False
    o = sk.operands[xv.attrs["operand"]]
    return o.index in prefetch and o.dtype in ("bfloat16", "float16") and vec % 2 == 0


def smx_of(values, needed, passes):
    out = {p: [] for p in range(passes)}
    for vid in sorted(needed):
        if values[vid].op == "softmax":
            out[values[vid].avail - 1].append(vid)
    return out


def _causal_masked_only_operands(sk: SubKernel, closures, reds, smx, materialize) -> dict:
    """Prefetched operands read only as the `a` of a causal softmax(a + mask):
    {operand index: mask value id}.  Their fully masked slots are skipped."""
    values = sk.values
    out = {}
    for p, vs in smx.items():
        to_mat = {m for m, pm in materialize.items() if pm == p and values[m].op != "softmax"}
        if len(vs) != 1 or reds.get(p) or to_mat:
            continue
        parts = _causal_softmax_parts(values, vs[0], closures[p])
        if parts is None:
            continue
        a, mk = parts
        av = values[a]
        if av.op != "load":
            continue
        i = av.attrs["operand"]
        used_elsewhere = any(a in closures[q] for q in closures if q != p)
        if not used_elsewhere:
            out[i] = mk
    return out
