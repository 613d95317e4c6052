// Fused attention scores on sm_100a: P = softmax(Q K^T * scale) over the
// last dim, for a stack of `batch` independent problems (heads) with
// Q [batch*m, d] and K [batch*n, d] row-major (K is read K-major: no
// transpose is materialised), P [batch*m, n] in bf16 or fp16.
//
// One CTA owns work items (head h, 128-row block of Q) in a persistent loop
// and runs two passes over the item's n columns, recomputing Q K^T on the
// tensor cores instead of storing fp32 scores:
//
//   pass 0   per row (one epilogue thread = one row = one TMEM lane, per
//            column part): online max of the raw scores s and sum of
//            2^((s - max) * C2), C2 = scale * log2(e) > 0;
//   pass 1   p = 2^(s * C2 - (max * C2 + log2(sum))), rounded once and stored.
//
//   warp 0      TMA producer: the item's Q tile (d/64 boxes {64, 128}) into
//               a resident area, then per pass and column block the K tiles
//               ({64, BN} boxes of K's rows) through a STAGES-deep ring;
//   warp 1      TMEM owner + MMA issuer (tcgen05.mma.cta_group::1.kind::f16,
//               fp32 accumulators in 2 or 4 TMEM buffers of BN columns);
//   warps 4..   epilogue: EPI_WARPS / 4 warps per TMEM lane quarter
//               (warp % 4), in GROUPS groups that take alternate tiles (so
//               group g always reads accumulator buffer g: one group's TMEM
//               loads overlap the other's arithmetic instead of every warp
//               waiting on the same load), each warp taking one part of its
//               tiles' columns, up to 64 columns per load; at the end of
//               pass 0 the warps of a quarter merge their per-row (max, sum)
//               through shared memory, in the same order in every warp.  Pass-1 rows
//               go to HBM either through a per-warp staging tile and a TMA
//               store (32 rows x 32 or 64 columns, swizzled: conflict-free
//               row-per-thread writes, full-line global writes) or, where a
//               box could cross into another head's rows, by direct stores.
//
// HBM sees Q and K about twice (L2 holds K across a head's row blocks) and
// P once; the fp32 score matrix of the two-kernel form never exists.  Every
// mbarrier wait is bounded; on timeout the CTA sets a status bit, stops,
// drains its copies, frees TMEM and returns.
#pragma once

#include "molten/gemm_sm100.cuh"

namespace molten {

struct alignas(64) AttnArgs {
  CUtensorMap tmap_q;              // Q [batch*m, d], box {64, 128}, 128B swizzle
  CUtensorMap tmap_k;              // K [batch*n, d], box {64, BN}, 128B swizzle
  CUtensorMap tmap_p;              // P [batch*m, n], box {LCOLS, 32}, 2*LCOLS-byte swizzle
  void* out;                       // P
  long long m, n, d;               // one problem: P[m, n] = softmax(Q[m, d] K[n, d]^T)
  long long row_offset;            // unused (no row-dependent terms)
  int* status;                     // error bits (may be null)
  int batch;                       // stacked problems (0 or 1: one)
};

enum AttnStatus { kAttnTimeout = 512 };

template <int BN_, int DCH_, int STAGES_, int EPI_WARPS_ = 8, int GROUPS_ = 1>
struct AttnLayout {
  static constexpr int BM = 128, BN = BN_, DCH = DCH_, STAGES = STAGES_;
  static constexpr int EPI_WARP0 = 4, EPI_WARPS = EPI_WARPS_, GROUPS = GROUPS_;
  static constexpr int SLOTS = EPI_WARPS / 4;               // warps per TMEM lane quarter
  static_assert(GROUPS == 1 || GROUPS == 2, "one group, or two taking alternate tiles");
  static_assert(SLOTS % GROUPS == 0, "whole groups per quarter");
  static constexpr int PARTS = SLOTS / GROUPS;              // column parts of one tile
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, a multiple of 64");
  static_assert(DCH >= 1 && DCH <= 4, "d must be at most 256");
  static_assert(EPI_WARPS % 4 == 0 && EPI_WARPS >= 4 && EPI_WARPS <= 16, "4, 8, 12 or 16 epilogue warps");
  static_assert((BN / 32) % PARTS == 0, "each column part holds whole 32-column chunks");
  static constexpr int RELEASERS = EPI_WARPS / GROUPS;      // warps that read one buffer
  static constexpr int PCOLS = BN / PARTS;                  // columns per part and tile
  static constexpr int LCOLS = PCOLS % 64 == 0 ? 64 : 32;   // columns per TMEM load and store
  static_assert(PCOLS % LCOLS == 0, "a part is whole loads");
  static constexpr int Q_CHUNK = BM * 128;                  // {64, 128} box, 128-byte rows
  static constexpr int Q_BYTES = DCH * Q_CHUNK;
  static constexpr int STAGE_BYTES = BN * 128;              // {64, BN} box of K
  static constexpr int OUT_TILE = 32 * LCOLS * 2;           // 32 rows x LCOLS 16-bit columns
  static constexpr int OUT_BUFS = EPI_WARPS <= 8 ? 2 : 1;   // staging tiles per warp
  static constexpr int OUT_BYTES = EPI_WARPS * OUT_BUFS * OUT_TILE;
  static constexpr int STAT_BYTES = 2 * EPI_WARPS * 32 * 8;  // (max, sum) per row and slot, x2
  // accumulator buffers: as many BN-column tiles as TMEM holds (at most 4),
  // so the MMA can run up to ACC_BUFS - 1 tiles ahead of the epilogue
  static constexpr int ACC_BUFS = (4 * BN <= 512) ? 4 : 2;
  static constexpr int TMEM_COLS = (ACC_BUFS * BN <= 256) ? 256 : 512;
  static_assert(ACC_BUFS * BN <= 512, "accumulators fit TMEM");
  // barriers: full[S], empty[S], acc_full[B], acc_empty[B], q_full, q_empty, done, stat[4]
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 7;
  static constexpr int OUT_OFFSET = Q_BYTES + STAGES * STAGE_BYTES;
  static constexpr int STAT_OFFSET = OUT_OFFSET + OUT_BYTES;
  static constexpr int BAR_OFFSET = STAT_OFFSET + STAT_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
};

template <class L> struct AttnBars {
  uint32_t base;
  __device__ __forceinline__ explicit AttnBars(uint32_t b) : base(b) {}
  __device__ __forceinline__ uint32_t full(int i) const { return base + 8u * i; }
  __device__ __forceinline__ uint32_t empty(int i) const { return base + 8u * (L::STAGES + i); }
  static constexpr int A0 = 2 * L::STAGES, B2 = 2 * L::ACC_BUFS;
  __device__ __forceinline__ uint32_t acc_full(int b) const { return base + 8u * (A0 + b); }
  __device__ __forceinline__ uint32_t acc_empty(int b) const { return base + 8u * (A0 + L::ACC_BUFS + b); }
  __device__ __forceinline__ uint32_t q_full() const { return base + 8u * (A0 + B2); }
  __device__ __forceinline__ uint32_t q_empty() const { return base + 8u * (A0 + B2 + 1); }
  __device__ __forceinline__ uint32_t done() const { return base + 8u * (A0 + B2 + 2); }
  __device__ __forceinline__ uint32_t stat(int quarter) const { return base + 8u * (A0 + B2 + 3 + quarter); }
};

struct AttnShared {
  uint8_t* q;              // 1024-aligned resident Q tile
  uint8_t* ring;           // K stages
  uint8_t* outs;           // epilogue staging tiles
  float2* stats;           // [2][4 quarters][SLOTS][32 rows] (max, sum)
  uint32_t bars;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

template <class L>
__device__ __forceinline__ AttnShared attn_carve(uint8_t* raw) {
  AttnShared s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023);
  s.q = reinterpret_cast<uint8_t*>(base);
  s.ring = s.q + L::Q_BYTES;
  s.outs = s.q + L::OUT_OFFSET;
  s.stats = reinterpret_cast<float2*>(s.q + L::STAT_OFFSET);
  s.bars = smem_u32(s.q + L::BAR_OFFSET);
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.q + L::BAR_OFFSET + L::NUM_BARS * 8);
  s.abort_flag = reinterpret_cast<volatile int*>(s.tmem_slot + 1);
  return s;
}

__device__ __forceinline__ void attn_fail(const AttnShared& s, const AttnArgs& args) {
  *s.abort_flag = 1;
  if (args.status) atomicOr(args.status, kAttnTimeout);
}

template <class L>
__device__ __forceinline__ void attn_init(const AttnShared& s, const AttnArgs& args) {
  const int tid = gemm_tid(), warp = tid / 32;
  if (tid == 0) {
    const AttnBars<L> b(s.bars);
    for (int i = 0; i < L::STAGES; ++i) { mbar_init(b.full(i), 1); mbar_init(b.empty(i), 1); }
    for (int i = 0; i < L::ACC_BUFS; ++i) { mbar_init(b.acc_full(i), 1); mbar_init(b.acc_empty(i), L::RELEASERS); }
    mbar_init(b.q_full(), 1);
    mbar_init(b.q_empty(), 1);
    mbar_init(b.done(), 1);
    for (int i = 0; i < 4; ++i) mbar_init(b.stat(i), 32 * L::SLOTS);   // all warps of a quarter
    *s.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(&args.tmap_q) : "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(&args.tmap_k) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(s.tmem_slot)), "r"((uint32_t)L::TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
}

// ----------------------------------------------------------- primitives
// try_wait with a suspend-time hint: a waiting warp sleeps (issuing
// nothing) until the phase completes or `ns` nanoseconds pass.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity), "r"(ns) : "memory");
  return ok != 0;
}
// Bounded wait (MOLTEN_WAIT_NS in total); false on timeout.
__device__ __forceinline__ bool attn_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity, 1000000u)) {
    if (globaltimer_ns() - t0 > MOLTEN_WAIT_NS) return false;
  }
  return true;
}

// 32 lanes x 64 consecutive fp32 columns -> 64 registers per thread.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&r)[64]) {
  uint32_t u[64];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 "
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
               "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
               "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
               : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]),
                 "=r"(u[6]), "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]),
                 "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]),
                 "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]),
                 "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]),
                 "=r"(u[30]), "=r"(u[31]), "=r"(u[32]), "=r"(u[33]), "=r"(u[34]), "=r"(u[35]),
                 "=r"(u[36]), "=r"(u[37]), "=r"(u[38]), "=r"(u[39]), "=r"(u[40]), "=r"(u[41]),
                 "=r"(u[42]), "=r"(u[43]), "=r"(u[44]), "=r"(u[45]), "=r"(u[46]), "=r"(u[47]),
                 "=r"(u[48]), "=r"(u[49]), "=r"(u[50]), "=r"(u[51]), "=r"(u[52]), "=r"(u[53]),
                 "=r"(u[54]), "=r"(u[55]), "=r"(u[56]), "=r"(u[57]), "=r"(u[58]), "=r"(u[59]),
                 "=r"(u[60]), "=r"(u[61]), "=r"(u[62]), "=r"(u[63])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) r[i] = __uint_as_float(u[i]);
}
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&r)[N]) {
  static_assert(N == 32 || N == 64, "32 or 64 columns per load");
  if constexpr (N == 64) tmem_ld64(taddr, r);
  else tmem_ld32(taddr, r);
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               :: "l"(map), "r"(src), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// at most N bulk groups of this thread still reading shared memory
template <int N> __device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
               :: "r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2^x for element i of a block: the last POLY of every 32 on the FMA pipe
// (exp2_poly3), the rest on the EX2 unit -- both units busy at once.
template <int POLY>
__device__ __forceinline__ float attn_exp2(int i, float x) {
  return (i % 32) >= 32 - POLY ? exp2_poly3(x) : fast_exp2(x);
}

// Packed fp32 pairs (one FFMA2 / FADD2 instruction for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Two f16 exponentials per EX2 instruction: x rounded to f16, 2^x in f16
// (ex2.approx.f16x2), the pair summed as f16x2.
__device__ __forceinline__ uint32_t f16x2_pack(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t f16x2_exp2(uint32_t x) {
  uint32_t r;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
__device__ __forceinline__ uint32_t f16x2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float f16x2_sum_f32(uint32_t x) {
  const __half2 h = *reinterpret_cast<const __half2*>(&x);
  const float2 f = __half22float2(h);
  return f.x + f.y;
}

// Pass 0 on N columns of one row: running raw max `mx` and sum of
// 2^((s - mx) * C2); with MASK, columns from `valid` on are ignored
// (valid >= 1).  SUM16: the sum's exponentials in f16 pairs (half the EX2
// instructions; each term within about 2^-10 relative, the N/16-term f16
// partial sums within 2^-9, the rest in fp32) -- the sum only scales the
// row, so its error reaches every output of the row as one factor of about
// 1 + 1e-3 at worst.
template <int N, int POLY, bool MASK, bool SUM16 = false, bool X2 = false>
__device__ __forceinline__ void attn_stats(float (&a)[N], int valid, float C2, float& mx, float& sum) {
  constexpr int K = 8;                             // independent chains
  if constexpr (MASK) {
#pragma unroll
    for (int i = 0; i < N; ++i) a[i] = i < valid ? a[i] : -INFINITY;
  }
  float m[K];
#pragma unroll
  for (int j = 0; j < K; ++j) m[j] = a[j];
#pragma unroll
  for (int i = K; i < N; ++i) m[i % K] = fmaxf(m[i % K], a[i]);
#pragma unroll
  for (int w = K / 2; w >= 1; w /= 2) {
#pragma unroll
    for (int j = 0; j < w; ++j) m[j] = fmaxf(m[j], m[j + w]);
  }
  const float mn = fmaxf(mx, m[0]);                // finite: valid >= 1
  const float off = -mn * C2;
  if constexpr (SUM16) {
    uint32_t h[K];
#pragma unroll
    for (int j = 0; j < K; ++j) h[j] = 0u;
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const uint32_t e = f16x2_exp2(f16x2_pack(fmaf(a[i], C2, off), fmaf(a[i + 1], C2, off)));
      h[(i / 2) % K] = f16x2_add(h[(i / 2) % K], e);
    }
    float t[K];
#pragma unroll
    for (int j = 0; j < K; ++j) t[j] = f16x2_sum_f32(h[j]);
#pragma unroll
    for (int w = K / 2; w >= 1; w /= 2) {
#pragma unroll
      for (int j = 0; j < w; ++j) t[j] += t[j + w];
    }
    sum = sum * fast_exp2((mx - mn) * C2) + t[0];
    mx = mn;
    return;
  }
  float t[K];
  if constexpr (X2) {
    // arguments and sums in packed pairs: K/2 chains of (even, odd) columns
    float2 t2[K / 2];
#pragma unroll
    for (int j = 0; j < K / 2; ++j) t2[j] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 x = ffma2(make_float2(a[i], a[i + 1]), make_float2(C2, C2), make_float2(off, off));
      t2[(i / 2) % (K / 2)] = fadd2(t2[(i / 2) % (K / 2)],
                                    make_float2(attn_exp2<POLY>(i, x.x), attn_exp2<POLY>(i + 1, x.y)));
    }
#pragma unroll
    for (int j = 0; j < K / 2; ++j) { t[2 * j] = t2[j].x; t[2 * j + 1] = t2[j].y; }
  } else {
#pragma unroll
    for (int j = 0; j < K; ++j) t[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) t[i % K] += attn_exp2<POLY>(i, fmaf(a[i], C2, off));   // 2^-inf = 0
  }
#pragma unroll
  for (int w = K / 2; w >= 1; w /= 2) {
#pragma unroll
    for (int j = 0; j < w; ++j) t[j] += t[j + w];
  }
  sum = sum * fast_exp2((mx - mn) * C2) + t[0];   // 0 * 2^-inf on the first block
  mx = mn;
}

// OT: bf16 or f16 output.  TMA_STORE: pass-1 rows leave through the staging
// tiles and tmap_p (the caller guarantees that no 32-row box of a quarter
// whose first row is in [0, m) reaches another head's rows: m % 32 == 0 or
// batch == 1); else direct stores, 16 bytes at a time when ROWS_ALIGNED
// (n * 2 % 16 == 0), element by element otherwise.  C2 = scale * log2(e).
// POLY0 / POLY1: of every 32 exponentials, how many pass 0 / pass 1
// computes on the FMA pipe.  SUM16: pass-0 sums from f16 exponential pairs.
// X2: exponent arguments and pass-0 sums as packed fp32 pairs (FFMA2/FADD2).
// batch * m and batch * n are below 2^31.
template <class L, bool F16IN, typename OT, bool TMA_STORE, bool ROWS_ALIGNED, int POLY0 = 0,
          int POLY1 = 0, bool SUM16 = false, bool X2 = false>
__device__ __forceinline__ void attn_roles(const AttnShared& s, const AttnArgs& args, float C2) {
  tc_fence_after();
  const int tid = gemm_tid(), warp = tid / 32, lane = tid % 32;
  const uint32_t tmem = *s.tmem_slot;
  const AttnBars<L> bar(s.bars);
  const int M = (int)args.m, N = (int)args.n;
  const int MB = (M + L::BM - 1) / L::BM;
  const int NB = (N + L::BN - 1) / L::BN;
  const int T = (args.batch > 1 ? args.batch : 1) * MB;           // work items

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t st = 0, ph = 0, qph = 0;
      long long issued = 0;
      bool q_issued = false;
      for (int it = blockIdx.x; it < T && !*s.abort_flag; it += gridDim.x) {
        const int h = it / MB, mb = it - h * MB;
        if (!attn_wait(bar.q_empty(), qph ^ 1u)) { attn_fail(s, args); break; }
        qph ^= 1u;
        mbar_expect_tx(bar.q_full(), (uint32_t)L::Q_BYTES);
#pragma unroll
        for (int kc = 0; kc < L::DCH; ++kc)
          tma_load_2d(smem_u32(s.q + kc * L::Q_CHUNK), &args.tmap_q, bar.q_full(), kc * 64,
                      h * M + mb * L::BM);
        q_issued = true;
        bool ok = true;
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int nb = 0; nb < NB && ok; ++nb) {
#pragma unroll 1
            for (int kc = 0; kc < L::DCH; ++kc) {
              if (!attn_wait(bar.empty(st), ph ^ 1u)) { attn_fail(s, args); ok = false; break; }
              if (*s.abort_flag) { ok = false; break; }
              mbar_expect_tx(bar.full(st), (uint32_t)L::STAGE_BYTES);
              tma_load_2d(smem_u32(s.ring + st * L::STAGE_BYTES), &args.tmap_k, bar.full(st),
                          kc * 64, h * N + nb * L::BN);
              ++issued;
              if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
            }
          }
        }
        if (!ok) break;
      }
      if (*s.abort_flag) {
        // let the copies this thread issued land before the CTA can exit
        uint32_t ds = st, dp = ph;
        for (long long i = 0; i < issued && i < L::STAGES; ++i) {
          if (ds == 0) { ds = L::STAGES - 1; dp ^= 1u; } else { --ds; }
          if (!attn_wait(bar.full(ds), dp)) { if (args.status) atomicOr(args.status, kAttnTimeout); }
        }
        if (q_issued && !attn_wait(bar.q_full(), qph ^ 1u)) {
          if (args.status) atomicOr(args.status, kAttnTimeout);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = umma_idesc<L::BM, L::BN, F16IN, true>();
      uint32_t st = 0, ph = 0, qph = 0;
      uint32_t tile = 0;                           // accumulator buffers alternate per tile
      bool ok = true;
      for (int it = blockIdx.x; it < T && ok && !*s.abort_flag; it += gridDim.x) {
        if (!attn_wait(bar.q_full(), qph)) { attn_fail(s, args); break; }
        qph ^= 1u;
        tc_fence_after();
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int nb = 0; nb < NB && ok; ++nb, ++tile) {
            const int b = (int)(tile % (uint32_t)L::ACC_BUFS);
            const uint32_t acc_ph = (tile / (uint32_t)L::ACC_BUFS) & 1u;
            if (!attn_wait(bar.acc_empty(b), acc_ph ^ 1u)) { attn_fail(s, args); ok = false; break; }
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(b * L::BN);
            for (int kc = 0; kc < L::DCH; ++kc) {
              if (!attn_wait(bar.full(st), ph)) { attn_fail(s, args); ok = false; break; }
              tc_fence_after();
              const uint32_t a_base = smem_u32(s.q + kc * L::Q_CHUNK);
              const uint32_t b_base = smem_u32(s.ring + st * L::STAGE_BYTES);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_f16(d, umma_desc(a_base + 32u * kk, 16u, 1024u),
                         umma_desc(b_base + 32u * kk, 16u, 1024u), IDESC, (kc | kk) != 0 ? 1u : 0u);
              umma_commit(bar.empty(st));
              if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
            }
            if (ok) umma_commit(bar.acc_full(b));
          }
        }
        // the item's MMAs read Q: release the area once they have completed
        umma_commit(bar.q_empty());
      }
      umma_commit(bar.done());
      if (!attn_wait(bar.done(), 0u)) { if (args.status) atomicOr(args.status, kAttnTimeout); }
    }
  } else if (warp >= L::EPI_WARP0 && warp < L::EPI_WARP0 + L::EPI_WARPS) {
    // ------------------------------------------------------------- epilogue
    constexpr int LC = L::LCOLS, LOADS = L::PCOLS / L::LCOLS;
    const int ew = warp - L::EPI_WARP0;
    const int quarter = warp % 4, slot = ew / 4;
    const int group = slot % L::GROUPS, part = slot / L::GROUPS;
    const uint32_t lane_tmem = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(part * L::PCOLS);
    const uint32_t stage0 = smem_u32(s.outs + ew * L::OUT_BUFS * L::OUT_TILE);
    const int nb_full = N / L::BN;                 // column blocks with every column valid
    int sbuf = 0;
    uint32_t tile = 0, ni = 0;                     // tiles / items done by this CTA
    bool ok = true;
    for (int it = blockIdx.x; it < T && ok; it += gridDim.x, ++ni) {
      const int h = it / MB, mb = it - h * MB;
      const int qrow0 = mb * L::BM + quarter * 32;              // quarter's first row in the head
      const int mrow = qrow0 + lane;
      // ---- pass 0: row statistics
      float mx = -INFINITY, sum = 0.0f;            // raw-score max; sum of 2^((s - mx) * C2)
      for (int nb = 0; nb < NB; ++nb, ++tile) {
        const int b = (int)(tile % (uint32_t)L::ACC_BUFS);
        if (L::GROUPS == 2 && (b % 2) != group) continue;        // the other group's tile
        const bool got = attn_wait(bar.acc_full(b), (tile / (uint32_t)L::ACC_BUFS) & 1u);
        if (!__all_sync(0xffffffffu, got ? 1 : 0)) {
          if (lane == 0) attn_fail(s, args);
          ok = false;
          break;
        }
        tc_fence_after();
        const int colp = nb * L::BN + part * L::PCOLS;
#pragma unroll
        for (int u = 0; u < LOADS; ++u) {
          const int col0 = colp + u * LC;
          if (col0 >= N) break;                                  // warp-uniform
          float a[LC];
          tmem_ld_cols<LC>(lane_tmem + (uint32_t)(b * L::BN + u * LC), a);
          if (nb < nb_full) attn_stats<LC, POLY0, false, SUM16, X2>(a, LC, C2, mx, sum);
          else attn_stats<LC, POLY0, true, SUM16, X2>(a, N - col0, C2, mx, sum);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.acc_empty(b));
        if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) { ok = false; break; }
      }
      if (!ok) break;
      // merge the slots of each row, in slot order, so every warp of the
      // quarter derives the same lse (a slot that saw no column has
      // mx = -inf, sum = 0)
      float lse;
      {
        float2* stv = s.stats + (int)((ni & 1u) * 4 + quarter) * L::SLOTS * 32;
        stv[slot * 32 + lane] = make_float2(mx, sum);
        mbar_arrive(bar.stat(quarter));
        const bool merged = attn_wait(bar.stat(quarter), ni & 1u);
        if (!__all_sync(0xffffffffu, merged ? 1 : 0)) {
          if (lane == 0) attn_fail(s, args);
          ok = false;
          break;
        }
        float2 v[L::SLOTS];
#pragma unroll
        for (int j = 0; j < L::SLOTS; ++j) v[j] = stv[j * 32 + lane];
        float Mx = v[0].x;
#pragma unroll
        for (int j = 1; j < L::SLOTS; ++j) Mx = fmaxf(Mx, v[j].x);
        float S = 0.0f;
#pragma unroll
        for (int j = 0; j < L::SLOTS; ++j)
          if (v[j].x != -INFINITY) S += v[j].y * fast_exp2((v[j].x - Mx) * C2);
        lse = Mx * C2 + __log2f(S);                              // S >= 1 (the max term)
      }
      // ---- pass 1: probabilities
      for (int nb = 0; nb < NB; ++nb, ++tile) {
        const int b = (int)(tile % (uint32_t)L::ACC_BUFS);
        if (L::GROUPS == 2 && (b % 2) != group) continue;        // the other group's tile
        const bool got = attn_wait(bar.acc_full(b), (tile / (uint32_t)L::ACC_BUFS) & 1u);
        if (!__all_sync(0xffffffffu, got ? 1 : 0)) {
          if (lane == 0) attn_fail(s, args);
          ok = false;
          break;
        }
        tc_fence_after();
        const int colp = nb * L::BN + part * L::PCOLS;
#pragma unroll
        for (int u = 0; u < LOADS; ++u) {
          const int col0 = colp + u * LC;
          if (col0 >= N) break;                                  // warp-uniform
          float a[LC];
          tmem_ld_cols<LC>(lane_tmem + (uint32_t)(b * L::BN + u * LC), a);
          if constexpr (X2) {
#pragma unroll
            for (int i = 0; i < LC; i += 2) {
              const float2 x = ffma2(make_float2(a[i], a[i + 1]), make_float2(C2, C2),
                                     make_float2(-lse, -lse));
              a[i] = attn_exp2<POLY1>(i, x.x);
              a[i + 1] = attn_exp2<POLY1>(i + 1, x.y);
            }
          } else {
#pragma unroll
            for (int i = 0; i < LC; ++i) a[i] = attn_exp2<POLY1>(i, fmaf(a[i], C2, -lse));
          }
          if constexpr (TMA_STORE) {
            if (qrow0 >= M) continue;                            // warp-uniform
            const uint32_t tile_addr = stage0 + (uint32_t)(sbuf * L::OUT_TILE);
            if (lane == 0) bulk_wait_read<L::OUT_BUFS - 1>();     // this buffer's last store read it
            __syncwarp();
            // row `lane` is LC * 2 bytes; its 16-byte chunk q goes to chunk
            // q ^ pattern(row): the tensor map's 64-byte (LC = 32) or
            // 128-byte (LC = 64) swizzle, conflict-free across 8 lanes
            const uint32_t pat = LC == 64 ? (uint32_t)(lane & 7) : (uint32_t)((lane >> 1) & 3);
#pragma unroll
            for (int q = 0; q < LC / 8; ++q) {
              Slot<OT, 8> sl;
              pack_slot<OT, 8>(sl, *reinterpret_cast<const float(*)[8]>(&a[8 * q]));
              st_shared_v4(tile_addr + (uint32_t)lane * (LC * 2) + (((uint32_t)q ^ pat) * 16u),
                           *reinterpret_cast<const uint4*>(&sl));
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&args.tmap_p, tile_addr, col0, h * M + qrow0);
              bulk_commit();
            }
            if (L::OUT_BUFS == 2) sbuf ^= 1;
          } else {
            if (mrow >= M) continue;
            OT* dst = static_cast<OT*>(args.out) + ((long long)h * M + mrow) * N + col0;
            const int valid = N - col0 < LC ? N - col0 : LC;
#pragma unroll
            for (int q = 0; q < LC / 8; ++q) {
              if (ROWS_ALIGNED && 8 * q + 8 <= valid) {
                Slot<OT, 8> sl;
                pack_slot<OT, 8>(sl, *reinterpret_cast<const float(*)[8]>(&a[8 * q]));
                store_slot<kStoreDefault, OT, 8>(dst + 8 * q, sl);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (8 * q + e < valid) dst[8 * q + e] = from_f32<OT>(a[8 * q + e]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.acc_empty(b));
        if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) { ok = false; break; }
      }
    }
    if (TMA_STORE && lane == 0) bulk_wait_all();
  }
}

template <class L>
__device__ __forceinline__ void attn_teardown(const AttnShared& s) {
  const int warp = gemm_tid() / 32;
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(*s.tmem_slot), "r"((uint32_t)L::TMEM_COLS) : "memory");
  }
}

}  // namespace molten
