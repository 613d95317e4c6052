// tcgen05 / TMEM / TMA GEMM engine for C[M,N] = epilogue(A[M,K] @ B[K,N]).
//
// A is row-major (K-major operand), B is row-major [K, N] (MN-major operand,
// the layout the reference's matmul reads, codegen.py:354-355).  One CTA per
// SM runs a persistent loop over BM x BN output tiles with three roles:
//
//   warp 0      TMA producer: A box {BK, BM} and BN/64 B boxes {64, BK},
//               128-byte swizzle, into a STAGES-deep shared-memory ring;
//   warp 1      TMEM owner + MMA issuer: one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (bf16 in, fp32 in TMEM)
//               and tcgen05.commit's the ring slots and accumulators back;
//   warps 4..7  epilogue: tcgen05.ld 32 columns at a time, apply the
//               generated elementwise epilogue (bias, GELU ...) in fp32,
//               round once and store.
//
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.  Every TMA copy
// lands in the issuing CTA's own shared memory.
// Every mbarrier wait is bounded: on timeout the CTA records an error bit in
// *status, stops issuing work, drains what it issued and frees its TMEM.
#pragma once

#include <cuda.h>
#include "molten/common.cuh"

namespace molten {

// Kernel parameter block; mirrored by `molten_gemm_args` in include/molten_rt.h.
struct alignas(64) GemmArgs {
  CUtensorMap tmap_a;              // A [M, K], box {BK, BM}, 128B swizzle
  CUtensorMap tmap_b;              // B [K, N], box {64, BK}; or Bt [N, K], box {64, BN}
  const void* in[8];               // epilogue operands (kernel order)
  void* out[8];                    // outputs
  long long m, n, k;               // one problem: C[m, n] = A[m, k] B[k, n]
  long long row_offset;            // global row of local row 0
  int* status;                     // error bits (may be null)
  int batch;                       // stacked independent problems (0 or 1: one)
  float* work;                     // stream-K partial tiles (stream-K kernels only)
  int* tile_count;                 // stream-K per-tile arrival counters, kept at 0 between calls
};

enum GemmStatus { kGemmTimeoutFull = 1, kGemmTimeoutEmpty = 2, kGemmTimeoutAcc = 4,
                  kGemmTimeoutDrain = 8 };

#ifndef MOLTEN_WAIT_NS
#define MOLTEN_WAIT_NS 1000000000ull   // 1 s per wait
#endif

// ------------------------------------------------------------ primitives
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > MOLTEN_WAIT_NS) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
               " [%0], [%1, {%3, %4}], [%2];"
               :: "r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y) : "memory");
}

// tcgen05 shared-memory matrix descriptor (sm_100 version 1).
//   start address, LBO, SBO in 16-byte units; layout 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;           // version
  d |= (uint64_t)2 << 61;           // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D f32, A/B bf16 (or f16), A K-major,
// B MN-major (B [K, N] row-major) or K-major (B given as the rows of an
// [N, K] matrix, i.e. a transposed operand), shape M x N.
template <int M, int N, bool F16IN, bool B_KMAJOR = false>
__device__ __forceinline__ constexpr uint32_t umma_idesc() {
  return (1u << 4)                                  // D format f32
       | ((F16IN ? 0u : 1u) << 7)                    // A format
       | ((F16IN ? 0u : 1u) << 10)                   // B format
       | (0u << 15)                                  // A K-major
       | ((B_KMAJOR ? 0u : 1u) << 16)                // B MN-major / K-major
       | ((uint32_t)(N >> 3) << 17)
       | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\t"
               "setp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
               :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 32 lanes x 32 consecutive fp32 columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t u[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]),
                 "=r"(u[6]), "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]),
                 "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]),
                 "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]),
                 "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]),
                 "=r"(u[30]), "=r"(u[31])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(u[i]);
}

// ------------------------------------------------------- fp32 by bf16 planes
// An fp32 value x is split into three bf16 values x0 + x1 + x2 (each the
// round-to-nearest bf16 of what the previous ones left; 24 significand bits
// in all).  The product of two such sums is taken as the six terms with
// plane indices pa + pb <= 2; the three dropped terms and the split's
// residues are each below 2^-24 of |a b|.  This is the bf16x3 scheme of
// Henry, Tang and Heinecke, "Leveraging the bfloat16 Artificial Intelligence
// Datatype For Higher-Precision Computations" (ARITH 2019).
constexpr int kSplit3Products = 6;
// K step ks of the six-product loop -> (k-block, A plane, B plane); the
// products run from the smallest terms to x0 * y0.
__device__ __forceinline__ void split3_step(int ks, int KB, int& kb, int& pa, int& pb) {
  const int j = ks / KB;
  kb = ks - j * KB;
  // j:  0      1      2      3      4      5
  //    (2,0)  (1,1)  (0,2)  (1,0)  (0,1)  (0,0)
  pa = (0x001012 >> (4 * j)) & 0xF;
  pb = (0x010210 >> (4 * j)) & 0xF;
}

// x -> (x0, x1, x2).  A finite x whose x0 overflows (|x| above the largest
// bf16, ~3.39e38) becomes an infinity; an infinity or NaN is carried by x0
// alone, so products with it are the infinity or NaN of fp32 arithmetic.
__device__ __forceinline__ void split3_value(float x, bf16& x0, bf16& x1, bf16& x2) {
  x0 = __float2bfloat16_rn(x);
  const float h0 = __bfloat162float(x0);
  const float r1 = isfinite(h0) ? x - h0 : 0.0f;      // exact
  x1 = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(x1);          // exact
  x2 = __float2bfloat16_rn(r2);
}

// ------------------------------------------------------------ the engine
// PRO_: an RMSNorm prologue (see gemm_roles): 4 more warps, a "ready"
// barrier per stage, a double-buffered per-row 1/rms and its barriers.
template <int BM_, int BN_, int BK_, int STAGES_, int GROUP_M_ = 16, bool PRO_ = false>
struct GemmLayout {
  static constexpr int BM = BM_, BN = BN_, BK = BK_, STAGES = STAGES_, GROUP_M = GROUP_M_;
  static constexpr bool PRO = PRO_;
  static_assert(BM == 128, "one CTA owns the 128 TMEM lanes");
  static_assert(BK == 64, "BK is one 128-byte swizzle row of 16-bit elements");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, a multiple of 64");
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_CHUNK_BYTES = BK * 64 * 2;          // one {64, BK} box
  static constexpr int B_BYTES = (BN / 64) * B_CHUNK_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ACC_BUFS = 2;
  static constexpr int TMEM_COLS = (2 * BN <= 128) ? 128 : ((2 * BN <= 256) ? 256 : 512);
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2], done
  //           [+ ready[S], rms_full[2], rms_empty[2] with the prologue]
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 5 + (PRO ? STAGES + 4 : 0);
  static constexpr int RSQ_BYTES = PRO ? 2 * BM * 4 : 0;     // 1/rms of the tile rows, x2
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + RSQ_BYTES + 1024;
  static constexpr int THREADS = PRO ? 512 : 256;            // 8 warps (+8 prologue warps)
  static constexpr int PRO_WARP0 = 8;
  static constexpr int PRO_WARPS = 8;                         // 2 threads per A-tile row
  static constexpr int EPI_WARP0 = 4;                        // warps 4..7: TMEM lane quarters 0..3
  static constexpr int EPI_WARPS = 4;
};

struct GemmShared {
  uint8_t* tiles;          // 1024-aligned ring of stages
  uint64_t* bars;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
  float* rsq;              // prologue only: [2][BM] per-row 1/rms
};

// No prologue: A is used as loaded.
struct NoPrologue {
  static constexpr bool ENABLED = false;
  static constexpr float EPS = 0.0f;
  __device__ __forceinline__ static void w32(const GemmArgs&, long long, float (&w)[32]) {
#pragma unroll
    for (int e = 0; e < 32; ++e) w[e] = 1.0f;
  }
};

template <class L>
__device__ __forceinline__ GemmShared gemm_carve(uint8_t* raw) {
  GemmShared s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  s.bars = reinterpret_cast<uint64_t*>(s.tiles + L::BAR_OFFSET);
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.bars + L::NUM_BARS);
  s.abort_flag = reinterpret_cast<volatile int*>(s.tmem_slot + 1);
  s.rsq = reinterpret_cast<float*>(s.tmem_slot + 4);      // 16-byte aligned
  return s;
}

__device__ __forceinline__ int gemm_tid() { return threadIdx.y * blockDim.x + threadIdx.x; }

// Output tile of persistent-loop index `tile`.  Tiles are walked in groups
// of GROUP_M row blocks, column-major inside a group, so the CTAs running at
// the same time share a GROUP_M-block panel of A and a few panels of B, which
// stay in L2 instead of being re-read from HBM on every wave.
template <class L>
__device__ __forceinline__ void gemm_tile_coords(long long tile, long long MB, long long NB,
                                                 int& m0, int& n0, int& h) {
  // problem h of a batch: its MB x NB tiles are consecutive
  h = (int)(tile / (MB * NB));
  tile -= (long long)h * MB * NB;
  const long long G = L::GROUP_M;
  const long long span = G * NB;                       // tiles of a full group
  const long long g = tile / span;
  const long long r = tile - g * span;
  const long long rows_g = (MB - g * G) < G ? (MB - g * G) : G;   // last group may be short
  m0 = (int)((g * G + r % rows_g) * L::BM);
  n0 = (int)((r / rows_g) * L::BN);
}

// barrier addresses
template <class L> struct Bars {
  uint32_t base;
  __device__ __forceinline__ explicit Bars(const GemmShared& s) : base(smem_u32(s.bars)) {}
  __device__ __forceinline__ uint32_t full(int i) const { return base + 8u * i; }
  __device__ __forceinline__ uint32_t empty(int i) const { return base + 8u * (L::STAGES + i); }
  __device__ __forceinline__ uint32_t acc_full(int b) const { return base + 8u * (2 * L::STAGES + b); }
  __device__ __forceinline__ uint32_t acc_empty(int b) const { return base + 8u * (2 * L::STAGES + 2 + b); }
  __device__ __forceinline__ uint32_t done() const { return base + 8u * (2 * L::STAGES + 4); }
  __device__ __forceinline__ uint32_t ready(int i) const { return base + 8u * (2 * L::STAGES + 5 + i); }
  __device__ __forceinline__ uint32_t rms_full(int b) const { return base + 8u * (3 * L::STAGES + 5 + b); }
  __device__ __forceinline__ uint32_t rms_empty(int b) const { return base + 8u * (3 * L::STAGES + 7 + b); }
};

__device__ __forceinline__ void gemm_fail(const GemmShared& s, const GemmArgs& args, int code) {
  *s.abort_flag = 1;
  if (args.status) atomicOr(args.status, code);
}

// Barrier init + TMEM allocation.  Every thread calls it; the caller then
// runs __syncthreads() before gemm_roles.
template <class L>
__device__ __forceinline__ void gemm_init(const GemmShared& s, const GemmArgs& args) {
  const int tid = gemm_tid(), warp = tid / 32;
  if (tid == 0) {
    const Bars<L> b(s);
    for (int i = 0; i < L::STAGES; ++i) { mbar_init(b.full(i), 1); mbar_init(b.empty(i), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(b.acc_full(i), 1); mbar_init(b.acc_empty(i), L::EPI_WARPS); }
    mbar_init(b.done(), 1);
    if constexpr (L::PRO) {
      for (int i = 0; i < L::STAGES; ++i) mbar_init(b.ready(i), L::PRO_WARPS);   // one per warp
      for (int i = 0; i < 2; ++i) { mbar_init(b.rms_full(i), L::PRO_WARPS); mbar_init(b.rms_empty(i), L::EPI_WARPS); }
    }
    *s.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(&args.tmap_a) : "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(&args.tmap_b) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(s.tmem_slot)), "r"((uint32_t)L::TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
}

// ---------------------------------------------- SPLIT3: promoted accumulation
// The tensor core's fp32 accumulation loses accuracy with the length of the
// chain it sums (measured on the six-product fp32 GEMM: 1.4e-6 of max|C| at
// K = 1024, 4.6e-6 at K = 4096).  So the SPLIT3 K loop is cut into chunks of
// kSplit3Chunk k-steps: the MMA issuer starts a fresh accumulator (the two
// TMEM buffers alternate per chunk) and the epilogue warps add each chunk
// into fp32 registers (round to nearest), one BN-column row per thread.
constexpr int kSplit3Chunk = 4;

template <class L, bool B_KMAJOR>
__device__ __forceinline__ void gemm_split3_mma(const GemmShared& s, const GemmArgs& args,
                                                uint32_t tmem, long long T, int KSTEPS) {
  constexpr uint32_t IDESC = umma_idesc<L::BM, L::BN, false, B_KMAJOR>();
  const Bars<L> bar(s);
  uint32_t st = 0, ph = 0;
  long long chunk = 0;
  bool ok = true;
  for (long long tile = blockIdx.x; tile < T && ok && !*s.abort_flag; tile += gridDim.x) {
    for (int c0 = 0; c0 < KSTEPS && ok; c0 += kSplit3Chunk, ++chunk) {
      const int b = (int)(chunk & 1);
      const uint32_t acc_ph = (uint32_t)((chunk >> 1) & 1);
      if (!mbar_wait(bar.acc_empty(b), acc_ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutAcc); ok = false; break; }
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(b * L::BN);
      const int c1 = (c0 + kSplit3Chunk < KSTEPS) ? c0 + kSplit3Chunk : KSTEPS;
      for (int ks = c0; ks < c1; ++ks) {
        if (!mbar_wait(bar.full(st), ph)) { gemm_fail(s, args, kGemmTimeoutFull); ok = false; break; }
        tc_fence_after();
        const uint32_t a_base = smem_u32(s.tiles + st * L::STAGE_BYTES);
        const uint32_t b_base = a_base + L::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < L::BK / 16; ++kk) {
          const uint64_t ad = umma_desc(a_base + 32u * kk, 16u, 1024u);
          const uint64_t bd = B_KMAJOR
              ? umma_desc(b_base + 32u * kk, 16u, 1024u)
              : umma_desc(b_base + 2048u * kk, (uint32_t)L::B_CHUNK_BYTES, 1024u);
          umma_f16(d, ad, bd, IDESC, ((ks - c0) | kk) != 0 ? 1u : 0u);
        }
        umma_commit(bar.empty(st));
        if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
      }
      if (ok) umma_commit(bar.acc_full(b));
    }
  }
  // all MMAs this thread issued must finish before TMEM is released
  umma_commit(bar.done());
  if (!mbar_wait(bar.done(), 0u)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
}

template <class L, class Epi>
__device__ __forceinline__ void gemm_split3_epilogue(const GemmShared& s, const GemmArgs& args,
                                                     uint32_t tmem, long long T, int KSTEPS,
                                                     long long MB, long long NB) {
  static_assert(L::BN == 128, "one 128-column accumulator row per thread");
  const int warp = gemm_tid() / 32, lane = gemm_tid() % 32;
  const int quarter = warp % 4;                  // TMEM lanes 32*quarter .. +31
  const Bars<L> bar(s);
  long long chunk = 0;
  bool ok = true;
  for (long long tile = blockIdx.x; tile < T && ok; tile += gridDim.x) {
    float sum[L::BN];
#pragma unroll
    for (int q = 0; q < L::BN; ++q) sum[q] = 0.0f;
#pragma unroll 1
    for (int c0 = 0; c0 < KSTEPS; c0 += kSplit3Chunk, ++chunk) {
      const int b = (int)(chunk & 1);
      const uint32_t acc_ph = (uint32_t)((chunk >> 1) & 1);
      const bool got = mbar_wait(bar.acc_full(b), acc_ph);
      if (!__all_sync(0xffffffffu, got ? 1 : 0)) {
        if (lane == 0) gemm_fail(s, args, kGemmTimeoutAcc);
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < L::BN / 32; ++c) {
        float part[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * L::BN + c * 32), part);
#pragma unroll
        for (int q = 0; q < 32; ++q) sum[32 * c + q] += part[q];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.acc_empty(b));
    }
    if (!ok) break;
    int m0, n0, h;
    gemm_tile_coords<L>(tile, MB, NB, m0, n0, h);
    const long long mrow = (long long)m0 + quarter * 32 + lane;   // row of problem h
    const long long row = (long long)h * args.m + mrow;           // row of stacked C
#pragma unroll
    for (int c = 0; c < L::BN / 32; ++c) {
      const long long col0 = (long long)n0 + 32 * c;
      if (col0 < args.n && mrow < args.m)
        Epi::apply(args, row, col0, *reinterpret_cast<const float(*)[32]>(&sum[32 * c]));
    }
    if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) break;
  }
}

// The three roles.  Epi::apply(args, row, col0, acc[32]) writes C[row, col0..col0+31]
// (row of the stacked C, always a valid row; columns from col0 < n).
// B_KMAJOR: tmap_b describes Bt [N, K] (inner K) with box {64, BN}; a stage
// holds BN rows of 128 bytes, the same 128-byte-swizzled K-major layout as A.
// Pro (ENABLED): C = diag(1/rms(x)) ((x * w) B) for A = rmsnorm(x, w) with
// rms(x) = sqrt(mean_k x^2 + EPS): warps 8..11 (one tile row per thread)
// take each landed A stage, multiply row r's elements by w[k] in shared
// memory (one bf16/fp16 rounding of x*w; the 128-byte swizzle puts logical
// 16-byte chunk c of row r at chunk c ^ (r mod 8)), accumulate sum x^2,
// make the writes visible to the tensor core (async proxy) and arrive on
// the stage's "ready" barrier, which the MMA waits for instead of "full".
// After a tile's K loop they publish 1/rms per row; the epilogue scales the
// accumulator rows by it.
// SPLIT3: fp32 operands given as three bf16 planes each (x ~ x0 + x1 + x2,
// split3_planes), stacked by rows: A planes [3 * batch*m, k], B planes
// [3 * batch*k, n] (or Bt planes [3 * batch*n, k]).  The K loop runs over the
// six products with plane indices pa + pb <= 2 (smallest first), so the
// accumulator holds A @ B to about fp32 accuracy.
template <class L, bool F16IN, class Epi, bool B_KMAJOR = false, class Pro = NoPrologue,
          bool SPLIT3 = false>
__device__ __forceinline__ void gemm_roles(const GemmShared& s, const GemmArgs& args) {
  tc_fence_after();
  const int tid = gemm_tid(), warp = tid / 32, lane = tid % 32;
  const uint32_t tmem = *s.tmem_slot;
  const Bars<L> bar(s);
  const long long MB = (args.m + L::BM - 1) / L::BM;
  const long long NB = (args.n + L::BN - 1) / L::BN;
  const long long T = (args.batch > 1 ? args.batch : 1) * MB * NB;
  const int KB = (int)((args.k + L::BK - 1) / L::BK);
  const int KSTEPS = SPLIT3 ? kSplit3Products * KB : KB;     // k-blocks per tile
  // Batched problems are stacked: A [batch*m, k], B [batch*k, n] (or
  // Bt [batch*n, k]), C [batch*m, n].  A tile of problem h that runs past its
  // m rows (or n columns) reads the next problem's rows; those products land
  // in rows / columns the epilogue never stores.  Past k, A is zero-filled
  // (its columns end at k), so whatever B rows sit there multiply zeros.

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t st = 0, ph = 0;
      long long issued = 0;
      for (long long tile = blockIdx.x; tile < T && !*s.abort_flag; tile += gridDim.x) {
        int m0, n0, h;
        gemm_tile_coords<L>(tile, MB, NB, m0, n0, h);
        const int nb = args.batch > 1 ? args.batch : 1;
        for (int ks = 0; ks < KSTEPS; ++ks) {
          int kb = ks, pa = 0, pb = 0;
          if constexpr (SPLIT3) split3_step(ks, KB, kb, pa, pb);
          const int a_row = (int)((pa * nb + h) * args.m) + m0;
          if (!mbar_wait(bar.empty(st), ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutEmpty); break; }
          if (*s.abort_flag) break;
#ifdef MOLTEN_TEST_SKIP_KSTEP
          // Failure-detection test builds only: k-step MOLTEN_TEST_SKIP_KSTEP
          // of this CTA's first tile is neither armed nor copied, so the MMA
          // issuer's bounded wait for that stage runs out.
          if (tile == (long long)blockIdx.x && ks == MOLTEN_TEST_SKIP_KSTEP) {
            if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
            continue;
          }
#endif
          const uint32_t a_dst = smem_u32(s.tiles + st * L::STAGE_BYTES);
          const uint32_t b_dst = a_dst + L::A_BYTES;
          mbar_expect_tx(bar.full(st), (uint32_t)L::STAGE_BYTES);
          tma_load_2d(a_dst, &args.tmap_a, bar.full(st), kb * L::BK, a_row);
          if constexpr (B_KMAJOR) {
            tma_load_2d(b_dst, &args.tmap_b, bar.full(st), kb * L::BK,
                        (int)((pb * nb + h) * args.n) + n0);
          } else {
#pragma unroll
            for (int c = 0; c < L::BN / 64; ++c)
              tma_load_2d(b_dst + c * L::B_CHUNK_BYTES, &args.tmap_b, bar.full(st), n0 + 64 * c,
                          (int)((pb * nb + h) * args.k) + kb * L::BK);
          }
          ++issued;
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
      }
      if (*s.abort_flag) {
        // let the copies this thread issued land before the CTA can exit
        uint32_t ds = st, dp = ph;
        for (long long i = 0; i < issued && i < L::STAGES; ++i) {
          if (ds == 0) { ds = L::STAGES - 1; dp ^= 1u; } else { --ds; }
          if (!mbar_wait(bar.full(ds), dp)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (SPLIT3 && lane == 0) {
      gemm_split3_mma<L, B_KMAJOR>(s, args, tmem, T, KSTEPS);
    } else if (lane == 0) {
      constexpr uint32_t IDESC = umma_idesc<L::BM, L::BN, F16IN, B_KMAJOR>();
      uint32_t st = 0, ph = 0;
      long long i = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; tile < T && ok && !*s.abort_flag; tile += gridDim.x, ++i) {
        const int b = (int)(i & 1);
        const uint32_t acc_ph = (uint32_t)((i >> 1) & 1);
        if (!mbar_wait(bar.acc_empty(b), acc_ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutAcc); break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * L::BN);
        for (int kb = 0; kb < KSTEPS; ++kb) {
          const uint32_t in_bar = Pro::ENABLED ? bar.ready(st) : bar.full(st);
          if (!mbar_wait(in_bar, ph)) { gemm_fail(s, args, kGemmTimeoutFull); ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(s.tiles + st * L::STAGE_BYTES);
          const uint32_t b_base = a_base + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < L::BK / 16; ++kk) {
            const uint64_t ad = umma_desc(a_base + 32u * kk, 16u, 1024u);
            const uint64_t bd = B_KMAJOR
                ? umma_desc(b_base + 32u * kk, 16u, 1024u)
                : umma_desc(b_base + 2048u * kk, (uint32_t)L::B_CHUNK_BYTES, 1024u);
            umma_f16(d, ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(bar.empty(st));
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
        if (ok) umma_commit(bar.acc_full(b));
      }
      // all MMAs this thread issued must finish before TMEM is released
      umma_commit(bar.done());
      if (!mbar_wait(bar.done(), 0u)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
    }
  } else if (Pro::ENABLED && warp >= L::PRO_WARP0) {
    // ------------------------------------------------------------- prologue
    if constexpr (Pro::ENABLED) {
      const int p = tid - L::PRO_WARP0 * 32;       // 0 .. 2*BM-1
      const int r = p >> 1, half = p & 1;          // tile row; 16-byte chunks 4*half .. +3
      const uint32_t swz = (uint32_t)(r & 7);
      uint32_t st = 0, ph = 0;
      long long i = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; tile < T && ok && !*s.abort_flag; tile += gridDim.x, ++i) {
        float ss = 0.0f;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(bar.full(st), ph)) { gemm_fail(s, args, kGemmTimeoutFull); ok = false; break; }
          const uint32_t row_addr = smem_u32(s.tiles + st * L::STAGE_BYTES) + (uint32_t)r * 128u;
          const long long kh = (long long)kb * L::BK + 32 * half;       // first k of this half
          // all loads first: 4 chunks of A, 32 weights
          uint4 v[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a = row_addr + ((((uint32_t)(4 * half + j)) ^ swz) << 4);
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v[j].x), "=r"(v[j].y), "=r"(v[j].z), "=r"(v[j].w) : "r"(a));
          }
          float w[32];
          Pro::w32(args, kh, w);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (kh + 8 * j >= args.k) break;          // K is a multiple of 8; the rest is zero
            uint32_t* u = reinterpret_cast<uint32_t*>(&v[j]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x0, x1;
              if constexpr (F16IN) {
                const __half2 hx = *reinterpret_cast<const __half2*>(&u[q]);
                x0 = __low2float(hx); x1 = __high2float(hx);
                const __half2 y = __floats2half2_rn(x0 * w[8 * j + 2 * q], x1 * w[8 * j + 2 * q + 1]);
                u[q] = *reinterpret_cast<const uint32_t*>(&y);
              } else {
                x0 = __uint_as_float(u[q] << 16);
                x1 = __uint_as_float(u[q] & 0xFFFF0000u);
                const __nv_bfloat162 y = __floats2bfloat162_rn(x0 * w[8 * j + 2 * q], x1 * w[8 * j + 2 * q + 1]);
                u[q] = *reinterpret_cast<const uint32_t*>(&y);
              }
              ss = fmaf(x0, x0, fmaf(x1, x1, ss));
            }
            const uint32_t a = row_addr + ((((uint32_t)(4 * half + j)) ^ swz) << 4);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};"
                         :: "r"(a), "r"(v[j].x), "r"(v[j].y), "r"(v[j].z), "r"(v[j].w) : "memory");
          }
          // generic-proxy writes -> visible to the tensor core's reads; one
          // arrival per warp once all its lanes are done
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(bar.ready(st));
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
        if (!ok) break;
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);    // the row's two halves
        const int b = (int)(i & 1);
        const uint32_t rph = (uint32_t)((i >> 1) & 1);
        if (!mbar_wait(bar.rms_empty(b), rph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutAcc); break; }
        if (half == 0) s.rsq[b * L::BM + r] = rsqrtf(ss / (float)args.k + Pro::EPS);
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.rms_full(b));
      }
    }
  } else if (warp >= L::EPI_WARP0 && warp < L::EPI_WARP0 + L::EPI_WARPS) {
    // ------------------------------------------------------------- epilogue
    if constexpr (SPLIT3) {
      gemm_split3_epilogue<L, Epi>(s, args, tmem, T, KSTEPS, MB, NB);
      return;
    }
    const int quarter = warp % 4;                  // TMEM lanes 32*quarter .. +31
    long long i = 0;
    for (long long tile = blockIdx.x; tile < T; tile += gridDim.x, ++i) {
      const int b = (int)(i & 1);
      const uint32_t acc_ph = (uint32_t)((i >> 1) & 1);
      const bool got = mbar_wait(bar.acc_full(b), acc_ph);
      if (!__all_sync(0xffffffffu, got ? 1 : 0)) {
        if (lane == 0) gemm_fail(s, args, kGemmTimeoutAcc);
        break;
      }
      tc_fence_after();
      int m0, n0, h;
      gemm_tile_coords<L>(tile, MB, NB, m0, n0, h);
      const long long mrow = (long long)m0 + quarter * 32 + lane;   // row of problem h
      const long long row = (long long)h * args.m + mrow;           // row of stacked C
      const long long nbase = n0;
      float rinv = 1.0f;
      if constexpr (Pro::ENABLED) {
        const bool gr = mbar_wait(bar.rms_full(b), acc_ph);
        if (!__all_sync(0xffffffffu, gr ? 1 : 0)) {
          if (lane == 0) gemm_fail(s, args, kGemmTimeoutAcc);
          break;
        }
        rinv = s.rsq[b * L::BM + quarter * 32 + lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.rms_empty(b));
      }
#pragma unroll 1
      for (int c = 0; c < L::BN / 32; ++c) {
        float acc[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * L::BN + c * 32), acc);
        if constexpr (Pro::ENABLED) {
#pragma unroll
          for (int q = 0; q < 32; ++q) acc[q] *= rinv;
        }
        const long long col0 = nbase + 32 * c;
        if (col0 < args.n && mrow < args.m) Epi::apply(args, row, col0, acc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.acc_empty(b));
      if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) break;
    }
  }
}

// Release TMEM.  Every thread calls it after the caller's final __syncthreads().
template <class L>
__device__ __forceinline__ void gemm_teardown(const GemmShared& s) {
  const int warp = gemm_tid() / 32;
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(*s.tmem_slot), "r"((uint32_t)L::TMEM_COLS) : "memory");
  }
}

}  // namespace molten
