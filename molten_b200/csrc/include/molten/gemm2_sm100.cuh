// Two-SM tcgen05 GEMM for sm_100a: a cluster of 2 CTAs (an SM pair) owns a
// 256 x BN output tile and computes it with tcgen05.mma.cta_group::2
// (M = 256): each CTA stages its own 128 rows of A and its own BN/2 columns
// of B, the pair's MMA reads both halves, and each CTA's TMEM receives its
// 128 rows x BN columns of fp32 accumulators.  Per FLOP, shared memory and
// L2 deliver half the B bytes of the one-SM engine (molten/gemm_sm100.cuh),
// whose GemmArgs, epilogue functors and primitives this engine reuses.
//
//   warp 0  (both CTAs)  TMA producer: its CTA's A and B halves of each k
//                        block into its own shared memory, completing bytes
//                        on the even CTA's `full` barrier (tensor copies with
//                        .cta_group::2); the even CTA alone arms `full` for both
//                        CTAs' bytes with a local arrive.expect_tx (a remote,
//                        cluster-release arrive per stage measured 1.7x
//                        slower: its fence starved the MMA);
//   warp 1  (even CTA)   MMA issuer: waits on `full`, issues the pair's
//                        MMAs, commits `empty` stages and `acc_full`
//                        buffers to both CTAs (one tcgen05.commit with a
//                        2-CTA mask);
//   warp 1  (both)       TMEM allocation and release, done collectively by
//                        the pair (tcgen05.alloc/dealloc .cta_group::2);
//   warps 4..7 (both)    epilogue of the CTA's 128 rows, releasing an
//                        accumulator buffer on the even CTA's `acc_empty`
//                        (8 arrivals: 4 warps per CTA).
//
// Every mbarrier wait is bounded; a CTA that times out sets its abort flag
// and a status bit, drains its own copies and leaves; the pair meets at a
// cluster barrier before TMEM is released and the CTAs exit.
#pragma once

#include "molten/gemm_sm100.cuh"

namespace molten {

template <int BN_, int STAGES_, int GROUP_M_ = 16>
struct Gemm2Layout {
  static constexpr int BM = 256, CTA_M = 128, BN = BN_, BK = 64, STAGES = STAGES_, GROUP_M = GROUP_M_;
  static_assert(BN % 128 == 0 && BN >= 128 && BN <= 256, "BN must be 128 or 256 (BN/2 per CTA)");
  static constexpr int A_BYTES = CTA_M * BK * 2;              // this CTA's 128 rows
  static constexpr int B_COLS = BN / 2;                        // this CTA's columns of B
  static constexpr int B_CHUNK_BYTES = BK * 64 * 2;            // one {64, BK} box (MN-major B)
  static constexpr int B_BYTES = B_COLS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;        // per CTA
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2], done
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static constexpr int THREADS = 256;
  static constexpr int EPI_WARP0 = 4, EPI_WARPS = 4;
};

// ------------------------------------------------------ pair primitives
__device__ __forceinline__ uint32_t pair_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r & 1u;
}
// The same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t pair_map(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on an mbarrier of either CTA of the pair
__device__ __forceinline__ void pair_arrive(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
               :: "r"(cluster_bar) : "memory");
}
// TMA tile load into this CTA's shared memory, completing bytes on an
// mbarrier of either CTA of the pair.
__device__ __forceinline__ void pair_tma_load_2d(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t cluster_bar, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
               " [%0], [%1, {%3, %4}], [%2];"
               :: "r"(dst), "l"(map), "r"(cluster_bar), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void pair_umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\t"
               "setp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
               :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on the mbarrier at this shared-memory offset in both CTAs once the
// pair's MMAs issued so far have completed.
__device__ __forceinline__ void pair_umma_commit_both(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
               " [%0], %1;" :: "r"(bar), "h"((uint16_t)3) : "memory");
}

__device__ __forceinline__ GemmShared gemm2_carve_base(uint8_t* raw, int bar_offset, int num_bars) {
  GemmShared s;
  const uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023);
  s.tiles = reinterpret_cast<uint8_t*>(base);
  s.bars = reinterpret_cast<uint64_t*>(s.tiles + bar_offset);
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.bars + num_bars);
  s.abort_flag = reinterpret_cast<volatile int*>(s.tmem_slot + 1);
  s.rsq = nullptr;
  return s;
}
template <class L>
__device__ __forceinline__ GemmShared gemm2_carve(uint8_t* raw) {
  return gemm2_carve_base(raw, L::BAR_OFFSET, L::NUM_BARS);
}

// Barrier init, TMEM allocation (both CTAs' warp 1 together) and a pair
// barrier, so that no remote arrival or byte count reaches a barrier before
// its initialisation.  Every thread of both CTAs calls it.
template <class L>
__device__ __forceinline__ void gemm2_init(const GemmShared& s, const GemmArgs& args) {
  const int tid = gemm_tid(), warp = tid / 32;
  if (tid == 0) {
    const Bars<L> b(s);
    // full: the even CTA's arrive.expect_tx for both CTAs' bytes; acc_empty:
    // 4 epilogue warps per CTA
    for (int i = 0; i < L::STAGES; ++i) { mbar_init(b.full(i), 1); mbar_init(b.empty(i), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(b.acc_full(i), 1); mbar_init(b.acc_empty(i), 2 * L::EPI_WARPS); }
    mbar_init(b.done(), 1);
    *s.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(&args.tmap_a) : "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(&args.tmap_b) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(s.tmem_slot)), "r"((uint32_t)L::TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  pair_sync();
}

// The roles.  Epi::apply(args, row, col0, acc[32]) as in gemm_roles.
// B_KMAJOR: tmap_b describes Bt [N, K] (inner K) with box {64, BN/2}.
// SPLIT3: fp32 operands as stacked bf16 planes, six products per k-block
// (see gemm_roles in molten/gemm_sm100.cuh).
template <class L, bool F16IN, class Epi, bool B_KMAJOR = false, bool SPLIT3 = false>
__device__ __forceinline__ void gemm2_roles(const GemmShared& s, const GemmArgs& args) {
  tc_fence_after();
  const int tid = gemm_tid(), warp = tid / 32, lane = tid % 32;
  const uint32_t rank = pair_rank();
  const uint32_t tmem = *s.tmem_slot;
  const Bars<L> bar(s);
  const long long MB = (args.m + L::BM - 1) / L::BM;
  const long long NB = (args.n + L::BN - 1) / L::BN;
  const long long T = (args.batch > 1 ? args.batch : 1) * MB * NB;
  const int KB = (int)((args.k + L::BK - 1) / L::BK);
  const int KSTEPS = SPLIT3 ? kSplit3Products * KB : KB;     // k-blocks per tile
  const long long pair = blockIdx.x / 2, pairs = gridDim.x / 2;

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t st = 0, ph = 0;
      long long issued = 0;
      for (long long tile = pair; tile < T && !*s.abort_flag; tile += pairs) {
        int m0, n0, h;
        gemm_tile_coords<L>(tile, MB, NB, m0, n0, h);
        const int nb = args.batch > 1 ? args.batch : 1;
        const int b_col = n0 + (int)rank * L::B_COLS;
        for (int ks = 0; ks < KSTEPS; ++ks) {
          int kb = ks, pa = 0, pb = 0;
          if constexpr (SPLIT3) split3_step(ks, KB, kb, pa, pb);
          const int a_row = (int)((pa * nb + h) * args.m) + m0 + (int)rank * L::CTA_M;
          if (!mbar_wait(bar.empty(st), ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutEmpty); break; }
          if (*s.abort_flag) break;
          const uint32_t a_dst = smem_u32(s.tiles + st * L::STAGE_BYTES);
          const uint32_t b_dst = a_dst + L::A_BYTES;
          const uint32_t full0 = pair_map(bar.full(st), 0u);     // the even CTA's barrier
          // Bytes may land before the arming: the phase cannot complete
          // without the even CTA's arrival, and neither producer refills a
          // stage before both CTAs' `empty` commit for it.
          if (rank == 0) mbar_expect_tx(bar.full(st), (uint32_t)(2 * L::STAGE_BYTES));
          pair_tma_load_2d(a_dst, &args.tmap_a, full0, kb * L::BK, a_row);
          if constexpr (B_KMAJOR) {
            pair_tma_load_2d(b_dst, &args.tmap_b, full0, kb * L::BK,
                             (int)((pb * nb + h) * args.n) + b_col);
          } else {
#pragma unroll
            for (int c = 0; c < L::B_COLS / 64; ++c)
              pair_tma_load_2d(b_dst + c * L::B_CHUNK_BYTES, &args.tmap_b, full0, b_col + 64 * c,
                               (int)((pb * nb + h) * args.k) + kb * L::BK);
          }
          ++issued;
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
      }
      if (*s.abort_flag && rank == 0) {
        // the even CTA's barriers count both CTAs' bytes: wait for the stages
        // this thread armed (the peer's copies land in the peer's memory)
        uint32_t ds = st, dp = ph;
        for (long long i = 0; i < issued && i < L::STAGES; ++i) {
          if (ds == 0) { ds = L::STAGES - 1; dp ^= 1u; } else { --ds; }
          if (!mbar_wait(bar.full(ds), dp)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------- MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t IDESC = umma_idesc<L::BM, L::BN, F16IN, B_KMAJOR>();
      uint32_t st = 0, ph = 0;
      long long i = 0;
      bool ok = true;
      for (long long tile = pair; tile < T && ok && !*s.abort_flag; tile += pairs, ++i) {
        const int b = (int)(i & 1);
        const uint32_t acc_ph = (uint32_t)((i >> 1) & 1);
        if (!mbar_wait(bar.acc_empty(b), acc_ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutAcc); break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * L::BN);
        for (int kb = 0; kb < KSTEPS; ++kb) {
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
            pair_umma_f16(d, ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
          }
          pair_umma_commit_both(bar.empty(st));
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
        if (ok) pair_umma_commit_both(bar.acc_full(b));
      }
      // all MMAs this thread issued must finish before TMEM is released
      pair_umma_commit_both(bar.done());
    }
    if (lane == 0) {
      // both CTAs: the pair's MMAs are complete before the collective release
      if (!mbar_wait(bar.done(), 0u)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
    }
  } else if (warp >= L::EPI_WARP0 && warp < L::EPI_WARP0 + L::EPI_WARPS) {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp % 4;                  // TMEM lanes 32*quarter .. +31
    const uint32_t acc_empty0 = pair_map(bar.acc_empty(0), 0u);
    const uint32_t acc_empty1 = pair_map(bar.acc_empty(1), 0u);
    long long i = 0;
    for (long long tile = pair; tile < T; tile += pairs, ++i) {
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
      const long long mrow = (long long)m0 + rank * L::CTA_M + quarter * 32 + lane;   // row of problem h
      const long long row = (long long)h * args.m + mrow;                            // row of stacked C
#pragma unroll 1
      for (int c = 0; c < L::BN / 32; ++c) {
        float acc[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * L::BN + c * 32), acc);
        const long long col0 = (long long)n0 + 32 * c;
        if (col0 < args.n && mrow < args.m) Epi::apply(args, row, col0, acc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) pair_arrive(b ? acc_empty1 : acc_empty0);
      if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) break;
    }
  }
}

// Pair barrier, then the collective TMEM release.  Every thread of both
// CTAs calls it after the caller's final __syncthreads().
template <class L>
__device__ __forceinline__ void gemm2_teardown(const GemmShared& s) {
  const int warp = gemm_tid() / 32;
  pair_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                 :: "r"(*s.tmem_slot), "r"((uint32_t)L::TMEM_COLS) : "memory");
  }
}

}  // namespace molten
