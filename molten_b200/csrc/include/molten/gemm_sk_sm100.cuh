// Stream-K tcgen05 GEMM for sm_100a: for GEMMs with fewer output tiles than
// SMs (decode-size M), the tiles x k-blocks iteration space is cut into one
// equal, contiguous range per persistent CTA, so every SM streams the same
// share of B instead of some SMs idling.  A CTA's range covers whole tiles
// (epilogue as in molten/gemm_sm100.cuh) and/or parts of tiles ("segments").
// The CTAs whose segments share a tile never wait for one another: each
// writes its fp32 partial tile to its own workspace slot, publishes it
// (fence, then an arrival on the tile's counter), and the CTA that arrives
// last sums the tile's slots in slot order -- the same order whoever is last,
// so results are deterministic -- applies the epilogue, stores C and resets
// the counter to 0 for the next call.
//
// Roles and barriers as in gemm_roles (TMA producer warp 0, MMA issuer
// warp 1, epilogue warps 4..7), iterating the CTA's segments instead of
// whole tiles; two more mbarriers let the four epilogue warps agree on who
// arrived last.  Every wait is bounded.
#pragma once

#include "molten/gemm_sm100.cuh"

namespace molten {

// Shared-memory tail of a stream-K CTA, after the layout's barrier area.
struct SkShared {
  uint32_t rdv_written;        // the 4 epilogue warps wrote (and fenced) their partial rows
  uint32_t rdv_decided;        // the counter was bumped; `last` is set
  volatile int* last;          // this CTA sums the tile
};
static constexpr int kSkSmemExtra = 64;   // bytes a stream-K kernel adds to the layout's

template <class L>
__device__ __forceinline__ SkShared sk_carve(const GemmShared& s) {
  SkShared k;
  const uint32_t base = smem_u32(s.tmem_slot) + 16u;          // past tmem_slot / abort flag
  k.rdv_written = base;
  k.rdv_decided = base + 8u;
  k.last = reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(s.tmem_slot) + 32);
  return k;
}

template <class L>
__device__ __forceinline__ void gemm_sk_init(const GemmShared& s, const GemmArgs& args) {
  gemm_init<L>(s, args);
  if (gemm_tid() == 0) {
    const SkShared k = sk_carve<L>(s);
    mbar_init(k.rdv_written, L::EPI_WARPS);
    mbar_init(k.rdv_decided, L::EPI_WARPS);
    *k.last = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
}

// First iteration of CTA c's range of I iterations over G CTAs.
__device__ __forceinline__ long long sk_lo(long long c, long long I, long long G) { return c * I / G; }
// The CTA whose range holds iteration x.
__device__ __forceinline__ long long sk_owner(long long x, long long I, long long G) {
  long long c = x * G / I;
  while (c + 1 < G && sk_lo(c + 1, I, G) <= x) ++c;
  while (c > 0 && sk_lo(c, I, G) > x) --c;
  return c;
}

// Segment j of this CTA's range: tile t, k-blocks [kb0, kb1).  Returns
// false past the range's end.
__device__ __forceinline__ bool sk_segment(long long lo, long long hi, long long KB, long long& it,
                                           long long& t, int& kb0, int& kb1) {
  if (it >= hi) return false;
  t = it / KB;
  kb0 = (int)(it - t * KB);
  const long long left = hi - it;
  kb1 = (int)((KB - kb0) < left ? KB : kb0 + left);
  it += kb1 - kb0;
  (void)lo;
  return true;
}

// The segments of this CTA, in order: with SPLITS == 0 its stream-K range;
// with SPLITS = S, split-K units u = blockIdx.x + j * gridDim.x of the
// (split s = u / T, tile t = u % T) space -- k-blocks [s*KB/S, (s+1)*KB/S)
// -- so the CTAs running together read the same one or two k-regions of B
// (DRAM rows shared across CTAs).  `slot` is the segment's workspace slot
// and `nseg` the tile's segment count.
template <int SPLITS>
struct SkWalk {
  long long T, KB, I, G, lo, hi, it, u;
  __device__ __forceinline__ SkWalk(long long T_, long long KB_, long long G_) : T(T_), KB(KB_), G(G_) {
    I = T * KB;
    lo = sk_lo(blockIdx.x, I, G);
    hi = sk_lo((long long)blockIdx.x + 1, I, G);
    it = lo;
    u = blockIdx.x;
  }
  __device__ __forceinline__ bool next(long long& t, int& kb0, int& kb1, int& slot, int& nseg) {
    if constexpr (SPLITS > 0) {
      if (u >= T * SPLITS) return false;
      const long long sp = u / T;
      t = u - sp * T;
      kb0 = (int)(sp * KB / SPLITS);
      kb1 = (int)((sp + 1) * KB / SPLITS);
      slot = (int)sp;
      nseg = SPLITS;
      u += G;
      return true;
    } else {
      if (!sk_segment(lo, hi, KB, it, t, kb0, kb1)) return false;
      const long long c_first = sk_owner(t * KB, I, G);
      slot = (int)(blockIdx.x - c_first);
      nseg = (int)(sk_owner((t + 1) * KB - 1, I, G) - c_first + 1);
      return true;
    }
  }
};

// MAXSEG: workspace slots per tile (the most CTAs that share one tile).
template <class L, bool F16IN, class Epi, bool B_KMAJOR, int MAXSEG, int SPLITS = 0>
__device__ __forceinline__ void gemm_sk_roles(const GemmShared& s, const GemmArgs& args) {
  tc_fence_after();
  const int tid = gemm_tid(), warp = tid / 32, lane = tid % 32;
  const uint32_t tmem = *s.tmem_slot;
  const Bars<L> bar(s);
  const long long MB = (args.m + L::BM - 1) / L::BM;
  const long long NB = (args.n + L::BN - 1) / L::BN;
  const long long T = (args.batch > 1 ? args.batch : 1) * MB * NB;
  const long long KB = (args.k + L::BK - 1) / L::BK;

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t st = 0, ph = 0;
      long long issued = 0, t;
      int kb0, kb1, slot, nseg;
      SkWalk<SPLITS> walk(T, KB, gridDim.x);
      while (!*s.abort_flag && walk.next(t, kb0, kb1, slot, nseg)) {
        int m0, n0, h;
        gemm_tile_coords<L>(t, MB, NB, m0, n0, h);
        const int a_row = (int)(h * args.m) + m0;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(bar.empty(st), ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutEmpty); ok = false; break; }
          if (*s.abort_flag) { ok = false; break; }
          const uint32_t a_dst = smem_u32(s.tiles + st * L::STAGE_BYTES);
          const uint32_t b_dst = a_dst + L::A_BYTES;
          mbar_expect_tx(bar.full(st), (uint32_t)L::STAGE_BYTES);
          tma_load_2d(a_dst, &args.tmap_a, bar.full(st), kb * L::BK, a_row);
          if constexpr (B_KMAJOR) {
            tma_load_2d(b_dst, &args.tmap_b, bar.full(st), kb * L::BK, (int)(h * args.n) + n0);
          } else {
#pragma unroll
            for (int c = 0; c < L::BN / 64; ++c)
              tma_load_2d(b_dst + c * L::B_CHUNK_BYTES, &args.tmap_b, bar.full(st), n0 + 64 * c,
                          (int)(h * args.k) + kb * L::BK);
          }
          ++issued;
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
        if (!ok) break;
      }
      if (*s.abort_flag) {
        uint32_t ds = st, dp = ph;
        for (long long i = 0; i < issued && i < L::STAGES; ++i) {
          if (ds == 0) { ds = L::STAGES - 1; dp ^= 1u; } else { --ds; }
          if (!mbar_wait(bar.full(ds), dp)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = umma_idesc<L::BM, L::BN, F16IN, B_KMAJOR>();
      uint32_t st = 0, ph = 0;
      long long i = 0, t;
      int kb0, kb1, slot, nseg;
      bool ok = true;
      SkWalk<SPLITS> walk(T, KB, gridDim.x);
      while (ok && !*s.abort_flag && walk.next(t, kb0, kb1, slot, nseg)) {
        const int b = (int)(i & 1);
        const uint32_t acc_ph = (uint32_t)((i >> 1) & 1);
        ++i;
        if (!mbar_wait(bar.acc_empty(b), acc_ph ^ 1u)) { gemm_fail(s, args, kGemmTimeoutAcc); break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * L::BN);
        for (int kb = kb0; kb < kb1; ++kb) {
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
            umma_f16(d, ad, bd, IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          umma_commit(bar.empty(st));
          if (++st == (uint32_t)L::STAGES) { st = 0; ph ^= 1u; }
        }
        if (ok) umma_commit(bar.acc_full(b));
      }
      umma_commit(bar.done());
      if (!mbar_wait(bar.done(), 0u)) { if (args.status) atomicOr(args.status, kGemmTimeoutDrain); }
    }
  } else if (warp >= L::EPI_WARP0 && warp < L::EPI_WARP0 + L::EPI_WARPS) {
    // ------------------------------------------------------------- epilogue
    const SkShared sk = sk_carve<L>(s);
    const int quarter = warp % 4;                  // TMEM lanes 32*quarter .. +31
    const bool leader = (warp == L::EPI_WARP0) && lane == 0;
    long long i = 0, t;
    int kb0, kb1, slot, nseg;
    uint32_t nsplit = 0;                           // split segments handled (rendezvous phases)
    SkWalk<SPLITS> walk(T, KB, gridDim.x);
    while (walk.next(t, kb0, kb1, slot, nseg)) {
      const int b = (int)(i & 1);
      const uint32_t acc_ph = (uint32_t)((i >> 1) & 1);
      ++i;
      const bool got = mbar_wait(bar.acc_full(b), acc_ph);
      if (!__all_sync(0xffffffffu, got ? 1 : 0)) {
        if (lane == 0) gemm_fail(s, args, kGemmTimeoutAcc);
        break;
      }
      tc_fence_after();
      int m0, n0, h;
      gemm_tile_coords<L>(t, MB, NB, m0, n0, h);
      const long long mrow = (long long)m0 + quarter * 32 + lane;   // row of problem h
      const long long row = (long long)h * args.m + mrow;           // row of stacked C
      const bool whole = kb0 == 0 && kb1 == KB;
      float* part = args.work + ((t * MAXSEG + slot) * L::BM + quarter * 32 + lane) * (long long)L::BN;
#pragma unroll 1
      for (int c = 0; c < L::BN / 32; ++c) {
        float acc[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * L::BN + c * 32), acc);
        const long long col0 = (long long)n0 + 32 * c;
        if (whole) {
          if (col0 < args.n && mrow < args.m) Epi::apply(args, row, col0, acc);
        } else if (mrow < args.m) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(part + 32 * c + 4 * q) =
                make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.acc_empty(b));     // the accumulator is free again
      if (!whole) {
        // publish: every thread's partial rows reach the GPU before the
        // counter moves; the CTA that moves it to the tile's segment count
        // has everyone's rows
        __threadfence();
        __syncwarp();
        if (lane == 0) mbar_arrive(sk.rdv_written);
        bool okw = mbar_wait(sk.rdv_written, nsplit & 1u);
        if (leader) {
          int old = -1;
          if (okw) {
            old = atomicAdd(args.tile_count + t, 1);
            __threadfence();
          }
          *sk.last = (old == nseg - 1) ? 1 : 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(sk.rdv_decided);
        const bool okd = mbar_wait(sk.rdv_decided, nsplit & 1u);
        ++nsplit;
        if (!__all_sync(0xffffffffu, (okw && okd) ? 1 : 0)) {
          if (lane == 0) gemm_fail(s, args, kGemmTimeoutAcc);
          break;
        }
        const bool last = *sk.last != 0;
        if (last) {
          // every slot of the tile, in slot order, then the epilogue
          const float* base = args.work + ((t * MAXSEG) * L::BM + quarter * 32 + lane) * (long long)L::BN;
#pragma unroll 1
          for (int c = 0; c < L::BN / 32; ++c) {
            const long long col0 = (long long)n0 + 32 * c;
            if (col0 >= args.n || mrow >= args.m) continue;
            float acc[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
            for (int j = 0; j < nseg; ++j) {
              const float* src = base + (long long)j * L::BM * L::BN + 32 * c;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(src + 4 * q));
                acc[4 * q] += v.x; acc[4 * q + 1] += v.y; acc[4 * q + 2] += v.z; acc[4 * q + 3] += v.w;
              }
            }
            Epi::apply(args, row, col0, acc);
          }
          if (leader) args.tile_count[t] = 0;        // ready for the next call
        }
      }
      if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) break;
    }
  }
}

}  // namespace molten
