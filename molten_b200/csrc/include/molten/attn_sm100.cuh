// Fused attention scores on sm_100a: P = softmax(Q K^T * scale) over the
// last dim, for a stack of `batch` independent problems (heads) with
// Q [batch*m, d] and K [batch*n, d] row-major (K is read K-major: no
// transpose is materialised), P [batch*m, n] in bf16 or fp16.
//
// One CTA owns work items (head h, 128-row block of Q) in a persistent loop
// and runs two passes over the item's n columns, recomputing Q K^T on the
// tensor cores instead of storing fp32 scores:
//
//   pass 0   per row (one epilogue thread = one row = one TMEM lane): online
//            max and sum of 2^(t - max) over all columns, t = s * scale*log2(e);
//   pass 1   p = 2^(t - max) / sum, rounded once and stored.
//
//   warp 0      TMA producer: the item's Q tile (d/64 boxes {64, 128}) into
//               a resident area, then per pass and column block the K tiles
//               ({64, BN} boxes of K's rows) through a STAGES-deep ring;
//   warp 1      TMEM owner + MMA issuer (tcgen05.mma.cta_group::1.kind::f16,
//               fp32 accumulators double-buffered in TMEM);
//   warps 4..7  epilogue (TMEM lane quarter = warp % 4).  Pass-1 rows go to
//               HBM either through a per-warp staging tile and a TMA store
//               (32 rows x 32 columns, 64-byte swizzle: conflict-free
//               row-per-thread writes, full-line global writes) or, where a
//               box could cross into another head's rows, by direct stores.
//
// HBM sees Q and K about twice (L2 holds K across a head's row blocks) and
// P once; the fp32 score matrix of the two-kernel form never exists.  Every
// mbarrier wait is bounded (molten/gemm_sm100.cuh); on timeout the CTA sets
// a status bit, stops, drains its copies, frees TMEM and returns.
#pragma once

#include "molten/gemm_sm100.cuh"

namespace molten {

struct alignas(64) AttnArgs {
  CUtensorMap tmap_q;              // Q [batch*m, d], box {64, 128}, 128B swizzle
  CUtensorMap tmap_k;              // K [batch*n, d], box {64, BN}, 128B swizzle
  CUtensorMap tmap_p;              // P [batch*m, n], box {32, 32}, 64B swizzle (TMA stores)
  void* out;                       // P
  long long m, n, d;               // one problem: P[m, n] = softmax(Q[m, d] K[n, d]^T)
  long long row_offset;            // unused (no row-dependent terms)
  int* status;                     // error bits (may be null)
  int batch;                       // stacked problems (0 or 1: one)
};

enum AttnStatus { kAttnTimeout = 512 };

template <int BN_, int DCH_, int STAGES_>
struct AttnLayout {
  static constexpr int BM = 128, BN = BN_, DCH = DCH_, STAGES = STAGES_;
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, a multiple of 64");
  static_assert(DCH >= 1 && DCH <= 4, "d must be at most 256");
  static constexpr int Q_CHUNK = BM * 128;                  // {64, 128} box, 128-byte rows
  static constexpr int Q_BYTES = DCH * Q_CHUNK;
  static constexpr int STAGE_BYTES = BN * 128;              // {64, BN} box of K
  static constexpr int OUT_TILE = 32 * 64;                  // 32 rows x 32 16-bit columns
  static constexpr int OUT_BYTES = 4 * 2 * OUT_TILE;        // 4 warps, double-buffered
  static constexpr int TMEM_COLS = (2 * BN <= 128) ? 128 : ((2 * BN <= 256) ? 256 : 512);
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2], q_full, q_empty, done
  static constexpr int NUM_BARS = 2 * STAGES + 7;
  static constexpr int OUT_OFFSET = Q_BYTES + STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = OUT_OFFSET + OUT_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFFSET + NUM_BARS * 8 + 16 + 1024;
  static constexpr int THREADS = 256;
  static constexpr int EPI_WARP0 = 4, EPI_WARPS = 4;
};

template <class L> struct AttnBars {
  uint32_t base;
  __device__ __forceinline__ explicit AttnBars(uint32_t b) : base(b) {}
  __device__ __forceinline__ uint32_t full(int i) const { return base + 8u * i; }
  __device__ __forceinline__ uint32_t empty(int i) const { return base + 8u * (L::STAGES + i); }
  __device__ __forceinline__ uint32_t acc_full(int b) const { return base + 8u * (2 * L::STAGES + b); }
  __device__ __forceinline__ uint32_t acc_empty(int b) const { return base + 8u * (2 * L::STAGES + 2 + b); }
  __device__ __forceinline__ uint32_t q_full() const { return base + 8u * (2 * L::STAGES + 4); }
  __device__ __forceinline__ uint32_t q_empty() const { return base + 8u * (2 * L::STAGES + 5); }
  __device__ __forceinline__ uint32_t done() const { return base + 8u * (2 * L::STAGES + 6); }
};

struct AttnShared {
  uint8_t* q;              // 1024-aligned resident Q tile
  uint8_t* ring;           // K stages
  uint8_t* outs;           // epilogue staging tiles
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
    for (int i = 0; i < 2; ++i) { mbar_init(b.acc_full(i), 1); mbar_init(b.acc_empty(i), L::EPI_WARPS); }
    mbar_init(b.q_full(), 1);
    mbar_init(b.q_empty(), 1);
    mbar_init(b.done(), 1);
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

// ------------------------------------------------------ output primitives
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

// OT: bf16 or f16 output.  TMA_STORE: pass-1 rows leave through the staging
// tiles and tmap_p (the caller guarantees that no 32-row box of a quarter
// whose first row is in [0, m) reaches another head's rows: m % 32 == 0 or
// batch == 1); else direct stores, 16 bytes at a time when ROWS_ALIGNED
// (n * 2 % 16 == 0), element by element otherwise.  C2 = scale * log2(e).
template <class L, bool F16IN, typename OT, bool TMA_STORE, bool ROWS_ALIGNED>
__device__ __forceinline__ void attn_roles(const AttnShared& s, const AttnArgs& args, float C2) {
  tc_fence_after();
  const int tid = gemm_tid(), warp = tid / 32, lane = tid % 32;
  const uint32_t tmem = *s.tmem_slot;
  const AttnBars<L> bar(s.bars);
  const long long MB = (args.m + L::BM - 1) / L::BM;
  const int NB = (int)((args.n + L::BN - 1) / L::BN);
  const long long T = (args.batch > 1 ? args.batch : 1) * MB;     // work items

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t st = 0, ph = 0, qph = 0;
      long long issued = 0;
      bool q_issued = false;
      for (long long it = blockIdx.x; it < T && !*s.abort_flag; it += gridDim.x) {
        const int h = (int)(it / MB), mb = (int)(it - (long long)h * MB);
        if (!mbar_wait(bar.q_empty(), qph ^ 1u)) { attn_fail(s, args); break; }
        qph ^= 1u;
        mbar_expect_tx(bar.q_full(), (uint32_t)L::Q_BYTES);
#pragma unroll
        for (int kc = 0; kc < L::DCH; ++kc)
          tma_load_2d(smem_u32(s.q + kc * L::Q_CHUNK), &args.tmap_q, bar.q_full(), kc * 64,
                      (int)(h * args.m) + mb * L::BM);
        q_issued = true;
        bool ok = true;
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int nb = 0; nb < NB && ok; ++nb) {
#pragma unroll 1
            for (int kc = 0; kc < L::DCH; ++kc) {
              if (!mbar_wait(bar.empty(st), ph ^ 1u)) { attn_fail(s, args); ok = false; break; }
              if (*s.abort_flag) { ok = false; break; }
              mbar_expect_tx(bar.full(st), (uint32_t)L::STAGE_BYTES);
              tma_load_2d(smem_u32(s.ring + st * L::STAGE_BYTES), &args.tmap_k, bar.full(st),
                          kc * 64, (int)(h * args.n) + nb * L::BN);
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
          if (!mbar_wait(bar.full(ds), dp)) { if (args.status) atomicOr(args.status, kAttnTimeout); }
        }
        if (q_issued && !mbar_wait(bar.q_full(), qph ^ 1u)) {
          if (args.status) atomicOr(args.status, kAttnTimeout);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = umma_idesc<L::BM, L::BN, F16IN, true>();
      uint32_t st = 0, ph = 0, qph = 0;
      long long tile = 0;                          // accumulator buffers alternate per tile
      bool ok = true;
      for (long long it = blockIdx.x; it < T && ok && !*s.abort_flag; it += gridDim.x) {
        if (!mbar_wait(bar.q_full(), qph)) { attn_fail(s, args); break; }
        qph ^= 1u;
        tc_fence_after();
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int nb = 0; nb < NB && ok; ++nb, ++tile) {
            const int b = (int)(tile & 1);
            const uint32_t acc_ph = (uint32_t)((tile >> 1) & 1);
            if (!mbar_wait(bar.acc_empty(b), acc_ph ^ 1u)) { attn_fail(s, args); ok = false; break; }
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(b * L::BN);
            for (int kc = 0; kc < L::DCH; ++kc) {
              if (!mbar_wait(bar.full(st), ph)) { attn_fail(s, args); ok = false; break; }
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
      if (!mbar_wait(bar.done(), 0u)) { if (args.status) atomicOr(args.status, kAttnTimeout); }
    }
  } else if (warp >= L::EPI_WARP0 && warp < L::EPI_WARP0 + L::EPI_WARPS) {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp % 4;
    const uint32_t stage0 = smem_u32(s.outs + quarter * 2 * L::OUT_TILE);
    int sbuf = 0;
    long long tile = 0;
    bool ok = true;
    for (long long it = blockIdx.x; it < T && ok; it += gridDim.x) {
      const int h = (int)(it / MB), mb = (int)(it - (long long)h * MB);
      const long long qrow0 = (long long)mb * L::BM + quarter * 32;   // quarter's first row in the head
      const long long mrow = qrow0 + lane;
      const long long row = (long long)h * args.m + mrow;
      float mx = -INFINITY, sum = 0.0f, rinv = 0.0f;
      for (int pass = 0; pass < 2 && ok; ++pass) {
        for (int nb = 0; nb < NB; ++nb, ++tile) {
          const int b = (int)(tile & 1);
          const uint32_t acc_ph = (uint32_t)((tile >> 1) & 1);
          const bool got = mbar_wait(bar.acc_full(b), acc_ph);
          if (!__all_sync(0xffffffffu, got ? 1 : 0)) {
            if (lane == 0) attn_fail(s, args);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < L::BN / 32; ++c) {
            const long long col0 = (long long)nb * L::BN + 32 * c;
            if (col0 >= args.n) break;                                   // warp-uniform
            const int valid = (int)(args.n - col0 < 32 ? args.n - col0 : 32);
            float acc[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * L::BN + c * 32), acc);
            if (pass == 0) {
              float cm = -INFINITY;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                acc[i] = i < valid ? acc[i] * C2 : -INFINITY;
                cm = fmaxf(cm, acc[i]);
              }
              const float mn = fmaxf(mx, cm);                            // finite: valid >= 1
              float add = 0.0f;
#pragma unroll
              for (int i = 0; i < 32; ++i) add += fast_exp2(acc[i] - mn);   // 2^-inf = 0
              sum = sum * fast_exp2(mx - mn) + add;                      // 0 * 2^-inf on the first chunk
              mx = mn;
              continue;
            }
            float p[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) p[i] = fast_exp2(fmaf(acc[i], C2, -mx)) * rinv;
            if constexpr (TMA_STORE) {
              if (qrow0 >= args.m) continue;                             // warp-uniform
              const uint32_t tile_addr = stage0 + (uint32_t)(sbuf * L::OUT_TILE);
              if (lane == 0) bulk_wait_read<1>();                        // this buffer's last store read it
              __syncwarp();
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                Slot<OT, 8> sl;
                pack_slot<OT, 8>(sl, *reinterpret_cast<const float(*)[8]>(&p[8 * q]));
                const uint32_t chunk = (uint32_t)(q ^ ((lane >> 1) & 3));
                st_shared_v4(tile_addr + (uint32_t)lane * 64u + chunk * 16u,
                             *reinterpret_cast<const uint4*>(&sl));
              }
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&args.tmap_p, tile_addr, (int)col0, (int)(h * args.m + qrow0));
                bulk_commit();
              }
              sbuf ^= 1;
            } else {
              if (mrow >= args.m) continue;
              OT* dst = static_cast<OT*>(args.out) + row * args.n + col0;
              if (ROWS_ALIGNED && valid == 32) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  Slot<OT, 8> sl;
                  pack_slot<OT, 8>(sl, *reinterpret_cast<const float(*)[8]>(&p[8 * q]));
                  store_slot<kStoreDefault, OT, 8>(dst + 8 * q, sl);
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) if (i < valid) dst[i] = from_f32<OT>(p[i]);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar.acc_empty(b));
          if (__any_sync(0xffffffffu, *s.abort_flag ? 1 : 0)) { ok = false; break; }
        }
        rinv = 1.0f / sum;                                               // sum >= 1 (the max term)
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
