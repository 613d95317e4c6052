// Row engine: the scaffolding that every generated row / elementwise kernel
// is built on.  A row of `cols` elements is split into slots of VEC elements;
// a team of TPC threads in each of CL CTAs of a cluster owns one row, thread
// t of CTA rank r holding slots  j = (r * TPC + t) + k * (TPC * CL),
// k = 0 .. NV-1, so that a warp touches 32 consecutive slots per k.
// A CTA runs RPC such teams side by side (RPC rows at a time).
//
// The generated code keeps its slots in registers, so a row is read from
// HBM once; reductions go warp shuffle -> shared memory -> (cluster) DSMEM.
#pragma once

#include "molten/common.cuh"

namespace molten {

#define MOLTEN_MAX_IO 8

// Kernel parameter block of every row / elementwise kernel.  Mirrored by
// `molten_row_args` in include/molten_rt.h and by the ctypes structure in
// molten_b200/_capi.py.
struct RowArgs {
  const void* in[MOLTEN_MAX_IO];   // external inputs, kernel order
  void* out[MOLTEN_MAX_IO];        // outputs, kernel order
  long long rows;                  // rows handled by this launch
  long long row_offset;            // global index of this launch's row 0
  long long cols;                  // elements per row (must equal COLS)
  int* status;                     // wait-timeout bits (bounded waits); may be null
};

// ------------------------------------------------------------ reductions
struct OpSum {
  static constexpr float identity = 0.0f;
  __device__ __forceinline__ float operator()(float a, float b) const { return a + b; }
};
struct OpMax {
  static constexpr float identity = -INFINITY;
  __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
struct OpMin {
  static constexpr float identity = INFINITY;
  __device__ __forceinline__ float operator()(float a, float b) const { return fminf(a, b); }
};

__host__ __device__ constexpr int pow2_ceil(int x) { return x <= 1 ? 1 : 2 * pow2_ceil((x + 1) / 2); }

__device__ __forceinline__ unsigned cluster_ctarank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
// arrive without release semantics: for barriers that hand over no data
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem(const float* local, unsigned rank) {
  unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(local)), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// ------------------------------------------- per-thread row staging (stream)
// In the persistent "stream" form of a row kernel every thread copies its
// own slots of the rows ahead into its own shared-memory lanes with
// cp.async (16 bytes per copy, L1 bypassed), one commit group per row.
// Only the issuing thread reads what it copied, so cp.async.wait_group is
// the whole synchronisation; no registers are held by the copies in flight.
__device__ __forceinline__ uint32_t shared_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" :: "r"(dst), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory");
}
// Bulk form (one CTA per row): one thread copies a whole row of a staged
// operand with one untiled bulk copy into this CTA's shared memory,
// completing bytes on the stage's mbarrier.  Source and size are 16-byte
// multiples.
__device__ __forceinline__ void bulk_row_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                             uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
enum RowStageStatus { kRowTimeoutStage = 256 };

// Zero tail of a masked row: `bytes` zero bytes at global `dst` (both
// 16-byte multiples), written by the TMA engine from a zero-filled shared
// buffer of `zbytes` at `zsrc` (bulk stores of up to zbytes each, one bulk
// group).  The issuing thread goes on at once; bulk_zero_drain() before it
// exits waits for all of them.
__device__ __forceinline__ void bulk_zero_tail(void* dst, long long bytes, uint32_t zsrc,
                                               uint32_t zbytes) {
  char* p = static_cast<char*>(dst);
  while (bytes > 0) {
    const uint32_t n = bytes < (long long)zbytes ? (uint32_t)bytes : zbytes;
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 :: "l"(p), "r"(zsrc), "r"(n) : "memory");
    p += n;
    bytes -= n;
  }
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_zero_drain() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Fill `bytes` (a multiple of 16 * blockDim.x) of shared memory at `zbuf`
// with zeros and make them visible to the TMA engine; every thread calls
// it, followed by a barrier.
__device__ __forceinline__ void zero_shared_for_bulk(uint4* zbuf, int bytes) {
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) zbuf[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T, int VEC>
__device__ __forceinline__ Slot<T, VEC> lds_slot16(uint32_t addr) {
  static_assert(sizeof(T) * VEC == 16, "staged slots are 16 bytes");
  Slot<T, VEC> s;
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr) : "memory");
  *reinterpret_cast<uint4*>(&s) = r;
  return s;
}

// ------------------------------------------------- push-style cluster exchange
// A persistent row kernel stores row n's outputs right before row n+1's
// reductions.  A barrier.cluster round there would be a release fence behind
// those stores; instead each CTA pushes its partials into its peers' shared
// memory with st.async, which completes bytes on the receiving CTA's
// mbarrier, and waits only on its own barrier.  One barrier per exchange
// area, armed once per use by thread 0 of the receiving CTA; areas alternate
// with the row's parity, so phase (use count & 1) of an area never mixes
// rows.  Waits are bounded by a number of polls; on timeout the CTA raises a
// shared abort flag, skips all later waits, and the kernel reports
// kRowTimeoutExchange in *status when it ends (a timer-bounded loop or a
// status atomic inside the wait costs ~48 registers in the row kernels).
enum RowExchangeStatus { kRowTimeoutExchange = 128 };

#ifndef MOLTEN_ROW_WAIT_TRIES
#define MOLTEN_ROW_WAIT_TRIES (1u << 22)   // try_wait polls before a wait gives up
#endif

struct ClusterExchange {
  float* slots;          // [areas][RPC][CL][nr_max] floats
  uint32_t bars;         // shared address of the areas' mbarriers (8 bytes each)
  int nr_max;            // slot stride (largest NR of any call)
  volatile int* abort;   // shared flag: a wait timed out
};

__device__ __forceinline__ uint32_t mapa_u32(uint32_t local, unsigned rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async_f32(uint32_t remote, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];"
               :: "r"(remote), "f"(v), "r"(remote_bar) : "memory");
}
__device__ __forceinline__ void xch_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void xch_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void xch_arm(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool xch_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Wait for the phase of `parity` to complete; false on timeout (or when an
// earlier wait of this CTA timed out).
__device__ __forceinline__ bool xch_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (xch_try_wait(bar, parity)) return true;
  if (*abort) return false;
  for (uint32_t i = 0; i < MOLTEN_ROW_WAIT_TRIES; ++i)
    if (xch_try_wait(bar, parity)) return true;
  *abort = 1;
  return false;
}

template <int TPC, int RPC, int CL>
struct RowTeam {
  static constexpr int BLOCK = TPC * RPC;
  static constexpr int WPR = TPC >= 32 ? TPC / 32 : 1;   // warps per row team
  static_assert(TPC >= 32 ? TPC % 32 == 0 : (32 % TPC == 0), "team size must tile a warp");
  static_assert(BLOCK % 32 == 0 && BLOCK <= 1024, "bad block size");

  // shared-memory floats needed by `reduce` for NR values in `passes` passes
  __host__ __device__ static constexpr int smem_floats(int nr, int calls) {
    return RPC * WPR * nr + (CL > 1 ? calls * RPC * nr : 0);
  }

  int t;            // thread index inside the team
  int team;         // team index inside the CTA
  int rank;         // CTA rank inside the cluster
  long long row;    // local row index (may be >= rows for idle teams)
  bool row_ok;

  __device__ __forceinline__ RowTeam(long long rows, long long row_base) {
    t = threadIdx.x % TPC;
    team = threadIdx.x / TPC;
    rank = CL > 1 ? static_cast<int>(cluster_ctarank()) : 0;
    const long long cta_row0 = row_base + (long long)(blockIdx.x / CL) * RPC;
    row = cta_row0 + team;
    row_ok = row < rows;
  }

  // slot index of this thread's k-th slot (a row has < 2^31 slots)
  __device__ __forceinline__ int slot(int k) const {
    return (rank * TPC + t) + k * (TPC * CL);
  }

  // Levels 1-2 of every all-reduce: inside the warp (or sub-warp team), then
  // across the warps of the team through `smem` (RPC * WPR * NR floats).
  // Every thread of the CTA must call this (idle teams pass neutral values).
  template <int NR, class Op>
  __device__ __forceinline__ void reduce_cta(float (&v)[NR], Op op, float* smem) const {
    constexpr int W = TPC < 32 ? TPC : 32;
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1)
#pragma unroll
      for (int i = 0; i < NR; ++i) v[i] = op(v[i], __shfl_xor_sync(0xffffffffu, v[i], off));
    if constexpr (WPR > 1) {
      const int warp = t / 32, lane = t % 32;
      float* red = smem + team * WPR * NR;
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < NR; ++i) red[warp * NR + i] = v[i];
      }
      __syncthreads();
      if constexpr (WPR <= 4) {
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          float a = red[i];
#pragma unroll
          for (int w = 1; w < WPR; ++w) a = op(a, red[w * NR + i]);
          v[i] = a;
        }
      } else {
        // lane l takes warp (l mod P)'s partial, then a butterfly over each
        // aligned group of P lanes, so that every lane ends with the total
        constexpr int P = pow2_ceil(WPR);
        const int src = lane % P;
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          float a = src < WPR ? red[src * NR + i] : Op::identity;
#pragma unroll
          for (int off = P / 2; off > 0; off >>= 1) a = op(a, __shfl_xor_sync(0xffffffffu, a, off));
          v[i] = a;
        }
      }
      __syncthreads();   // the area is reused by the next call
    }
  }

  // All-reduce NR values across the row team (all CTAs of the cluster).
  // `smem` must hold smem_floats(NR, calls) floats; `pass` selects the
  // cluster exchange area so consecutive calls never overwrite a value a
  // peer CTA may still be reading.  The cluster level is a
  // barrier.cluster round (release/acquire).
  template <int NR, class Op>
  __device__ __forceinline__ void reduce(float (&v)[NR], Op op, float* smem, int pass) const {
    reduce_cta<NR>(v, op, smem);
    if constexpr (CL > 1) {
      float* part = smem + RPC * WPR * NR + pass * RPC * NR + team * NR;
      if (t == 0) {
#pragma unroll
        for (int i = 0; i < NR; ++i) part[i] = v[i];
      }
      cluster_arrive();
      cluster_wait();
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        float a = ld_dsmem(part + i, 0);
#pragma unroll
        for (int r = 1; r < CL; ++r) a = op(a, ld_dsmem(part + i, r));
        v[i] = a;
      }
    }
  }

  // Same, with the cluster level done by pushing (see ClusterExchange):
  // no barrier.cluster and so no release fence behind earlier global stores.
  template <int NR, class Op>
  __device__ __forceinline__ void reduce_push(float (&v)[NR], Op op, float* smem,
                                              const ClusterExchange& x, int area,
                                              uint32_t phase) const {
    reduce_cta<NR>(v, op, smem);
    if constexpr (CL > 1) {
      const float* slots = exchange<NR>(v, x, area, phase);
      float a[NR];
#pragma unroll
      for (int i = 0; i < NR; ++i) a[i] = rank == 0 ? v[i] : slots[i];
#pragma unroll
      for (int r = 1; r < CL; ++r)
#pragma unroll
        for (int i = 0; i < NR; ++i) a[i] = op(a[i], r == rank ? v[i] : slots[r * x.nr_max + i]);
#pragma unroll
      for (int i = 0; i < NR; ++i) v[i] = a[i];
    }
  }

  // (max, sum-of-exponentials) pair of one softmax row, combined across the
  // team: (m1, s1) + (m2, s2) = (M, s1 e^(m1-M) + s2 e^(m2-M)), M = max.
  // A side whose max is -inf (all its elements masked) contributes 0.
  __device__ __forceinline__ static void softmax_combine(float& m, float& s, float m2, float s2) {
    const float M = fmaxf(m, m2);
    const float a = (m == -INFINITY) ? 0.0f : s * fast_exp2((m - M) * MOLTEN_LOG2E);
    const float b = (m2 == -INFINITY) ? 0.0f : s2 * fast_exp2((m2 - M) * MOLTEN_LOG2E);
    m = M;
    s = a + b;
  }

  // Butterfly all-reduce of (max, sum of 2^((x - max) log2e)) pairs over
  // aligned groups of W lanes, in two phases: the max first, then each lane
  // rescales its own sum once to the common max and the sums are added --
  // one EX2 per lane instead of two per butterfly step (merging pairs step by
  // step, as softmax_combine does, costs 2 log2(W) EX2).  Every lane of a
  // group ends with the same bits (xor pairing: the same additions, only
  // commuted).
  template <int W>
  __device__ __forceinline__ static void softmax_butterfly(float& m, float& s) {
    float M = m;
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float S = (m == -INFINITY) ? 0.0f : s * fast_exp2((m - M) * MOLTEN_LOG2E);
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) S += __shfl_xor_sync(0xffffffffu, S, off);
    m = M;
    s = S;
  }

  // Levels 1-2 of the softmax pair reduction (2 floats per warp of `smem`).
  __device__ __forceinline__ void softmax_cta(float& m, float& s, float* smem) const {
    constexpr int W = TPC < 32 ? TPC : 32;
    softmax_butterfly<W>(m, s);
    if constexpr (WPR > 1) {
      const int warp = t / 32, lane = t % 32;
      float* red = smem + team * WPR * 2;
      if (lane == 0) {
        red[warp * 2] = m;
        red[warp * 2 + 1] = s;
      }
      __syncthreads();
      // lane l takes warp (l mod P)'s pair, then a butterfly over each
      // aligned group of P lanes, so that every lane ends with the total
      constexpr int P = pow2_ceil(WPR);
      const int src = lane % P;
      float M = src < WPR ? red[src * 2] : -INFINITY;
      float S = src < WPR ? red[src * 2 + 1] : 0.0f;
      softmax_butterfly<P>(M, S);
      m = M;
      s = S;
      __syncthreads();
    }
  }

  // All-reduce of one softmax (max, sum) pair per row, in the same three
  // levels as `reduce`.
  __device__ __forceinline__ void reduce_softmax(float& m, float& s, float* smem, int pass) const {
    softmax_cta(m, s, smem);
    if constexpr (CL > 1) {
      float* part = smem + RPC * WPR * 2 + pass * RPC * 2 + team * 2;
      if (t == 0) {
        part[0] = m;
        part[1] = s;
      }
      cluster_arrive();
      cluster_wait();
      float M = ld_dsmem(part, 0), S = ld_dsmem(part + 1, 0);
#pragma unroll
      for (int r = 1; r < CL; ++r) softmax_combine(M, S, ld_dsmem(part, r), ld_dsmem(part + 1, r));
      m = M;
      s = S;
    }
  }

  // Same, with the cluster level done by pushing.  Pairs are combined in
  // rank order in every CTA, so all CTAs of the cluster get identical bits.
  __device__ __forceinline__ void reduce_softmax_push(float& m, float& s, float* smem,
                                                      const ClusterExchange& x, int area,
                                                      uint32_t phase) const {
    softmax_cta(m, s, smem);
    if constexpr (CL > 1) {
      float v[2] = {m, s};
      const float* slots = exchange<2>(v, x, area, phase);
      float M = rank == 0 ? m : slots[0], S = rank == 0 ? s : slots[1];
#pragma unroll
      for (int r = 1; r < CL; ++r)
        softmax_combine(M, S, r == rank ? m : slots[r * x.nr_max],
                        r == rank ? s : slots[r * x.nr_max + 1]);
      m = M;
      s = S;
    }
  }

  // Push this team's NR values into slot `rank` of the team's area in every
  // peer CTA (st.async, completing bytes on the peer's mbarrier of the
  // area), then wait for the peers' values to land in this CTA's area.
  // Returns the team's CL slots (stride x.nr_max).  Thread 0 of the CTA arms
  // the area's barrier for RPC * (CL - 1) * NR * 4 bytes.
  template <int NR>
  __device__ __forceinline__ const float* exchange(const float (&v)[NR], const ClusterExchange& x,
                                                   int area, uint32_t phase) const {
    const uint32_t bar = x.bars + 8u * (uint32_t)area;
    float* slots = x.slots + ((area * RPC + team) * CL) * x.nr_max;
    if (threadIdx.x == 0) xch_arm(bar, (uint32_t)(RPC * (CL - 1) * NR * 4));
    if (t == 0) {
      const uint32_t mine = shared_addr(slots + rank * x.nr_max);
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        if (r == rank) continue;
        const uint32_t dst = mapa_u32(mine, (unsigned)r), rbar = mapa_u32(bar, (unsigned)r);
#pragma unroll
        for (int i = 0; i < NR; ++i) st_async_f32(dst + 4u * i, v[i], rbar);
      }
    }
    xch_wait(bar, phase, x.abort);
    return slots;
  }

  // A CTA of a cluster must not exit while a peer may still read its shared
  // memory: call once after the last `reduce`, before leaving the kernel.
  __device__ __forceinline__ void cluster_done_arrive() const {
    if constexpr (CL > 1) cluster_arrive();
  }
  __device__ __forceinline__ void cluster_done_wait() const {
    if constexpr (CL > 1) cluster_wait();
  }
};

}  // namespace molten
