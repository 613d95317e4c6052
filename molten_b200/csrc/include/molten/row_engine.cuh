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
  int* status;                     // unused by row kernels; may be null
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

  // All-reduce NR values across the row team (all CTAs of the cluster).
  // Every thread of the CTA must call this (idle teams pass neutral values).
  // `smem` must hold smem_floats(NR, passes) floats; `pass` selects the
  // cluster exchange area so consecutive passes never overwrite a value a
  // peer CTA may still be reading.
  template <int NR, class Op>
  __device__ __forceinline__ void reduce(float (&v)[NR], Op op, float* smem, int pass) const {
    // 1) inside the warp (or the sub-warp team)
    constexpr int W = TPC < 32 ? TPC : 32;
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1)
#pragma unroll
      for (int i = 0; i < NR; ++i) v[i] = op(v[i], __shfl_xor_sync(0xffffffffu, v[i], off));
    // 2) across the warps of the team
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
      __syncthreads();   // the area is reused by the next pass
    }
    // 3) across the CTAs of the cluster
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

  // All-reduce of one softmax (max, sum) pair per row, in the same three
  // levels as `reduce` (uses 2 floats per warp / per CTA of `smem`).
  __device__ __forceinline__ void reduce_softmax(float& m, float& s, float* smem, int pass) const {
    constexpr int W = TPC < 32 ? TPC : 32;
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
      softmax_combine(m, s, m2, s2);
    }
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
#pragma unroll
      for (int off = P / 2; off > 0; off >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, M, off);
        const float s2 = __shfl_xor_sync(0xffffffffu, S, off);
        softmax_combine(M, S, m2, s2);
      }
      m = M;
      s = S;
      __syncthreads();
    }
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
