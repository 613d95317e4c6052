// TMA-staged row engine: a persistent CTA per SM streams whole rows of the
// row-indexed operands into a STAGES-deep shared-memory ring with
// cp.async.bulk (the untiled TMA copy, into this CTA only) while NC consumer
// teams of TW warps (one warp by default) each take one row at a time,
// reduce it with warp shuffles (and, for TW > 1, across the team's warps in
// shared memory) and write the outputs with 16-byte stores.
//
//   warp 0        producer: one lane waits for a free stage, arms the stage's
//                 "full" mbarrier with the row's byte count and issues one
//                 bulk copy per staged operand;
//   warps 1..     consumers: local row j is handled by team j % NC from
//                 stage j % STAGES; after its last shared-memory read each
//                 warp of the team arrives on the stage's "empty" mbarrier
//                 (TW arrivals free the stage).
//
// HBM sees one read of every staged byte; up to STAGES rows are in flight per
// SM independently of register pressure.  Every wait is bounded (on timeout
// the kernel sets a bit in *status and stops issuing/consuming rows).
#pragma once

#include "molten/common.cuh"
#include "molten/gemm_sm100.cuh"     // mbarrier helpers, smem_u32, timeouts
#include "molten/row_engine.cuh"     // RowArgs

namespace molten {

enum RowTmaStatus { kRowTimeoutFull = 16, kRowTimeoutEmpty = 32, kRowTimeoutDrain = 64,
                    kRowTimeoutTeam = 1024 };

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

template <typename T, int VEC>
__device__ __forceinline__ Slot<T, VEC> lds_slot(uint32_t addr) {
  Slot<T, VEC> s;
  constexpr int BYTES = sizeof(T) * VEC;
  static_assert(BYTES % 16 == 0, "staged slots are whole 16-byte vectors");
#pragma unroll
  for (int i = 0; i < BYTES / 16; ++i) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr + 16 * i));
    reinterpret_cast<uint4*>(&s)[i] = r;
  }
  return s;
}

template <int N>
__device__ __forceinline__ void warp_allreduce_sum(float (&v)[N]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], off);
}
template <int N>
__device__ __forceinline__ void warp_allreduce_max(float (&v)[N]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = fmaxf(v[i], __shfl_xor_sync(0xffffffffu, v[i], off));
}
template <int N>
__device__ __forceinline__ void warp_allreduce_min(float (&v)[N]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = fminf(v[i], __shfl_xor_sync(0xffffffffu, v[i], off));
}

// Shared-memory layout: STAGES stages of STAGE_BYTES, then CONST_BYTES of
// per-column operands (copied once per CTA), then full[S], empty[S] and the
// "constants landed" barrier.
template <int STAGES, int STAGE_BYTES, int CONST_BYTES = 0>
struct RowRing {
  static constexpr int CONST_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = CONST_OFFSET + CONST_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFFSET + (2 * STAGES + 1) * 8 + 16 + 128;
  uint32_t base;      // shared address of stage 0 (128-byte aligned)
  uint32_t bars;
  volatile int* abort_flag;
  __device__ __forceinline__ uint32_t stage(int s) const { return base + (uint32_t)(s * STAGE_BYTES); }
  __device__ __forceinline__ uint32_t consts() const { return base + (uint32_t)CONST_OFFSET; }
  __device__ __forceinline__ uint32_t full(int s) const { return bars + 8u * s; }
  __device__ __forceinline__ uint32_t empty(int s) const { return bars + 8u * (STAGES + s); }
  __device__ __forceinline__ uint32_t consts_full() const { return bars + 8u * (2 * STAGES); }
};

template <int STAGES, int STAGE_BYTES, int CONST_BYTES = 0>
__device__ __forceinline__ RowRing<STAGES, STAGE_BYTES, CONST_BYTES> row_ring_carve(uint8_t* raw) {
  typedef RowRing<STAGES, STAGE_BYTES, CONST_BYTES> R;
  R r;
  const uintptr_t p = (reinterpret_cast<uintptr_t>(raw) + 127) & ~uintptr_t(127);
  uint8_t* b = reinterpret_cast<uint8_t*>(p);
  r.base = smem_u32(b);
  r.bars = smem_u32(b + R::BAR_OFFSET);
  r.abort_flag = reinterpret_cast<volatile int*>(b + R::BAR_OFFSET + (2 * STAGES + 1) * 8);
  return r;
}

// empty_count: arrivals that free a stage (the warps of the team that
// consumes it).
template <class R>
__device__ __forceinline__ void row_ring_init(const R& r, int stages, int empty_count = 1) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(r.full(s), 1);
      mbar_init(r.empty(s), (uint32_t)empty_count);
    }
    mbar_init(r.consts_full(), 1);
    *r.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
}

__device__ __forceinline__ void row_ring_fail(volatile int* abort_flag, int* status, int code) {
  *abort_flag = 1;
  if (status) atomicOr(status, code);
}

// ------------------------------------------------------------ warp teams
// With TW > 1 a row is consumed by a team of TW warps (TW * 32 threads,
// slot j of the row owned by team thread j % (TW * 32)).  After each warp
// has reduced its lanes with shuffles, the team combines the TW warp
// partials through shared memory: lane 0 of every warp writes its partials
// and arrives on the team's mbarrier, every lane waits (bounded) for the
// phase and sums the TW partials in warp order, so every warp of the team
// holds the same, deterministic value.  Reduction calls alternate between
// two (buffer, mbarrier) pairs: a warp can only overwrite buffer b for
// call c + 2 after every warp has arrived for call c + 1, i.e. after every
// warp has read call c's partials.  On a wait timeout the function
// returns false (the caller abandons the row loop) so no wait is endless.
struct TeamRed {
  float* buf;          // [2][TW][N] floats of this team
  uint32_t bars;       // 2 mbarriers of this team (TW arrivals each)
  uint32_t calls;      // reductions done so far (same in every warp of the team)
};

template <int OP>
__device__ __forceinline__ float red_op(float a, float b) {
  if constexpr (OP == 0) return a + b;
  else if constexpr (OP == 1) return fmaxf(a, b);
  else return fminf(a, b);
}

template <int OP, int N, int TW>
__device__ __forceinline__ bool team_allreduce(float (&v)[N], TeamRed& tr, int tw, int lane) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = red_op<OP>(v[i], __shfl_xor_sync(0xffffffffu, v[i], off));
  if constexpr (TW == 1) {
    return true;
  } else {
    const uint32_t b = tr.calls & 1u, ph = (tr.calls >> 1) & 1u;
    float* buf = tr.buf + b * (TW * N);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < N; ++i) buf[tw * N + i] = v[i];
      mbar_arrive(tr.bars + 8u * b);
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait(tr.bars + 8u * b, ph) ? 1 : 0) != 0;
    ++tr.calls;
    if (!ok) return false;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float acc = buf[i];
#pragma unroll
      for (int t = 1; t < TW; ++t) acc = red_op<OP>(acc, buf[t * N + i]);
      v[i] = acc;
    }
    return true;
  }
}

// Team barriers: 2 per team, initialised by thread 0 before the CTA's first
// __syncthreads.
__device__ __forceinline__ void team_bars_init(uint32_t bars, int teams, int tw) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * teams; ++i) mbar_init(bars + 8u * i, (uint32_t)tw);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
}

}  // namespace molten
