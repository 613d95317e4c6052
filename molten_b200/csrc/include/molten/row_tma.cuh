// TMA-staged row engine: a persistent CTA per SM streams whole rows of the
// row-indexed operands into a STAGES-deep shared-memory ring with
// cp.async.bulk (the untiled TMA copy, into this CTA only) while NC consumer warps
// each take one row at a time, reduce it with warp shuffles and write the
// outputs with 16-byte stores.
//
//   warp 0        producer: one lane waits for a free stage, arms the stage's
//                 "full" mbarrier with the row's byte count and issues one
//                 bulk copy per staged operand;
//   warps 1..NC   consumers: local row j is handled by warp j % NC from
//                 stage j % STAGES; after its last shared-memory read the
//                 warp frees the stage through the stage's "empty" mbarrier.
//
// HBM sees one read of every staged byte; up to STAGES rows are in flight per
// SM independently of register pressure.  Every wait is bounded (on timeout
// the kernel sets a bit in *status and stops issuing/consuming rows).
#pragma once

#include "molten/common.cuh"
#include "molten/gemm_sm100.cuh"     // mbarrier helpers, smem_u32, timeouts
#include "molten/row_engine.cuh"     // RowArgs

namespace molten {

enum RowTmaStatus { kRowTimeoutFull = 16, kRowTimeoutEmpty = 32, kRowTimeoutDrain = 64 };

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

template <class R>
__device__ __forceinline__ void row_ring_init(const R& r, int stages) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(r.full(s), 1);
      mbar_init(r.empty(s), 1);
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

}  // namespace molten
