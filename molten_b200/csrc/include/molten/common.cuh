// Shared device helpers for every Molten sm_100a kernel: element types,
// 16-byte vector slots with cache-hinted loads/stores, fp32 conversions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

namespace molten {

typedef __nv_bfloat16 bf16;
typedef __half f16;

// ------------------------------------------- programmatic dependent launch
// Every generated kernel starts with this.  With the launch attribute
// (MOLTEN_LAUNCH_PDL) the next kernel of the stream may begin launching as
// soon as every CTA of this one is running, and this kernel waits here until
// the previous one has completed and its writes are visible -- before any
// global memory access, so no producer/consumer order is ever relaxed; what
// overlaps is launch processing, CTA scheduling and the prologue.  Both
// instructions are no-ops for a launch without the attribute.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------- conversion
__device__ __forceinline__ float to_f32(float v) { return v; }
// bf16 is the upper half of an fp32: widening is a 16-bit shift (integer
// pipe), exact, instead of a conversion instruction on the transcendental
// pipe that the exponentials of softmax already load.
__device__ __forceinline__ float to_f32(bf16 v) {
  return __uint_as_float(static_cast<uint32_t>(__bfloat16_as_ushort(v)) << 16);
}
__device__ __forceinline__ float to_f32(f16 v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 from_f32<bf16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ f16 from_f32<f16>(float v) { return __float2half_rn(v); }

// ------------------------------------------------------------------- slots
// A slot is VEC consecutive elements of one row, moved with the widest
// aligned access that fits (16, 8, 4 or 2 bytes; 32-byte slots use two
// 16-byte accesses).
template <typename T, int VEC>
struct alignas((sizeof(T) * VEC) >= 16 ? 16 : (sizeof(T) * VEC)) Slot {
  T v[VEC];
};

enum LoadHint { kLoadDefault = 0, kLoadStream = 1 };
enum StoreHint { kStoreDefault = 0, kStoreStream = 1 };

template <int HINT>
__device__ __forceinline__ uint4 ld16(const void* p) {
  uint4 r;
  if (HINT == kLoadStream) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  } else {
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  }
  return r;
}

template <int HINT>
__device__ __forceinline__ void st16(void* p, uint4 v) {
  if (HINT == kStoreStream) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  } else {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  }
}

template <int HINT, typename T, int VEC>
__device__ __forceinline__ Slot<T, VEC> load_slot(const T* p) {
  Slot<T, VEC> s;
  constexpr int BYTES = sizeof(T) * VEC;
  if constexpr (BYTES % 16 == 0) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i)
      reinterpret_cast<uint4*>(&s)[i] = ld16<HINT>(reinterpret_cast<const char*>(p) + 16 * i);
  } else if constexpr (BYTES == 8) {
    *reinterpret_cast<uint2*>(&s) = __ldg(reinterpret_cast<const uint2*>(p));
  } else if constexpr (BYTES == 4) {
    *reinterpret_cast<uint32_t*>(&s) = __ldg(reinterpret_cast<const unsigned int*>(p));
  } else {
    static_assert(BYTES == 2, "unsupported slot size");
    *reinterpret_cast<uint16_t*>(&s) = __ldg(reinterpret_cast<const unsigned short*>(p));
  }
  return s;
}

template <int HINT, typename T, int VEC>
__device__ __forceinline__ void store_slot(T* p, const Slot<T, VEC>& s) {
  constexpr int BYTES = sizeof(T) * VEC;
  if constexpr (BYTES % 16 == 0) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i)
      st16<HINT>(reinterpret_cast<char*>(p) + 16 * i, reinterpret_cast<const uint4*>(&s)[i]);
  } else if constexpr (BYTES == 8) {
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(&s);
  } else if constexpr (BYTES == 4) {
    *reinterpret_cast<uint32_t*>(p) = *reinterpret_cast<const uint32_t*>(&s);
  } else {
    *reinterpret_cast<uint16_t*>(p) = *reinterpret_cast<const uint16_t*>(&s);
  }
}

// Store a slot of VEC zeros: all-zero bits, +0.0 in every float format, so
// nothing is converted (masked-out softmax outputs).
template <int HINT, typename T, int VEC>
__device__ __forceinline__ void store_zero_slot(T* p) {
  constexpr int BYTES = sizeof(T) * VEC;
  if constexpr (BYTES % 16 == 0) {
#pragma unroll
    for (int i = 0; i < BYTES / 16; ++i)
      st16<HINT>(reinterpret_cast<char*>(p) + 16 * i, make_uint4(0u, 0u, 0u, 0u));
  } else if constexpr (BYTES == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(0u, 0u);
  } else if constexpr (BYTES == 4) {
    *reinterpret_cast<uint32_t*>(p) = 0u;
  } else {
    static_assert(BYTES == 2, "unsupported slot size");
    *reinterpret_cast<uint16_t*>(p) = 0;
  }
}

// Write VEC fp32 values into a slot of T, rounding to nearest even once.
template <typename T, int VEC>
__device__ __forceinline__ void pack_slot(Slot<T, VEC>& s, const float (&f)[VEC]) {
  if constexpr (sizeof(T) == 2 && VEC % 2 == 0) {
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      if constexpr (std::is_same<T, bf16>::value) {
        *reinterpret_cast<__nv_bfloat162*>(&s.v[e]) = __floats2bfloat162_rn(f[e], f[e + 1]);
      } else {
        *reinterpret_cast<__half2*>(&s.v[e]) = __floats2half2_rn(f[e], f[e + 1]);
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) s.v[e] = from_f32<T>(f[e]);
  }
}

// Clamp a 64-bit column limit into int range (limits outside [-1, 2^31-1]
// mask every / no column of any row the kernels can address).
__device__ __forceinline__ int clamp_col_limit(long long v) {
  return v < -1 ? -1 : (v > 2147483647LL ? 2147483647 : (int)v);
}

template <typename T>
__device__ __forceinline__ float load_scalar(const T* p) { return to_f32(p[0]); }

template <typename T>
__device__ __forceinline__ void store_scalar(T* p, float v) { p[0] = from_f32<T>(v); }

// 2^x with the MUFU.EX2 instruction (ex2.approx.ftz: about 2 ulp over the
// range softmax uses); e^(x - m) = 2^(x*log2e - m*log2e) is one FFMA + EX2.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
#define MOLTEN_LOG2E 1.4426950408889634f

// 2^x on the FMA pipe, for kernels whose EX2 unit is the bottleneck: Cody-
// Waite range reduction x = j + f, j = round(x) (adding 1.5 * 2^23 leaves
// round(x) in the low mantissa bits), f in [-1/2, 1/2]; 2^f by the cubic of
// least maximum relative error on that interval (Remez exchange, relative
// error 7.5e-5 -- enough for 16-bit results); 2^j added to the exponent
// field as an integer.  x is clamped at -126 so the exponent never wraps:
// results below 2^-126 come out as tiny values instead of 0.  x <= 1 here.
#define MOLTEN_EXP2_C0 0.9999280571937561f
#define MOLTEN_EXP2_C1 0.6932609677314758f
#define MOLTEN_EXP2_C2 0.2426111251115799f
#define MOLTEN_EXP2_C3 0.0551716685295105f
__device__ __forceinline__ float exp2_poly3(float x) {
  x = fmaxf(x, -126.0f);
  const float r = __fadd_rn(x, 12582912.0f);
  const float f = __fsub_rn(x, __fsub_rn(r, 12582912.0f));
  const float p = fmaf(fmaf(fmaf(MOLTEN_EXP2_C3, f, MOLTEN_EXP2_C2), f, MOLTEN_EXP2_C1), f,
                       MOLTEN_EXP2_C0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(r) << 23));
}

// 1/x with the MUFU.RCP instruction (rcp.approx.ftz: about 1 ulp); 1/inf = 0
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max of the 16-bit elements of a slot, two at a time
template <typename T, int VEC>
__device__ __forceinline__ float slot_max16(const Slot<T, VEC>& s, float m) {
  static_assert(sizeof(T) == 2 && VEC % 2 == 0, "16-bit slots");
  if constexpr (std::is_same<T, bf16>::value) {
    __nv_bfloat162 acc = *reinterpret_cast<const __nv_bfloat162*>(&s.v[0]);
#pragma unroll
    for (int e = 2; e < VEC; e += 2) acc = __hmax2(acc, *reinterpret_cast<const __nv_bfloat162*>(&s.v[e]));
    return fmaxf(m, fmaxf(__low2float(acc), __high2float(acc)));
  } else {
    __half2 acc = *reinterpret_cast<const __half2*>(&s.v[0]);
#pragma unroll
    for (int e = 2; e < VEC; e += 2) acc = __hmax2(acc, *reinterpret_cast<const __half2*>(&s.v[e]));
    return fmaxf(m, fmaxf(__low2float(acc), __high2float(acc)));
  }
}

// ------------------------------------------------------- elementwise math
// Every function computes in fp32.  PRECISE selects CUDA's full-precision
// library functions; otherwise the fast hardware intrinsics are used (the
// host picks fast math only when the output precision is 16-bit).
template <bool PRECISE> __device__ __forceinline__ float m_exp(float x) {
  if constexpr (PRECISE) return expf(x); else return __expf(x);
}
template <bool PRECISE> __device__ __forceinline__ float m_log(float x) {
  if constexpr (PRECISE) return logf(x); else return __logf(x);
}
template <bool PRECISE> __device__ __forceinline__ float m_div(float a, float b) {
  if constexpr (PRECISE) return a / b; else return __fdividef(a, b);
}
// logistic function 1 / (1 + e^-x)
template <bool PRECISE> __device__ __forceinline__ float m_sigmoid(float x) {
  return m_div<PRECISE>(1.0f, 1.0f + m_exp<PRECISE>(-x));
}
// x * sigmoid(x)
template <bool PRECISE> __device__ __forceinline__ float m_silu(float x) {
  return m_div<PRECISE>(x, 1.0f + m_exp<PRECISE>(-x));
}
// tanh; the 16-bit path uses tanh(x) = 1 - 2 / (e^{2x} + 1), whose absolute
// error stays near fp32 epsilon over the whole range.
template <bool PRECISE> __device__ __forceinline__ float m_tanh(float x) {
  if constexpr (PRECISE) return tanhf(x);
  else return 1.0f - __fdividef(2.0f, __expf(2.0f * x) + 1.0f);
}
// tanh-form GELU, 0.5 v (1 + tanh(k (v + 0.044715 v^3))) with k = sqrt(2/pi),
// evaluated through the identity 0.5 (1 + tanh(z)) = 1 / (1 + e^{-2z}), which
// has no cancellation for large negative v.
template <bool PRECISE> __device__ __forceinline__ float m_gelu_tanh(float v) {
  if constexpr (PRECISE) {
    const float k2 = 1.5957691216057308f;  // 2 * sqrt(2 / pi)
    const float z2 = k2 * v * fmaf(0.044715f * v, v, 1.0f);
    return v / (1.0f + expf(-z2));
  } else {
    // e^{-2z} = 2^{v (c1 + c2 v^2)}, c1 = -2 sqrt(2/pi) log2(e),
    // c2 = 0.044715 c1: three FP32 ops, EX2, one add, RCP, one multiply
    const float c1 = -2.3022082f, c2 = -0.10294324f;
    const float e = fast_exp2(v * fmaf(c2, v * v, c1));
    return v * fast_rcp(1.0f + e);
  }
}

}  // namespace molten
