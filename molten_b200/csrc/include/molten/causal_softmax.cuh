// Causal row softmax for long rows, split into row CTAs and zero-fill CTAs.
//
//   out[r, c] = softmax over c of (x[r, c] + mask[r, c]),
//   mask[r, c] = -inf  for  c > (grow mod P) + OFF,  0 elsewhere,
//
// (grow = the row's global index).  Row r has v = min((grow mod P) + OFF + 1,
// COLS) >= 1 visible logits; everything after them is exactly 0.  On long
// rows most of the output is those zeros (4096 x 32768: 94%), so the kernel
// is mostly a write stream, and it is laid out as one:
//
//   one CTA per row:        the visible part only -- a pass
//                           reading the row's first vs = ceil(v / VEC) 16-byte
//                           slots (online max / sum per thread, one (max, sum)
//                           reduction per CTA), a second pass re-reading them
//                           (from L2) and storing exp(x - M) / S, with the
//                           masked elements of the last visible slot as 0;
//   ZT zero tiles per row:  (ZCOLS columns each)
//                           16-byte zero stores of the tile's columns from
//                           slot vs on, which depend on no data at all.
//
// With ZT == 0 each row CTA also stores its own row's zeros.  INTERLEAVE
// (the default) launches each row CTA next to its row's zero tiles, so the
// zero stream keeps HBM busy while the row CTAs wait on their loads and
// reductions (bf16 4096 x 32768: 49.2 us interleaved, 55.6 us row CTAs
// first; zero tiles of 1 / 4 / 16 slots per thread 77.5 / 49.2 / 51.4 us).
#pragma once

#include "molten/common.cuh"
#include "molten/row_engine.cuh"

namespace molten {

template <bool PRECISE>
__device__ __forceinline__ float cs_exp(float x) {
  if constexpr (PRECISE) return expf(x);
  else return __expf(x);
}

// (m, s) <- the pair of the union: s = s1 e^(m1 - M) + s2 e^(m2 - M), M = max
template <bool PRECISE>
__device__ __forceinline__ void cs_merge(float& m, float& s, float m2, float s2) {
  const float M = fmaxf(m, m2);
  if (M == -INFINITY) return;                       // both empty
  const float a = (m == -INFINITY) ? 0.0f : s * cs_exp<PRECISE>(m - M);
  const float b = (m2 == -INFINITY) ? 0.0f : s2 * cs_exp<PRECISE>(m2 - M);
  m = M;
  s = a + b;
}

// 32 zero bytes with one 256-bit store (sm_100); p 32-byte aligned.
__device__ __forceinline__ void store_zero32(void* p) {
  asm volatile("st.global.v8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" :: "l"(p), "r"(0) : "memory");
}

// Online (max, sum-of-exponentials) update with the VEC values of one slot.
template <bool PRECISE, int VEC>
__device__ __forceinline__ void cs_update(float& m, float& s, const float (&f)[VEC]) {
  float sm = f[0];
#pragma unroll
  for (int e = 1; e < VEC; ++e) sm = fmaxf(sm, f[e]);
  const float M = fmaxf(m, sm);
  if (M == -INFINITY) return;                        // nothing visible yet
  float acc = (m == -INFINITY) ? 0.0f : s * cs_exp<PRECISE>(m - M);
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc += cs_exp<PRECISE>(f[e] - M);   // e^-inf = 0
  m = M;
  s = acc;
}

// Zero tile zt of `row`: its columns from the first fully masked slot on.
template <typename T, int THREADS, long long COLS, long long P, long long OFF,
          long long ZCOLS, bool W32>
__device__ __forceinline__ void causal_zero_tile(T* __restrict__ out, long long row_offset,
                                                 unsigned row, int zt) {
  constexpr int VEC = 16 / (int)sizeof(T);
  const long long vl = (row_offset + (long long)row) % P + OFF + 1;
  const int v = (int)(vl < COLS ? vl : COLS);
  const int vs = (v + VEC - 1) / VEC;
  T* o = out + (long long)row * COLS;
  const int c0 = zt * (int)ZCOLS;
  const int c1 = (c0 + (int)ZCOLS < (int)COLS) ? c0 + (int)ZCOLS : (int)COLS;
  int c = (vs * VEC > c0) ? vs * VEC : c0;           // first fully masked column here
  if constexpr (W32) {
    constexpr int V2 = 2 * VEC;                       // elements per 32-byte store
    if (c < c1 && (c % V2) != 0) {                   // a leading 16-byte slot
      if (threadIdx.x == 0) store_zero_slot<kStoreDefault, T, VEC>(o + c);
      c += VEC;
    }
    int j = c + (int)threadIdx.x * V2;
    for (; j + V2 <= c1; j += THREADS * V2) store_zero32(o + j);
    if (j < c1) store_zero_slot<kStoreDefault, T, VEC>(o + j);   // a trailing slot
  } else {
    for (int j = c + (int)threadIdx.x * VEC; j < c1; j += THREADS * VEC)
      store_zero_slot<kStoreDefault, T, VEC>(o + j);
  }
}

// Launch orders of the two kinds of CTA:
//   ZPERSIST > 0: CTAs [0, ZPERSIST) are persistent zero CTAs, each storing
//                 zero tiles t = b, b + ZPERSIST, ... of all rows' tiles (so
//                 their stores stream without a CTA launch and a store
//                 drain per 16 KB), then one CTA per row;
//   INTERLEAVE:   CTA b is part b % (1 + ZT) of row b / (1 + ZT) (part 0 the
//                 visible logits, part z > 0 zero tile z - 1);
//   otherwise:    the row CTAs, then the zero tiles.
// W32: rows start on 32-byte boundaries (the output pointer is 32-byte
// aligned and a row is a multiple of 32 bytes), so zero tiles store 32
// bytes at a time.
template <typename T, int THREADS, long long COLS, long long P, long long OFF, int ZT,
          long long ZCOLS, bool PRECISE, bool INTERLEAVE = false, bool W32 = false,
          int ZPERSIST = 0>
__device__ __forceinline__ void causal_softmax_cta(const RowArgs& args) {
  constexpr int VEC = 16 / (int)sizeof(T);
  static_assert(COLS % VEC == 0, "rows are whole 16-byte slots");
  static_assert(COLS < (1LL << 31) && ZCOLS % VEC == 0, "32-bit column indices");
  static_assert(OFF >= 0 && P >= 1, "every row keeps at least one logit");
  static_assert(!W32 || (COLS * (long long)sizeof(T)) % 32 == 0, "32-byte rows");
  static_assert(ZPERSIST == 0 || ZT > 0, "persistent zero CTAs store zero tiles");
  const T* __restrict__ x = static_cast<const T*>(args.in[0]);
  T* __restrict__ out = static_cast<T*>(args.out[0]);
  const unsigned b = blockIdx.x;
  unsigned row;
  int zt = -1;                              // >= 0: this CTA is zero tile zt of `row`
  if constexpr (ZPERSIST > 0) {
    if (b < (unsigned)ZPERSIST) {
      const long long tiles = args.rows * ZT;
      for (long long t = b; t < tiles; t += ZPERSIST) {
        const unsigned r = (unsigned)(t / ZT);
        causal_zero_tile<T, THREADS, COLS, P, OFF, ZCOLS, W32>(out, args.row_offset, r,
                                                               (int)(t - (long long)r * ZT));
      }
      return;
    }
    row = b - (unsigned)ZPERSIST;
  } else if constexpr (INTERLEAVE) {
    row = b / (1u + ZT);
    zt = (int)(b - row * (1u + ZT)) - 1;
  } else if ((long long)b >= args.rows) {
    const unsigned t = b - (unsigned)args.rows;
    row = t / (unsigned)(ZT > 0 ? ZT : 1);
    zt = (int)(t - row * (unsigned)ZT);
  } else {
    row = b;
  }
  if (zt >= 0) {
    causal_zero_tile<T, THREADS, COLS, P, OFF, ZCOLS, W32>(out, args.row_offset, row, zt);
    return;
  }
  // visible logits of the row: v in [1, COLS]
  const long long vl = (args.row_offset + (long long)row) % P + OFF + 1;
  const int v = (int)(vl < COLS ? vl : COLS);
  const int vs = (v + VEC - 1) / VEC;                // slots holding visible logits
  T* o = out + (long long)row * COLS;

  // --------------------------------------------------------- visible part
  const T* xr = x + (long long)row * COLS;
  const int vfull = v / VEC;                          // slots with no masked element
  float m = -INFINITY, s = 0.0f;
  for (int j = threadIdx.x; j < vfull; j += THREADS) {
    const Slot<T, VEC> sl = load_slot<kLoadDefault, T, VEC>(xr + j * VEC);
    float f[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) f[e] = to_f32(sl.v[e]);
    cs_update<PRECISE, VEC>(m, s, f);
  }
  const int jp = vfull;                               // the partial slot, if any
  const bool partial = vs > vfull && (int)threadIdx.x == jp % THREADS;
  if (partial) {
    const Slot<T, VEC> sl = load_slot<kLoadDefault, T, VEC>(xr + jp * VEC);
    float f[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) f[e] = (jp * VEC + e < v) ? to_f32(sl.v[e]) : -INFINITY;
    cs_update<PRECISE, VEC>(m, s, f);
  }
  // (max, sum) over the CTA: warp butterfly, then the warps' pairs
  constexpr int WARPS = THREADS / 32;
  __shared__ float red_m[WARPS], red_s[WARPS];
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, d);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, d);
    cs_merge<PRECISE>(m, s, m2, s2);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) { red_m[warp] = m; red_s[warp] = s; }
  __syncthreads();
  // every thread combines the warps' pairs in the same order: same (M, S)
  float M = red_m[0], S = red_s[0];
#pragma unroll
  for (int w = 1; w < WARPS; ++w) cs_merge<PRECISE>(M, S, red_m[w], red_s[w]);
  const float inv = 1.0f / S;
  for (int j = threadIdx.x; j < vs; j += THREADS) {
    const Slot<T, VEC> sl = load_slot<kLoadDefault, T, VEC>(xr + j * VEC);
    float f[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float p = cs_exp<PRECISE>(to_f32(sl.v[e]) - M);
      f[e] = PRECISE ? p / S : p * inv;
    }
    if (j == jp) {                                    // masked elements of the partial slot
#pragma unroll
      for (int e = 0; e < VEC; ++e) if (jp * VEC + e >= v) f[e] = 0.0f;
    }
    Slot<T, VEC> ov;
#pragma unroll
    for (int e = 0; e < VEC; ++e) ov.v[e] = from_f32<T>(f[e]);
    store_slot<kStoreDefault, T, VEC>(o + j * VEC, ov);
  }
  if constexpr (ZT == 0) {
    for (int c = (vs + (int)threadIdx.x) * VEC; c < (int)COLS; c += THREADS * VEC)
      store_zero_slot<kStoreDefault, T, VEC>(o + c);
  }
}

}  // namespace molten
