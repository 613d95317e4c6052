// Allocation-free attention-score rows: out = softmax(Q @ K) per row.
//
// Who this is for: callers that must not call cudaMalloc at all -- code
// running while a stream is being captured into a CUDA graph (an allocation
// would break the capture), hosts whose device memory is owned by another
// framework's allocator, and real-time loops that forbid allocating after
// start-up.  The regular path for this fusion group (GEMM, then a row
// softmax over an fp32 intermediate) gets its intermediate from the caller's
// allocator; this variant keeps the intermediate in a fixed file-scope device
// array instead, so it allocates nothing.
//
// Limits and sharing:
//   * m * n <= MOLTEN_NOALLOC_SCORES_MAX_ELEMENTS (8 Mi fp32 values, 32 MiB
//     held by every GPU that loads the library, until the process exits);
//     larger calls are rejected with MOLTEN_ERR_INVALID before any launch.
//   * All calls on a device share that array and the wait-status word, and
//     the array keeps the last call's contents.  Calls that overlap on the
//     GPU (different streams, no ordering between them) race on it; order
//     them on one stream or with events.
//   * The first call on a device resolves the arrays' device addresses with
//     cudaGetSymbolAddress and sets the GEMM kernel's shared-memory limit;
//     make that first call before any stream capture begins.
//   * A bounded wait that runs out inside the GEMM sets a bit in this file's
//     status word, which stays set until it is read: molten_read_status
//     reports it together with the runtime's own word (and clears both when
//     asked to), so callers check these calls the same way as any other.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "molten_rt.h"
#include "molten/gemm_sm100.cuh"
#include "molten/row_engine.cuh"

// the calling thread's error text (defined with molten_last_error)
void molten_internal_set_error(const char* msg);

namespace {

constexpr long long kMaxElements = MOLTEN_NOALLOC_SCORES_MAX_ELEMENTS;
constexpr int kBN = 128, kStages = 6;
typedef molten::GemmLayout<128, kBN, 64, kStages, 16> ScoresLayout;

// The scratch: the fp32 score rows between the two kernels, and the GEMM's
// bounded-wait error word (element 0; zero at load, sticky until read).
static __device__ __align__(256) float g_scores_scratch[kMaxElements];
static __device__ __align__(256) int g_scores_status[64];

int fail(int code, const std::string& msg);

// GEMM epilogue: the fp32 accumulators of C[row, col0 .. col0+31] go to the
// scratch unchanged (n is a multiple of 8, so every 4-float chunk that starts
// inside the row ends inside it).
struct ScoresToScratch {
  __device__ __forceinline__ static void apply(const molten::GemmArgs& args, long long row,
                                               long long col0, const float (&acc)[32]) {
    if (row >= args.m) return;
    float* dst = static_cast<float*>(args.out[0]) + row * args.n;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const long long c = col0 + 4 * q;
      if (c >= args.n) break;
      *reinterpret_cast<float4*>(dst + c) =
          make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
    }
  }
};

__global__ void __launch_bounds__(256, 1) scores_gemm_noalloc(const __grid_constant__ molten::GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const molten::GemmShared sh = molten::gemm_carve<ScoresLayout>(smem_raw);
  molten::gemm_init<ScoresLayout>(sh, args);
  __syncthreads();
  molten::gemm_roles<ScoresLayout, false, ScoresToScratch>(sh, args);
  __syncthreads();
  molten::gemm_teardown<ScoresLayout>(sh);
}

// One CTA per row: this thread's max, then its sum of e^(x - max), one
// (max, sum) all-reduce, then out = e^(x - M) / S rounded to bf16.
__global__ void __launch_bounds__(256) scores_softmax_noalloc(const float* __restrict__ s,
                                                              molten::bf16* __restrict__ out,
                                                              long long m, long long n) {
  typedef molten::RowTeam<256, 1, 1> Team;
  __shared__ float red[Team::smem_floats(2, 1)];
  const Team tm(m, 0);
  const long long row = tm.row;
  const float* r = s + (tm.row_ok ? row : 0) * n;
  float lm = -INFINITY;
  for (long long c = 4LL * threadIdx.x; tm.row_ok && c < n; c += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(r + c);
    lm = fmaxf(lm, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
  }
  const float lz = (lm == -INFINITY) ? 0.0f : lm;
  float ls = 0.0f;
  for (long long c = 4LL * threadIdx.x; tm.row_ok && c < n; c += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(r + c);
    ls += expf(v.x - lz) + expf(v.y - lz) + expf(v.z - lz) + expf(v.w - lz);
  }
  float M = lm, S = ls;
  tm.reduce_softmax(M, S, red, 0);
  if (!tm.row_ok) return;
  const float inv = 1.0f / S;
  molten::bf16* o = out + row * n;
  for (long long c = 4LL * threadIdx.x; c < n; c += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(r + c);
    const __nv_bfloat162 a = __floats2bfloat162_rn(expf(v.x - M) * inv, expf(v.y - M) * inv);
    const __nv_bfloat162 b = __floats2bfloat162_rn(expf(v.z - M) * inv, expf(v.w - M) * inv);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&a);
    pk.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(o + c) = pk;
  }
}

struct DeviceSetup {
  bool ready = false;
  float* scratch = nullptr;
  int* status = nullptr;
  int sms = 0;
};

// One slot per device ordinal, in storage that never moves: a pointer
// handed out by setup_device stays valid while other threads set up other
// devices.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceSetup g_setup[kMaxDevices];

int fail(int code, const std::string& msg) {
  molten_internal_set_error(msg.c_str());       // read back with molten_last_error()
  return code;
}

int cuda_err(cudaError_t e, const char* what) {
  return fail(MOLTEN_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Once per device, with that device current: the device addresses of the
// scratch arrays (in host code their names are only host-side stand-ins),
// the SM count and the GEMM kernel's dynamic shared-memory limit.
int setup_device(int dev, DeviceSetup** out) {
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MOLTEN_ERR_INVALID, "device ordinal " + std::to_string(dev) + " beyond " +
                                        std::to_string(kMaxDevices));
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceSetup& d = g_setup[dev];
  if (!d.ready) {
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), g_scores_scratch);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress(scores scratch)");
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_scores_status);
    if (e != cudaSuccess) return cuda_err(e, "cudaGetSymbolAddress(status word)");
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaDeviceGetAttribute(SM count)");
    e = cudaFuncSetAttribute(scores_gemm_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ScoresLayout::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_err(e, "cudaFuncSetAttribute(GEMM shared memory)");
    d.ready = true;
  }
  *out = &d;
  return MOLTEN_OK;
}

}  // namespace

// Read (and when reset != 0 clear) this file's status word on `device`;
// 0 when no allocation-free call ever ran there.  Called by
// molten_read_status, which ORs the value into the runtime's own word.
int molten_internal_noalloc_status(int device, int* value, int reset) {
  *value = 0;
  if (device < 0 || device >= kMaxDevices) return MOLTEN_OK;
  int* word = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_setup[device].ready) return MOLTEN_OK;
    word = g_setup[device].status;
  }
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess)
    return cuda_err(e, "cudaSetDevice");
  e = cudaMemcpy(value, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && reset && *value) e = cudaMemset(word, 0, sizeof(int));
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_err(e, "reading the allocation-free status word");
  return MOLTEN_OK;
}

extern "C" int molten_scores_softmax_bf16_noalloc(const void* q, const void* k, void* out,
                                                  long long m, long long n, long long kdim,
                                                  void* stream) {
  if (!q || !k || !out) return fail(MOLTEN_ERR_INVALID, "null q, k or out");
  if (m < 1 || n < 1 || kdim < 1) return fail(MOLTEN_ERR_INVALID, "m, n and k must be >= 1");
  if (m > kMaxElements || n > kMaxElements || m * n > kMaxElements)
    return fail(MOLTEN_ERR_INVALID,
                "m * n = " + std::to_string(m * n) + " exceeds the allocation-free limit of " +
                    std::to_string(kMaxElements) + " score elements");
  if (n % 8 || kdim % 8) return fail(MOLTEN_ERR_INVALID, "n and k must be multiples of 8");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(out)) % 16)
    return fail(MOLTEN_ERR_INVALID, "q, k and out must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  DeviceSetup* d = nullptr;
  int rc = setup_device(dev, &d);
  if (rc) return rc;

  molten::GemmArgs args;
  memset(&args, 0, sizeof(args));
  rc = molten_encode_tma_2d(&args.tmap_a, MOLTEN_DT_BF16, q, (uint64_t)kdim, (uint64_t)m,
                            (uint64_t)kdim * 2, 64, 128, 1);
  if (rc) return fail(rc, std::string("TMA descriptor of q: ") + molten_last_error());
  rc = molten_encode_tma_2d(&args.tmap_b, MOLTEN_DT_BF16, k, (uint64_t)n, (uint64_t)kdim,
                            (uint64_t)n * 2, 64, 64, 1);
  if (rc) return fail(rc, std::string("TMA descriptor of k: ") + molten_last_error());
  args.out[0] = d->scratch;
  args.m = m;
  args.n = n;
  args.k = kdim;
  args.status = d->status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long tiles = ((m + 127) / 128) * ((n + kBN - 1) / kBN);
  const unsigned grid = (unsigned)(tiles < d->sms ? tiles : d->sms);
  scores_gemm_noalloc<<<grid, dim3(128, 2), ScoresLayout::SMEM_BYTES, st>>>(args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(e, "launching the scores GEMM");
  scores_softmax_noalloc<<<(unsigned)m, 256, 0, st>>>(d->scratch, static_cast<molten::bf16*>(out),
                                                      m, n);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(e, "launching the row softmax");
  return MOLTEN_OK;
}
