/*
 * molten_rt.h -- C ABI of libmolten_rt.so, the runtime that loads the
 * nvcc-built sm_100a cubins emitted by Molten's code generator and launches
 * their kernels.  Plain pointers and sizes only; no torch or C++ types.
 *
 * It replaces, on the reference side (TxsharDev/molten v0.1.0):
 *   - torch.utils.cpp_extension.load() of the generated .cu
 *     (molten/runtime.py:72-79)                      -> molten_module_load*
 *   - the per-kernel pybind launch wrapper "<name>_launch" emitted by
 *     MoltenRuntime._make_extension (molten/runtime.py:96-199) and called by
 *     CompiledKernel.__call__ (molten/runtime.py:31-36) -> molten_launch
 *   - the implicit nvcc error path (molten/runtime.py:90-94)
 *                                                    -> status + molten_last_error
 *
 * Every function returns MOLTEN_OK (0) or a nonzero MOLTEN_ERR_* code; the
 * text of the last error of the calling thread is molten_last_error().
 * Launches are asynchronous on the given stream (NULL = the legacy default
 * stream) and never synchronise the device.
 */
#ifndef MOLTEN_RT_H
#define MOLTEN_RT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOLTEN_OK 0
#define MOLTEN_ERR_INVALID 1     /* bad argument: null pointer, size, alignment */
#define MOLTEN_ERR_CUDA 2        /* a CUDA runtime / driver call failed */
#define MOLTEN_ERR_NOT_FOUND 3   /* no such kernel in the module */
#define MOLTEN_ERR_IO 4          /* cubin file missing or unreadable */

#define MOLTEN_MAX_IO 8

#ifdef __cplusplus
#define MOLTEN_ALIGN64 alignas(64)
#else
#define MOLTEN_ALIGN64 _Alignas(64)
#endif

/* molten_launch_cfg.flags: launch with programmatic stream serialization
 * (programmatic dependent launch).  The kernel may start launching while
 * the previous kernel of the stream is finishing; every generated kernel
 * waits (griddepcontrol.wait) for it before touching global memory. */
#define MOLTEN_LAUNCH_PDL 1u

/* Launch geometry of one kernel.  cluster = {0,0,0} or {1,1,1}: no cluster. */
typedef struct molten_launch_cfg {
  uint32_t grid[3];
  uint32_t block[3];
  uint32_t cluster[3];
  uint32_t smem_bytes;           /* dynamic shared memory per CTA */
  uint32_t flags;                /* MOLTEN_LAUNCH_* bits */
} molten_launch_cfg;

/* Parameter block of every generated row / elementwise kernel
 * (device side: molten::RowArgs in molten/row_engine.cuh). */
typedef struct molten_row_args {
  const void* in[MOLTEN_MAX_IO];
  void* out[MOLTEN_MAX_IO];
  long long rows;                /* rows of this launch (a shard may be fewer) */
  long long row_offset;          /* global index of row 0 (masks, broadcasts) */
  long long cols;
  int* status;
} molten_row_args;

/* Parameter block of the generated tcgen05 GEMM kernels
 * (device side: molten::GemmArgs in molten/gemm_sm100.cuh). */
typedef struct molten_gemm_args {
  MOLTEN_ALIGN64 unsigned char tmap_a[128];  /* from molten_encode_tma_2d */
  MOLTEN_ALIGN64 unsigned char tmap_b[128];
  const void* in[MOLTEN_MAX_IO];
  void* out[MOLTEN_MAX_IO];
  long long m, n, k;             /* one problem: C[m, n] = A[m, k] B[k, n] */
  long long row_offset;
  int* status;
  int batch;                     /* stacked independent problems (0 or 1: one) */
  float* work;                   /* stream-K kernels: partial-tile workspace */
  int* tile_count;               /* stream-K kernels: per-tile counters, zero between calls */
} molten_gemm_args;

/* Parameter block of the generated fused attention-score kernels
 * (device side: molten::AttnArgs in molten/attn_sm100.cuh):
 * P[h] = softmax(Q[h] K[h]^T * scale) for h < batch. */
typedef struct molten_attn_args {
  MOLTEN_ALIGN64 unsigned char tmap_q[128];  /* Q [batch*m, d], box {64, 128}, 128B swizzle */
  MOLTEN_ALIGN64 unsigned char tmap_k[128];  /* K [batch*n, d], box {64, BN}, 128B swizzle */
  MOLTEN_ALIGN64 unsigned char tmap_p[128];  /* P [batch*m, n], box {32, 32}, 64B swizzle */
  void* out;                     /* P */
  long long m, n, d;
  long long row_offset;
  int* status;
  int batch;                     /* stacked independent problems (0 or 1: one) */
} molten_attn_args;

/* Version of this ABI (major * 100 + minor). */
int molten_version(void);

/* Text of the last error on the calling thread ("" when none). */
const char* molten_last_error(void);

/* Number of CUDA devices visible to the process. */
int molten_device_count(int* count);

/* Wait for all work on `device`. */
int molten_sync(int device);

/* Load an sm_100a cubin into `device`'s primary context.
 * Replaces torch.utils.cpp_extension.load (molten/runtime.py:72-79). */
int molten_module_load(const char* cubin_path, int device, void** mod);

/* Same from an in-memory cubin image. */
int molten_module_load_data(const void* image, size_t nbytes, int device, void** mod);

/* Unload a module; its kernels must no longer be running. */
int molten_module_unload(void* mod);

/* Registers per thread, max threads per block and static shared memory of
 * a kernel (any output pointer may be NULL). */
int molten_kernel_info(void* mod, const char* kernel, int* num_regs,
                       int* max_threads, int* static_smem);

/* How many CTAs of `kernel` fit on one SM with `cfg`'s block size and
 * dynamic shared memory (*ctas_per_sm), and how many clusters of
 * `cfg->cluster` fit on the whole device at once (*clusters; equals
 * ctas_per_sm x SMs without clusters).  Persistent kernels size their
 * grid with it.  No counterpart in the reference (its launches are one CTA
 * per row or tile). */
int molten_max_resident(void* mod, const char* kernel, const molten_launch_cfg* cfg,
                        int* ctas_per_sm, int* clusters);

/* Launch `kernel` of `mod` with one by-value parameter block of
 * `params_bytes` bytes (molten_row_args or molten_gemm_args).
 * Replaces the generated "<name>_launch" wrapper (molten/runtime.py:111-189)
 * called from CompiledKernel.__call__ (molten/runtime.py:31-36). */
int molten_launch(void* mod, const char* kernel, const molten_launch_cfg* cfg,
                  const void* params, size_t params_bytes, void* stream);

/* Element types for molten_encode_tma_2d. */
#define MOLTEN_DT_BF16 0
#define MOLTEN_DT_F16 1
#define MOLTEN_DT_F32 2

/* Encode a 2-D TMA descriptor (128 bytes, 64-byte aligned `tmap`) for a
 * row-major matrix of `outer` rows of `inner` elements, rows
 * `row_stride_bytes` apart, copied in boxes of box_inner x box_outer,
 * swizzled in spans of `swizzle` bytes: 0 none, 32, 64, or 128 (1 also
 * means 128); a swizzled box row must not exceed the span.  Out-of-range box
 * elements read as zero and are not written by stores.  base must be
 * 16-byte aligned and row_stride a multiple of 16 bytes. */
int molten_encode_tma_2d(void* tmap, int dtype, const void* base,
                         uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                         uint32_t box_inner, uint32_t box_outer, int swizzle);

/* Per-device error word that kernels with bounded waits set bits in
 * (allocated on first use, then reused). */
int molten_status_word(int device, int** dev_ptr);

/* Read (and when reset != 0 clear) the device error word; synchronises.
 * The value also carries the bits of molten_scores_softmax_bf16_noalloc's own
 * word on that device (that entry point may not allocate this one). */
int molten_read_status(int device, int* value, int reset);

/* Allocation-free attention-score rows (no counterpart in the reference):
 * out[m, n] = softmax over each row of (q[m, kdim] @ k[kdim, n]), bf16 in and
 * out, fp32 accumulation.  For callers that cannot call cudaMalloc (a stream
 * being captured into a CUDA graph, a device heap owned by another
 * allocator, loops that must not allocate after start-up): the fp32
 * intermediate lives in a fixed device array of
 * MOLTEN_NOALLOC_SCORES_MAX_ELEMENTS floats (32 MiB per GPU that loads the
 * library, held until exit), so m * n must not exceed that limit
 * (MOLTEN_ERR_INVALID otherwise).  Calls share that array: calls that overlap
 * on the GPU race.  n and kdim must be multiples of 8, pointers 16-byte
 * aligned.  The first call on a device resolves the array's address, so make
 * it before any stream capture.  Runs on the current device and `stream`.
 * A bounded wait that runs out inside it is reported by molten_read_status,
 * as for every other kernel; its status bits stay set until read with reset. */
#define MOLTEN_NOALLOC_SCORES_MAX_ELEMENTS (8LL * 1024 * 1024)
int molten_scores_softmax_bf16_noalloc(const void* q, const void* k, void* out,
                                       long long m, long long n, long long kdim,
                                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOLTEN_RT_H */
