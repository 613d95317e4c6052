// libmolten_rt.so: loads Molten's nvcc-built sm_100a cubins and launches
// their kernels behind the C ABI of include/molten_rt.h.
//
// The CUDA runtime (linked statically) owns device selection, primary
// contexts and the status words; module loading, launches with cluster
// dimensions and TMA descriptors go through driver entry points resolved at
// run time with cudaGetDriverEntryPoint, so the library loads on machines
// without a GPU driver (symbols resolve; calls then fail with an error).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "molten_rt.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MOLTEN_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                   cudaGetErrorString(e) + ")");
}

// ------------------------------------------------------ driver entry points
typedef CUresult (*PFN_GetErrorString)(CUresult, const char**);
typedef CUresult (*PFN_ModuleLoadData)(CUmodule*, const void*);
typedef CUresult (*PFN_ModuleUnload)(CUmodule);
typedef CUresult (*PFN_ModuleGetFunction)(CUfunction*, CUmodule, const char*);
typedef CUresult (*PFN_FuncSetAttribute)(CUfunction, CUfunction_attribute, int);
typedef CUresult (*PFN_FuncGetAttribute)(int*, CUfunction_attribute, CUfunction);
typedef CUresult (*PFN_LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**);
typedef CUresult (*PFN_FuncGetParamInfo)(CUfunction, size_t, size_t*, size_t*);
typedef CUresult (*PFN_OccupancyBlocks)(int*, CUfunction, int, size_t);
typedef CUresult (*PFN_OccupancyClusters)(int*, CUfunction, const CUlaunchConfig*);
typedef CUresult (*PFN_TensorMapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                             const cuuint64_t*, const cuuint64_t*,
                                             const cuuint32_t*, const cuuint32_t*,
                                             CUtensorMapInterleave, CUtensorMapSwizzle,
                                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Driver {
  PFN_GetErrorString get_error_string = nullptr;
  PFN_ModuleLoadData module_load_data = nullptr;
  PFN_ModuleUnload module_unload = nullptr;
  PFN_ModuleGetFunction module_get_function = nullptr;
  PFN_FuncSetAttribute func_set_attribute = nullptr;
  PFN_FuncGetAttribute func_get_attribute = nullptr;
  PFN_LaunchKernelEx launch_kernel_ex = nullptr;
  PFN_FuncGetParamInfo func_get_param_info = nullptr;   // optional (12.4+)
  PFN_OccupancyBlocks occupancy_blocks = nullptr;
  PFN_OccupancyClusters occupancy_clusters = nullptr;
  PFN_TensorMapEncodeTiled tensor_map_encode_tiled = nullptr;
  bool ok = false;
  std::string error;
};

template <class T>
bool resolve(const char* name, T* fn, bool required, std::string* err) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
    if (required) *err = std::string("driver entry point ") + name + " unavailable";
    return !required;
  }
  *fn = reinterpret_cast<T>(p);
  return true;
}

Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    std::string err;
    bool ok = resolve("cuGetErrorString", &d.get_error_string, true, &err) &&
              resolve("cuModuleLoadData", &d.module_load_data, true, &err) &&
              resolve("cuModuleUnload", &d.module_unload, true, &err) &&
              resolve("cuModuleGetFunction", &d.module_get_function, true, &err) &&
              resolve("cuFuncSetAttribute", &d.func_set_attribute, true, &err) &&
              resolve("cuFuncGetAttribute", &d.func_get_attribute, true, &err) &&
              resolve("cuLaunchKernelEx", &d.launch_kernel_ex, true, &err) &&
              resolve("cuTensorMapEncodeTiled", &d.tensor_map_encode_tiled, true, &err) &&
              resolve("cuOccupancyMaxActiveBlocksPerMultiprocessor", &d.occupancy_blocks, true,
                      &err) &&
              resolve("cuOccupancyMaxActiveClusters", &d.occupancy_clusters, true, &err);
    resolve("cuFuncGetParamInfo", &d.func_get_param_info, false, &err);
    d.ok = ok;
    d.error = err;
  });
  return d;
}

int drv_fail(CUresult r, const char* what) {
  const char* s = "unknown";
  if (driver().get_error_string) driver().get_error_string(r, &s);
  return fail(MOLTEN_ERR_CUDA, std::string(what) + ": CUresult " + std::to_string((int)r) + " (" + s + ")");
}

int need_driver() {
  Driver& d = driver();
  if (!d.ok) return fail(MOLTEN_ERR_CUDA, "CUDA driver unavailable: " + d.error);
  return MOLTEN_OK;
}

// Make `device` current on this thread.  With init != 0 also make sure its
// primary context exists (the runtime creates it lazily); launches pass 0 so
// that nothing but the launch itself happens while a stream is captured.
int use_device(int device, int init = 1) {
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (cur != device) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  }
  if (init) {
    e = cudaFree(nullptr);
    if (e != cudaSuccess) return cuda_fail(e, "initialising the device context");
  }
  return MOLTEN_OK;
}

struct Kernel {
  CUfunction fn = nullptr;
  int smem_set = 0;       // max dynamic smem configured so far
  size_t param_bytes = 0; // 0 = unknown
};

struct Module {
  CUmodule mod = nullptr;
  int device = 0;
  std::mutex mu;
  std::unordered_map<std::string, Kernel> kernels;
};

int lookup(Module* m, const char* name, Kernel** out) {
  std::lock_guard<std::mutex> lock(m->mu);
  auto it = m->kernels.find(name);
  if (it == m->kernels.end()) {
    Kernel k;
    CUresult r = driver().module_get_function(&k.fn, m->mod, name);
    if (r != CUDA_SUCCESS)
      return fail(MOLTEN_ERR_NOT_FOUND, std::string("kernel '") + name + "' not in module");
    if (driver().func_get_param_info) {
      size_t off = 0, sz = 0;
      if (driver().func_get_param_info(k.fn, 0, &off, &sz) == CUDA_SUCCESS) k.param_bytes = sz;
    }
    it = m->kernels.emplace(name, k).first;
  }
  *out = &it->second;
  return MOLTEN_OK;
}

std::mutex g_status_mu;
std::vector<int*> g_status;

}  // namespace

// Lets the library's other translation units report errors through
// molten_last_error() (C++ linkage: not part of the C ABI).
void molten_internal_set_error(const char* msg) { g_last_error = msg ? msg : ""; }

// The allocation-free entry point's own wait-status word (noalloc_scores.cu).
int molten_internal_noalloc_status(int device, int* value, int reset);

extern "C" {

int molten_version(void) { return 101; }

const char* molten_last_error(void) { return g_last_error.c_str(); }

int molten_device_count(int* count) {
  if (!count) return fail(MOLTEN_ERR_INVALID, "count is null");
  *count = 0;
  cudaError_t e = cudaGetDeviceCount(count);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    *count = 0;
    cudaGetLastError();
    return MOLTEN_OK;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  return MOLTEN_OK;
}

int molten_sync(int device) {
  int rc = use_device(device);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  return MOLTEN_OK;
}

int molten_module_load_data(const void* image, size_t nbytes, int device, void** mod) {
  if (!image || !nbytes || !mod) return fail(MOLTEN_ERR_INVALID, "null image or output handle");
  *mod = nullptr;
  int rc = need_driver();
  if (rc) return rc;
  rc = use_device(device);
  if (rc) return rc;
  Module* m = new Module();
  m->device = device;
  CUresult r = driver().module_load_data(&m->mod, image);
  if (r != CUDA_SUCCESS) {
    delete m;
    return drv_fail(r, "cuModuleLoadData");
  }
  *mod = m;
  return MOLTEN_OK;
}

int molten_module_load(const char* cubin_path, int device, void** mod) {
  if (!cubin_path || !mod) return fail(MOLTEN_ERR_INVALID, "null path or output handle");
  std::ifstream f(cubin_path, std::ios::binary);
  if (!f) return fail(MOLTEN_ERR_IO, std::string("cannot open ") + cubin_path);
  std::vector<char> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (buf.empty()) return fail(MOLTEN_ERR_IO, std::string("empty cubin ") + cubin_path);
  return molten_module_load_data(buf.data(), buf.size(), device, mod);
}

int molten_module_unload(void* mod) {
  if (!mod) return fail(MOLTEN_ERR_INVALID, "null module");
  Module* m = static_cast<Module*>(mod);
  int rc = use_device(m->device);
  if (rc) return rc;
  CUresult r = driver().module_unload(m->mod);
  delete m;
  if (r != CUDA_SUCCESS) return drv_fail(r, "cuModuleUnload");
  return MOLTEN_OK;
}

int molten_kernel_info(void* mod, const char* kernel, int* num_regs, int* max_threads,
                       int* static_smem) {
  if (!mod || !kernel) return fail(MOLTEN_ERR_INVALID, "null module or kernel name");
  Module* m = static_cast<Module*>(mod);
  Kernel* k = nullptr;
  int rc = lookup(m, kernel, &k);
  if (rc) return rc;
  int v = 0;
  if (num_regs) {
    driver().func_get_attribute(&v, CU_FUNC_ATTRIBUTE_NUM_REGS, k->fn);
    *num_regs = v;
  }
  if (max_threads) {
    driver().func_get_attribute(&v, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, k->fn);
    *max_threads = v;
  }
  if (static_smem) {
    driver().func_get_attribute(&v, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, k->fn);
    *static_smem = v;
  }
  return MOLTEN_OK;
}

// Allow `smem` bytes of dynamic shared memory for kernel `k`, once per size
// increase.  Any nonzero request is set explicitly: the 48 KB default
// counts static plus dynamic shared memory, so 48 KB of dynamic memory next
// to a few static bytes already needs the opt-in.
static int ensure_dynamic_smem(Module* m, Kernel* k, uint32_t smem) {
  if (smem > 0 && (int)smem > k->smem_set) {
    std::lock_guard<std::mutex> lock(m->mu);
    CUresult r = driver().func_set_attribute(k->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                             (int)smem);
    if (r != CUDA_SUCCESS) return drv_fail(r, "cuFuncSetAttribute(max dynamic smem)");
    k->smem_set = (int)smem;
  }
  return MOLTEN_OK;
}

int molten_max_resident(void* mod, const char* kernel, const molten_launch_cfg* cfg,
                        int* ctas_per_sm, int* clusters) {
  if (!mod || !kernel || !cfg) return fail(MOLTEN_ERR_INVALID, "null module, kernel or config");
  Module* m = static_cast<Module*>(mod);
  const uint32_t block = cfg->block[0] * cfg->block[1] * cfg->block[2];
  const uint32_t cl = cfg->cluster[0] * cfg->cluster[1] * cfg->cluster[2];
  if (block == 0 || block > 1024) return fail(MOLTEN_ERR_INVALID, "bad block size");
  Kernel* k = nullptr;
  int rc = lookup(m, kernel, &k);
  if (rc) return rc;
  rc = use_device(m->device);
  if (rc) return rc;
  rc = ensure_dynamic_smem(m, k, cfg->smem_bytes);
  if (rc) return rc;
  int per_sm = 0;
  CUresult r = driver().occupancy_blocks(&per_sm, k->fn, (int)block, cfg->smem_bytes);
  if (r != CUDA_SUCCESS) return drv_fail(r, "cuOccupancyMaxActiveBlocksPerMultiprocessor");
  if (ctas_per_sm) *ctas_per_sm = per_sm;
  if (clusters) {
    int n = 0;
    if (cl > 1) {
      CUlaunchConfig lc;
      std::memset(&lc, 0, sizeof(lc));
      lc.gridDimX = cfg->cluster[0];
      lc.gridDimY = cfg->cluster[1];
      lc.gridDimZ = cfg->cluster[2];
      lc.blockDimX = cfg->block[0];
      lc.blockDimY = cfg->block[1];
      lc.blockDimZ = cfg->block[2];
      lc.sharedMemBytes = cfg->smem_bytes;
      CUlaunchAttribute attr[1];
      attr[0].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
      attr[0].value.clusterDim.x = cfg->cluster[0];
      attr[0].value.clusterDim.y = cfg->cluster[1];
      attr[0].value.clusterDim.z = cfg->cluster[2];
      lc.attrs = attr;
      lc.numAttrs = 1;
      r = driver().occupancy_clusters(&n, k->fn, &lc);
      if (r != CUDA_SUCCESS) return drv_fail(r, "cuOccupancyMaxActiveClusters");
    } else {
      int sms = 0;
      cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
      n = per_sm * sms;
    }
    *clusters = n;
  }
  return MOLTEN_OK;
}

int molten_launch(void* mod, const char* kernel, const molten_launch_cfg* cfg,
                  const void* params, size_t params_bytes, void* stream) {
  if (!mod || !kernel || !cfg || !params)
    return fail(MOLTEN_ERR_INVALID, "null module, kernel, config or params");
  Module* m = static_cast<Module*>(mod);
  for (int i = 0; i < 3; ++i)
    if (cfg->grid[i] == 0 || cfg->block[i] == 0)
      return fail(MOLTEN_ERR_INVALID, "grid and block dims must be >= 1");
  if ((uint64_t)cfg->block[0] * cfg->block[1] * cfg->block[2] > 1024)
    return fail(MOLTEN_ERR_INVALID, "more than 1024 threads per block");
  const uint32_t cl = cfg->cluster[0] * cfg->cluster[1] * cfg->cluster[2];
  if (cl > 1) {
    for (int i = 0; i < 3; ++i)
      if (cfg->cluster[i] == 0 || cfg->grid[i] % cfg->cluster[i])
        return fail(MOLTEN_ERR_INVALID, "grid must be a multiple of the cluster dims");
    if (cl > 8) return fail(MOLTEN_ERR_INVALID, "clusters larger than 8 CTAs are not used");
  }
  Kernel* k = nullptr;
  int rc = lookup(m, kernel, &k);
  if (rc) return rc;
  if (k->param_bytes && k->param_bytes != params_bytes)
    return fail(MOLTEN_ERR_INVALID, std::string("kernel '") + kernel + "' takes a " +
                                        std::to_string(k->param_bytes) + "-byte parameter block, got " +
                                        std::to_string(params_bytes));
  rc = use_device(m->device, 0);
  if (rc) return rc;
  rc = ensure_dynamic_smem(m, k, cfg->smem_bytes);
  if (rc) return rc;
  CUlaunchConfig lc;
  std::memset(&lc, 0, sizeof(lc));
  lc.gridDimX = cfg->grid[0];
  lc.gridDimY = cfg->grid[1];
  lc.gridDimZ = cfg->grid[2];
  lc.blockDimX = cfg->block[0];
  lc.blockDimY = cfg->block[1];
  lc.blockDimZ = cfg->block[2];
  lc.sharedMemBytes = cfg->smem_bytes;
  lc.hStream = static_cast<CUstream>(stream);
  CUlaunchAttribute attr[2];
  unsigned n_attr = 0;
  if (cl > 1) {
    attr[n_attr].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr[n_attr].value.clusterDim.x = cfg->cluster[0];
    attr[n_attr].value.clusterDim.y = cfg->cluster[1];
    attr[n_attr].value.clusterDim.z = cfg->cluster[2];
    ++n_attr;
  }
  if (cfg->flags & MOLTEN_LAUNCH_PDL) {
    attr[n_attr].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr[n_attr].value.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
  }
  if (n_attr) {
    lc.attrs = attr;
    lc.numAttrs = n_attr;
  }
  void* args[1] = {const_cast<void*>(params)};
  CUresult r = driver().launch_kernel_ex(&lc, k->fn, args, nullptr);
  if (r != CUDA_SUCCESS) return drv_fail(r, "cuLaunchKernelEx");
  return MOLTEN_OK;
}

int molten_encode_tma_2d(void* tmap, int dtype, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         int swizzle) {
  if (!tmap || !base) return fail(MOLTEN_ERR_INVALID, "null tensor map or base pointer");
  if (reinterpret_cast<uintptr_t>(tmap) % 64)
    return fail(MOLTEN_ERR_INVALID, "tensor map storage must be 64-byte aligned");
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return fail(MOLTEN_ERR_INVALID, "TMA base address must be 16-byte aligned");
  if (row_stride_bytes % 16)
    return fail(MOLTEN_ERR_INVALID, "TMA row stride must be a multiple of 16 bytes");
  if (!inner || !outer || !box_inner || !box_outer || box_inner > 256 || box_outer > 256)
    return fail(MOLTEN_ERR_INVALID, "bad TMA extents or box");
  CUtensorMapDataType t;
  uint32_t esize;
  switch (dtype) {
    case MOLTEN_DT_BF16: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; esize = 2; break;
    case MOLTEN_DT_F16: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; esize = 2; break;
    case MOLTEN_DT_F32: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; esize = 4; break;
    default: return fail(MOLTEN_ERR_INVALID, "unknown TMA element type");
  }
  if ((box_inner * esize) % 16)
    return fail(MOLTEN_ERR_INVALID, "TMA box inner extent must be a multiple of 16 bytes");
  // swizzle: 0 none; 1 or 128: 128-byte; 64: 64-byte; 32: 32-byte
  const uint32_t span = swizzle == 1 ? 128u : (uint32_t)swizzle;
  CUtensorMapSwizzle sw;
  switch (span) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail(MOLTEN_ERR_INVALID, "swizzle must be 0, 32, 64 or 128 bytes");
  }
  if (span && box_inner * esize > span)
    return fail(MOLTEN_ERR_INVALID, "a swizzled box row must not exceed the swizzle span");
  int rc = need_driver();
  if (rc) return rc;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = driver().tensor_map_encode_tiled(
      static_cast<CUtensorMap*>(tmap), t, 2, const_cast<void*>(base), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE,
      sw,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return drv_fail(r, "cuTensorMapEncodeTiled");
  return MOLTEN_OK;
}

int molten_status_word(int device, int** dev_ptr) {
  if (!dev_ptr || device < 0) return fail(MOLTEN_ERR_INVALID, "bad device or null output");
  std::lock_guard<std::mutex> lock(g_status_mu);
  if ((int)g_status.size() <= device) g_status.resize(device + 1, nullptr);
  if (!g_status[device]) {
    int rc = use_device(device);
    if (rc) return rc;
    int* p = nullptr;
    cudaError_t e = cudaMalloc(&p, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(status word)");
    e = cudaMemset(p, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status word)");
    g_status[device] = p;
  }
  *dev_ptr = g_status[device];
  return MOLTEN_OK;
}

int molten_read_status(int device, int* value, int reset) {
  if (!value) return fail(MOLTEN_ERR_INVALID, "null output");
  int* p = nullptr;
  int rc = molten_status_word(device, &p);
  if (rc) return rc;
  cudaError_t e = cudaMemcpy(value, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading the status word");
  if (reset && *value) {
    e = cudaMemset(p, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the status word");
  }
  // the allocation-free entry point keeps its own word (it may not allocate
  // this one); its bits are reported here too
  int extra = 0;
  rc = molten_internal_noalloc_status(device, &extra, reset);
  if (rc) return rc;
  *value |= extra;
  return MOLTEN_OK;
}

}  // extern "C"
