// thork_rt.cu — host side of libthork_rt.so: the C-ABI declared in
// include/thork_rt.h over the CUDA runtime/driver, NVRTC and NCCL.
//
// Design notes
// * The CUDA runtime is linked statically, so the library loads on a machine
//   without a driver (the CPU test suite checks its exports there); every
//   call then fails with THORK_ERR_CUDA / THORK_ERR_UNAVAILABLE.
// * Driver-only entry points (module loading, cuLaunchKernelEx,
//   cuTensorMapEncodeTiled) are fetched with cudaGetDriverEntryPointByVersion,
//   so they run in the runtime's primary context of the current device.
// * NVRTC and NCCL are opened with dlopen on first use.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "thork_rt.h"
#include "thork_internal.h"

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local std::string g_last_error;

int thork_set_error(int code, const char *fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int thork_cuda_error(cudaError_t e, const char *what) {
  return thork_set_error(THORK_ERR_CUDA, "CUDA error (%s): %s: %s", what,
                         cudaGetErrorName(e), cudaGetErrorString(e));
}

#define CUDA_TRY(call, what)                                 \
  do {                                                       \
    cudaError_t _e = (call);                                 \
    if (_e != cudaSuccess) return thork_cuda_error(_e, what); \
  } while (0)

extern "C" int thork_version(void) { return 100; }

extern "C" int thork_last_error(char *buf, size_t n) {
  if (!buf || n == 0) return THORK_ERR_INVALID;
  size_t len = g_last_error.size() < n - 1 ? g_last_error.size() : n - 1;
  memcpy(buf, g_last_error.data(), len);
  buf[len] = 0;
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// driver entry points
// ---------------------------------------------------------------------------
struct DriverApi {
  bool loaded = false;
  bool ok = false;
  CUresult (*cuGetErrorName)(CUresult, const char **) = nullptr;
  CUresult (*cuGetErrorString)(CUresult, const char **) = nullptr;
  CUresult (*cuModuleLoadData)(CUmodule *, const void *) = nullptr;
  CUresult (*cuModuleUnload)(CUmodule) = nullptr;
  CUresult (*cuModuleGetFunction)(CUfunction *, CUmodule, const char *) = nullptr;
  CUresult (*cuFuncSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*cuLaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **, void **) = nullptr;
  CUresult (*cuTensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                     const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                     const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill) = nullptr;
};

static DriverApi g_drv;
static std::mutex g_drv_mu;

template <class F>
static bool get_entry(const char *name, F *out) {
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) return false;
  *out = reinterpret_cast<F>(p);
  return true;
}

static int driver_api(DriverApi **api) {
  std::lock_guard<std::mutex> lk(g_drv_mu);
  if (!g_drv.loaded) {
    g_drv.loaded = true;
    bool ok = true;
    ok &= get_entry("cuGetErrorName", &g_drv.cuGetErrorName);
    ok &= get_entry("cuGetErrorString", &g_drv.cuGetErrorString);
    ok &= get_entry("cuModuleLoadData", &g_drv.cuModuleLoadData);
    ok &= get_entry("cuModuleUnload", &g_drv.cuModuleUnload);
    ok &= get_entry("cuModuleGetFunction", &g_drv.cuModuleGetFunction);
    ok &= get_entry("cuFuncSetAttribute", &g_drv.cuFuncSetAttribute);
    ok &= get_entry("cuLaunchKernelEx", &g_drv.cuLaunchKernelEx);
    ok &= get_entry("cuTensorMapEncodeTiled", &g_drv.cuTensorMapEncodeTiled);
    g_drv.ok = ok;
  }
  if (!g_drv.ok) {
    g_drv.loaded = false;  // retry after a device is initialised
    return thork_set_error(THORK_ERR_UNAVAILABLE,
                           "CUDA driver entry points unavailable (no driver or no device)");
  }
  *api = &g_drv;
  return THORK_OK;
}

static int drv_error(CUresult r, const char *what) {
  const char *name = "CUDA_ERROR_UNKNOWN", *msg = "unknown";
  if (g_drv.cuGetErrorName) g_drv.cuGetErrorName(r, &name);
  if (g_drv.cuGetErrorString) g_drv.cuGetErrorString(r, &msg);
  return thork_set_error(THORK_ERR_CUDA, "CUDA error (%s): %s: %s", what, name, msg);
}

// ---------------------------------------------------------------------------
// devices
// ---------------------------------------------------------------------------
extern "C" int thork_device_count(int *count) {
  if (!count) return thork_set_error(THORK_ERR_INVALID, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    *count = 0;
    return THORK_OK;
  }
  *count = n;
  return THORK_OK;
}

extern "C" int thork_init(int dev) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaGetDeviceCount");
  if (dev < 0 || dev >= n)
    return thork_set_error(THORK_ERR_INVALID, "device %d out of range (have %d)", dev, n);
  CUDA_TRY(cudaSetDevice(dev), "cudaSetDevice");
  CUDA_TRY(cudaFree(nullptr), "context init");
  return THORK_OK;
}

extern "C" int thork_device_attr(int dev, int attr, int *value) {
  if (!value) return thork_set_error(THORK_ERR_INVALID, "value is NULL");
  cudaDeviceAttr a;
  switch (attr) {
    case THORK_ATTR_CC_MAJOR: a = cudaDevAttrComputeCapabilityMajor; break;
    case THORK_ATTR_CC_MINOR: a = cudaDevAttrComputeCapabilityMinor; break;
    case THORK_ATTR_SM_COUNT: a = cudaDevAttrMultiProcessorCount; break;
    case THORK_ATTR_SMEM_OPTIN: a = cudaDevAttrMaxSharedMemoryPerBlockOptin; break;
    case THORK_ATTR_L2_BYTES: a = cudaDevAttrL2CacheSize; break;
    case THORK_ATTR_CLOCK_KHZ: a = cudaDevAttrClockRate; break;
    case THORK_ATTR_MEM_CLOCK_KHZ: a = cudaDevAttrMemoryClockRate; break;
    case THORK_ATTR_PCI_DOMAIN: a = cudaDevAttrPciDomainId; break;
    case THORK_ATTR_PCI_BUS: a = cudaDevAttrPciBusId; break;
    case THORK_ATTR_PCI_DEVICE: a = cudaDevAttrPciDeviceId; break;
    default: return thork_set_error(THORK_ERR_INVALID, "unknown attribute %d", attr);
  }
  CUDA_TRY(cudaDeviceGetAttribute(value, a, dev), "cudaDeviceGetAttribute");
  return THORK_OK;
}

extern "C" int thork_device_synchronize(void) {
  CUDA_TRY(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// memory
// ---------------------------------------------------------------------------
extern "C" int thork_malloc(size_t nbytes, void **d_ptr) {
  if (!d_ptr) return thork_set_error(THORK_ERR_INVALID, "d_ptr is NULL");
  *d_ptr = nullptr;
  if (nbytes == 0) nbytes = 16;  // keep a valid, freeable pointer for empty arrays
  CUDA_TRY(cudaMalloc(d_ptr, nbytes), "cudaMalloc");
  return THORK_OK;
}

extern "C" int thork_free(void *d_ptr) {
  if (!d_ptr) return THORK_OK;
  CUDA_TRY(cudaFree(d_ptr), "cudaFree");
  return THORK_OK;
}

extern "C" int thork_host_alloc(size_t nbytes, void **h_ptr) {
  if (!h_ptr) return thork_set_error(THORK_ERR_INVALID, "h_ptr is NULL");
  if (nbytes == 0) nbytes = 16;
  CUDA_TRY(cudaHostAlloc(h_ptr, nbytes, cudaHostAllocPortable), "cudaHostAlloc");
  return THORK_OK;
}

extern "C" int thork_host_free(void *h_ptr) {
  if (!h_ptr) return THORK_OK;
  CUDA_TRY(cudaFreeHost(h_ptr), "cudaFreeHost");
  return THORK_OK;
}

static int do_copy(void *dst, const void *src, size_t n, cudaMemcpyKind kind, void *stream,
                   int sync, const char *what) {
  if (n == 0) return THORK_OK;
  if (!dst || !src) return thork_set_error(THORK_ERR_INVALID, "%s: NULL pointer", what);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // large copies to or from pageable memory take the pipelined pinned ring
  if (n >= thork_staged_min_bytes() && kind != cudaMemcpyDeviceToDevice &&
      thork_is_pageable(kind == cudaMemcpyHostToDevice ? src : dst)) {
    int rc = kind == cudaMemcpyHostToDevice ? thork_staged_htod(dst, src, n, s)
                                            : thork_staged_dtoh(dst, src, n, s);
    if (rc == THORK_OK && sync && kind == cudaMemcpyHostToDevice)
      CUDA_TRY(cudaStreamSynchronize(s), what);
    return rc;
  }
  if (sync && !s) {
    CUDA_TRY(cudaMemcpy(dst, src, n, kind), what);
  } else {
    CUDA_TRY(cudaMemcpyAsync(dst, src, n, kind, s), what);
    if (sync) CUDA_TRY(cudaStreamSynchronize(s), what);
  }
  return THORK_OK;
}

extern "C" int thork_memcpy_htod(void *d_dst, const void *h_src, size_t n, void *stream, int sync) {
  return do_copy(d_dst, h_src, n, cudaMemcpyHostToDevice, stream, sync, "memcpy HtoD");
}
extern "C" int thork_memcpy_dtoh(void *h_dst, const void *d_src, size_t n, void *stream, int sync) {
  return do_copy(h_dst, d_src, n, cudaMemcpyDeviceToHost, stream, sync, "memcpy DtoH");
}
extern "C" int thork_memcpy_dtod(void *d_dst, const void *d_src, size_t n, void *stream) {
  return do_copy(d_dst, d_src, n, cudaMemcpyDeviceToDevice, stream, 0, "memcpy DtoD");
}
extern "C" int thork_mem_info(size_t *free_bytes, size_t *total_bytes) {
  if (!free_bytes || !total_bytes) return thork_set_error(THORK_ERR_INVALID, "mem_info: NULL output");
  CUDA_TRY(cudaMemGetInfo(free_bytes, total_bytes), "cudaMemGetInfo");
  return THORK_OK;
}
extern "C" int thork_memset(void *d_ptr, int value, size_t n, void *stream) {
  if (n == 0) return THORK_OK;
  CUDA_TRY(cudaMemsetAsync(d_ptr, value, n, static_cast<cudaStream_t>(stream)), "cudaMemsetAsync");
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// streams / events
// ---------------------------------------------------------------------------
extern "C" int thork_stream_create(void **stream) {
  cudaStream_t s;
  CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
  *stream = s;
  return THORK_OK;
}
extern "C" int thork_stream_destroy(void *stream) {
  if (!stream) return THORK_OK;
  CUDA_TRY(cudaStreamDestroy(static_cast<cudaStream_t>(stream)), "cudaStreamDestroy");
  return THORK_OK;
}
extern "C" int thork_stream_synchronize(void *stream) {
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
  return THORK_OK;
}
extern "C" int thork_event_create(void **event) {
  cudaEvent_t e;
  CUDA_TRY(cudaEventCreate(&e), "cudaEventCreate");
  *event = e;
  return THORK_OK;
}
extern "C" int thork_event_destroy(void *event) {
  if (!event) return THORK_OK;
  CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "cudaEventDestroy");
  return THORK_OK;
}
extern "C" int thork_event_record(void *event, void *stream) {
  CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)),
           "cudaEventRecord");
  return THORK_OK;
}
extern "C" int thork_event_synchronize(void *event) {
  CUDA_TRY(cudaEventSynchronize(static_cast<cudaEvent_t>(event)), "cudaEventSynchronize");
  return THORK_OK;
}
extern "C" int thork_event_elapsed_ms(void *start, void *end, float *ms) {
  CUDA_TRY(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)),
           "cudaEventElapsedTime");
  return THORK_OK;
}

extern "C" int thork_stream_wait_event(void *stream, void *event) {
  CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0),
           "cudaStreamWaitEvent");
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// CUDA IPC (peer buffers of the fused GEMM + all-gather)
// ---------------------------------------------------------------------------
extern "C" int thork_ipc_handle(const void *d_ptr, void *handle64) {
  if (!d_ptr || !handle64) return thork_set_error(THORK_ERR_INVALID, "ipc_handle: NULL argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void *>(d_ptr)), "cudaIpcGetMemHandle");
  memcpy(handle64, &h, sizeof(h));
  return THORK_OK;
}

extern "C" int thork_ipc_open(const void *handle64, void **d_ptr) {
  if (!d_ptr || !handle64) return thork_set_error(THORK_ERR_INVALID, "ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return THORK_OK;
}

extern "C" int thork_ipc_close(void *d_ptr) {
  if (!d_ptr) return THORK_OK;
  CUDA_TRY(cudaIpcCloseMemHandle(d_ptr), "cudaIpcCloseMemHandle");
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// NVRTC (dlopen)
// ---------------------------------------------------------------------------
struct NvrtcApi {
  bool tried = false;
  void *handle = nullptr;
  nvrtcResult (*Version)(int *, int *);
  const char *(*GetErrorString)(nvrtcResult);
  nvrtcResult (*CreateProgram)(nvrtcProgram *, const char *, const char *, int, const char *const *,
                               const char *const *);
  nvrtcResult (*DestroyProgram)(nvrtcProgram *);
  nvrtcResult (*CompileProgram)(nvrtcProgram, int, const char *const *);
  nvrtcResult (*GetProgramLogSize)(nvrtcProgram, size_t *);
  nvrtcResult (*GetProgramLog)(nvrtcProgram, char *);
  nvrtcResult (*GetCUBINSize)(nvrtcProgram, size_t *);
  nvrtcResult (*GetCUBIN)(nvrtcProgram, char *);
};
static NvrtcApi g_nvrtc;
static std::mutex g_nvrtc_mu;

static void *open_first(const char *const *names) {
  for (int i = 0; names[i]; ++i) {
    void *h = dlopen(names[i], RTLD_NOW | RTLD_GLOBAL);
    if (h) return h;
  }
  return nullptr;
}

static int nvrtc_api(NvrtcApi **api) {
  std::lock_guard<std::mutex> lk(g_nvrtc_mu);
  if (!g_nvrtc.tried) {
    g_nvrtc.tried = true;
    std::string home;
    const char *ch = getenv("CUDA_HOME");
    if (ch) home = std::string(ch) + "/lib64/libnvrtc.so.12";
    const char *names[] = {"libnvrtc.so.12", home.empty() ? "libnvrtc.so" : home.c_str(),
                           "/usr/local/cuda/lib64/libnvrtc.so.12", "libnvrtc.so", nullptr};
    void *h = open_first(names);
    if (h) {
      bool ok = true;
#define LOAD(field, sym) ok &= (*(void **)&g_nvrtc.field = dlsym(h, sym)) != nullptr
      LOAD(Version, "nvrtcVersion");
      LOAD(GetErrorString, "nvrtcGetErrorString");
      LOAD(CreateProgram, "nvrtcCreateProgram");
      LOAD(DestroyProgram, "nvrtcDestroyProgram");
      LOAD(CompileProgram, "nvrtcCompileProgram");
      LOAD(GetProgramLogSize, "nvrtcGetProgramLogSize");
      LOAD(GetProgramLog, "nvrtcGetProgramLog");
      LOAD(GetCUBINSize, "nvrtcGetCUBINSize");
      LOAD(GetCUBIN, "nvrtcGetCUBIN");
#undef LOAD
      if (ok) g_nvrtc.handle = h;
    }
  }
  if (!g_nvrtc.handle)
    return thork_set_error(THORK_ERR_UNAVAILABLE, "NVRTC (libnvrtc.so.12) could not be loaded");
  *api = &g_nvrtc;
  return THORK_OK;
}

extern "C" int thork_nvrtc_version(int *major, int *minor) {
  NvrtcApi *api;
  int rc = nvrtc_api(&api);
  if (rc) return rc;
  nvrtcResult r = api->Version(major, minor);
  if (r != NVRTC_SUCCESS)
    return thork_set_error(THORK_ERR_NVRTC, "nvrtcVersion: %s", api->GetErrorString(r));
  return THORK_OK;
}

extern "C" int thork_nvrtc_compile(const char *source, const char *name, const char *arch,
                                   const char **opts, int n_opts, void **cubin,
                                   size_t *cubin_size, char **log) {
  if (!source || !cubin || !cubin_size || !log)
    return thork_set_error(THORK_ERR_INVALID, "thork_nvrtc_compile: NULL argument");
  *cubin = nullptr;
  *cubin_size = 0;
  *log = nullptr;
  NvrtcApi *api;
  int rc = nvrtc_api(&api);
  if (rc) return rc;
  nvrtcProgram prog;
  nvrtcResult r =
      api->CreateProgram(&prog, source, name ? name : "thork_kernel.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS)
    return thork_set_error(THORK_ERR_NVRTC, "nvrtcCreateProgram: %s", api->GetErrorString(r));
  std::string arch_opt = std::string("-arch=") + (arch ? arch : "sm_100a");
  const char **all = static_cast<const char **>(malloc(sizeof(char *) * (n_opts + 1)));
  all[0] = arch_opt.c_str();
  for (int i = 0; i < n_opts; ++i) all[i + 1] = opts[i];
  nvrtcResult cr = api->CompileProgram(prog, n_opts + 1, all);
  free(all);
  size_t log_size = 0;
  api->GetProgramLogSize(prog, &log_size);
  if (log_size > 1) {
    *log = static_cast<char *>(malloc(log_size + 1));
    api->GetProgramLog(prog, *log);
    (*log)[log_size] = 0;
  }
  if (cr != NVRTC_SUCCESS) {
    api->DestroyProgram(&prog);
    return thork_set_error(THORK_ERR_NVRTC, "NVRTC compile failed: %s", api->GetErrorString(cr));
  }
  size_t n = 0;
  r = api->GetCUBINSize(prog, &n);
  if (r != NVRTC_SUCCESS || n == 0) {
    api->DestroyProgram(&prog);
    return thork_set_error(THORK_ERR_NVRTC, "nvrtcGetCUBINSize: %s (is arch a real sm_ target?)",
                           api->GetErrorString(r));
  }
  char *buf = static_cast<char *>(malloc(n));
  api->GetCUBIN(prog, buf);
  api->DestroyProgram(&prog);
  *cubin = buf;
  *cubin_size = n;
  return THORK_OK;
}

extern "C" int thork_buffer_free(void *buf) {
  free(buf);
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// modules / launches
// ---------------------------------------------------------------------------
extern "C" int thork_module_load(const void *image, void **module) {
  if (!image || !module) return thork_set_error(THORK_ERR_INVALID, "module_load: NULL argument");
  DriverApi *d;
  int rc = driver_api(&d);
  if (rc) return rc;
  CUmodule m;
  CUresult r = d->cuModuleLoadData(&m, image);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuModuleLoadData");
  *module = m;
  return THORK_OK;
}

extern "C" int thork_module_unload(void *module) {
  if (!module) return THORK_OK;
  DriverApi *d;
  int rc = driver_api(&d);
  if (rc) return rc;
  CUresult r = d->cuModuleUnload(static_cast<CUmodule>(module));
  if (r != CUDA_SUCCESS) return drv_error(r, "cuModuleUnload");
  return THORK_OK;
}

extern "C" int thork_module_get_function(void *module, const char *name, void **function) {
  if (!module || !name || !function)
    return thork_set_error(THORK_ERR_INVALID, "get_function: NULL argument");
  DriverApi *d;
  int rc = driver_api(&d);
  if (rc) return rc;
  CUfunction f;
  CUresult r = d->cuModuleGetFunction(&f, static_cast<CUmodule>(module), name);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuModuleGetFunction");
  *function = f;
  return THORK_OK;
}

extern "C" int thork_function_set_max_dynamic_smem(void *function, int nbytes) {
  DriverApi *d;
  int rc = driver_api(&d);
  if (rc) return rc;
  CUresult r = d->cuFuncSetAttribute(static_cast<CUfunction>(function),
                                     CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, nbytes);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuFuncSetAttribute");
  return THORK_OK;
}

extern "C" int thork_launch(void *function, const unsigned grid[3], const unsigned block[3],
                            const unsigned cluster[3], unsigned smem_bytes, void *stream,
                            void **args) {
  if (!function || !grid || !block)
    return thork_set_error(THORK_ERR_INVALID, "launch: NULL argument");
  DriverApi *d;
  int rc = driver_api(&d);
  if (rc) return rc;
  CUlaunchConfig cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDimX = grid[0];
  cfg.gridDimY = grid[1];
  cfg.gridDimZ = grid[2];
  cfg.blockDimX = block[0];
  cfg.blockDimY = block[1];
  cfg.blockDimZ = block[2];
  cfg.sharedMemBytes = smem_bytes;
  cfg.hStream = static_cast<CUstream>(stream);
  CUlaunchAttribute attr;
  if (cluster && (cluster[0] * cluster[1] * cluster[2]) > 1) {
    attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr.value.clusterDim.x = cluster[0];
    attr.value.clusterDim.y = cluster[1];
    attr.value.clusterDim.z = cluster[2];
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
  }
  CUresult r = d->cuLaunchKernelEx(&cfg, static_cast<CUfunction>(function), args, nullptr);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuLaunchKernelEx");
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// TMA descriptors
// ---------------------------------------------------------------------------
int thork_encode_tmap_2d(void *out128, int dtype, const void *base, uint64_t rows, uint64_t cols,
                         uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols,
                         int swizzle_bytes) {
  if (!out128 || (reinterpret_cast<uintptr_t>(out128) & 63))
    return thork_set_error(THORK_ERR_INVALID, "tensor map output must be 64-byte aligned");
  DriverApi *d;
  int rc = driver_api(&d);
  if (rc) return rc;
  CUtensorMapDataType t;
  switch (dtype) {
    case THORK_DT_U8:
    case THORK_DT_E4M3: t = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case THORK_DT_U16: t = CU_TENSOR_MAP_DATA_TYPE_UINT16; break;
    case THORK_DT_BF16: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case THORK_DT_F16: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case THORK_DT_U32: t = CU_TENSOR_MAP_DATA_TYPE_UINT32; break;
    case THORK_DT_F32: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: return thork_set_error(THORK_ERR_INVALID, "tensor map: unknown dtype %d", dtype);
  }
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return thork_set_error(THORK_ERR_INVALID, "tensor map: bad swizzle %d", swizzle_bytes);
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = d->cuTensorMapEncodeTiled(
      reinterpret_cast<CUtensorMap *>(out128), t, 2, const_cast<void *>(base), dims, strides, box,
      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return drv_error(r, "cuTensorMapEncodeTiled");
  return THORK_OK;
}

extern "C" int thork_tensor_map_2d(void *out128, int dtype, const void *d_base, uint64_t rows,
                                   uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows,
                                   uint32_t box_cols, int swizzle_bytes) {
  return thork_encode_tmap_2d(out128, dtype, d_base, rows, cols, row_stride_bytes, box_rows,
                              box_cols, swizzle_bytes);
}

// ---------------------------------------------------------------------------
// NCCL (dlopen)
// ---------------------------------------------------------------------------
typedef struct {
  char internal[128];
} thork_nccl_id_t;
typedef int thork_ncclResult;  // ncclResult_t: 0 == ncclSuccess
struct NcclApi {
  bool tried = false;
  void *handle = nullptr;
  thork_ncclResult (*GetUniqueId)(thork_nccl_id_t *);
  thork_ncclResult (*CommInitRank)(void **, int, thork_nccl_id_t, int);
  thork_ncclResult (*CommDestroy)(void *);
  thork_ncclResult (*AllGather)(const void *, void *, size_t, int, void *, cudaStream_t);
  thork_ncclResult (*AllReduce)(const void *, void *, size_t, int, int, void *, cudaStream_t);
  const char *(*GetErrorString)(thork_ncclResult);
};
static NcclApi g_nccl;
static std::mutex g_nccl_mu;

static int nccl_api(NcclApi **api) {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (!g_nccl.tried) {
    g_nccl.tried = true;
    const char *names[] = {"libnccl.so.2", "/usr/lib/x86_64-linux-gnu/libnccl.so.2", "libnccl.so",
                           nullptr};
    void *h = open_first(names);
    if (h) {
      bool ok = true;
#define LOAD(field, sym) ok &= (*(void **)&g_nccl.field = dlsym(h, sym)) != nullptr
      LOAD(GetUniqueId, "ncclGetUniqueId");
      LOAD(CommInitRank, "ncclCommInitRank");
      LOAD(CommDestroy, "ncclCommDestroy");
      LOAD(AllGather, "ncclAllGather");
      LOAD(AllReduce, "ncclAllReduce");
      LOAD(GetErrorString, "ncclGetErrorString");
#undef LOAD
      if (ok) g_nccl.handle = h;
    }
  }
  if (!g_nccl.handle)
    return thork_set_error(THORK_ERR_UNAVAILABLE, "NCCL (libnccl.so.2) could not be loaded");
  *api = &g_nccl;
  return THORK_OK;
}

static int nccl_dtype(int dtype, int *out) {
  // ncclDataType_t values: ncclUint8=1, ncclUint32=3, ncclFloat16=6, ncclFloat32=7, ncclBfloat16=9
  switch (dtype) {
    case THORK_DT_U8:
    case THORK_DT_E4M3: *out = 1; return THORK_OK;
    case THORK_DT_U32: *out = 3; return THORK_OK;
    case THORK_DT_F16:
    case THORK_DT_U16: *out = 6; return THORK_OK;
    case THORK_DT_F32: *out = 7; return THORK_OK;
    case THORK_DT_BF16: *out = 9; return THORK_OK;
  }
  return thork_set_error(THORK_ERR_INVALID, "nccl: unsupported dtype %d", dtype);
}

static int nccl_error(NcclApi *api, thork_ncclResult r, const char *what) {
  return thork_set_error(THORK_ERR_NCCL, "NCCL error (%s): %s", what, api->GetErrorString(r));
}

extern "C" int thork_nccl_get_unique_id(void *id128) {
  if (!id128) return thork_set_error(THORK_ERR_INVALID, "id128 is NULL");
  NcclApi *api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  thork_nccl_id_t id;
  thork_ncclResult r = api->GetUniqueId(&id);
  if (r) return nccl_error(api, r, "ncclGetUniqueId");
  memcpy(id128, &id, sizeof(id));
  return THORK_OK;
}

extern "C" int thork_nccl_comm_init_rank(void **comm, int nranks, const void *id128, int rank) {
  if (!comm || !id128) return thork_set_error(THORK_ERR_INVALID, "comm_init_rank: NULL argument");
  const char *fault = getenv("THORK_FAULT_NCCL_INIT");
  if (fault && fault[0] == '1')
    return thork_set_error(THORK_ERR_NCCL,
                           "NCCL error (ncclCommInitRank): injected failure (THORK_FAULT_NCCL_INIT=1)");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return thork_set_error(THORK_ERR_INVALID, "comm_init_rank: rank %d of %d", rank, nranks);
  NcclApi *api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  thork_nccl_id_t id;
  memcpy(&id, id128, sizeof(id));
  thork_ncclResult r = api->CommInitRank(comm, nranks, id, rank);
  if (r) return nccl_error(api, r, "ncclCommInitRank");
  return THORK_OK;
}

extern "C" int thork_nccl_comm_destroy(void *comm) {
  if (!comm) return THORK_OK;
  NcclApi *api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  thork_ncclResult r = api->CommDestroy(comm);
  if (r) return nccl_error(api, r, "ncclCommDestroy");
  return THORK_OK;
}

extern "C" int thork_nccl_allgather(const void *d_send, void *d_recv, size_t count, int dtype,
                                    void *comm, void *stream) {
  NcclApi *api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  int t;
  if ((rc = nccl_dtype(dtype, &t))) return rc;
  thork_ncclResult r =
      api->AllGather(d_send, d_recv, count, t, comm, static_cast<cudaStream_t>(stream));
  if (r) return nccl_error(api, r, "ncclAllGather");
  return THORK_OK;
}

extern "C" int thork_nccl_allreduce_sum(void *d_buf, size_t count, int dtype, void *comm,
                                        void *stream) {
  NcclApi *api;
  int rc = nccl_api(&api);
  if (rc) return rc;
  int t;
  if ((rc = nccl_dtype(dtype, &t))) return rc;
  thork_ncclResult r =
      api->AllReduce(d_buf, d_buf, count, t, /*ncclSum=*/0, comm, static_cast<cudaStream_t>(stream));
  if (r) return nccl_error(api, r, "ncclAllReduce");
  return THORK_OK;
}
