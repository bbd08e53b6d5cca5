// multicast.cu — NVLink multicast buffers (NVSwitch "NVLS") for the fused
// GEMM + all-gather: one physical allocation per GPU, all bound to one
// multicast object, so a single `multimem.st` from any GPU lands at the same
// offset in every GPU's memory.  C-ABI in include/thork_rt.h (thork_mc_*).
//
// Life cycle (one process per GPU):
//   rank 0:   thork_mc_create  -> object + POSIX file descriptor to share
//   others:   thork_mc_import  (the descriptor travels over a Unix socket)
//   every rank: thork_mc_add_device   (host barrier: all devices added)
//   every rank: thork_mc_bind         (host barrier: all bound before use)
//   every rank: thork_mc_release      (after a host barrier: nobody writes)
// The driver's VMM and multicast entry points are looked up at run time, so
// the library still loads without a driver.
#include <cuda.h>
#include <cuda_runtime.h>
#include <unistd.h>

#include <cstdint>
#include <mutex>

#include "thork_internal.h"
#include "thork_rt.h"

namespace {

struct McApi {
  bool loaded = false, ok = false;
  CUresult (*GetErrorName)(CUresult, const char **) = nullptr;
  CUresult (*DeviceGet)(CUdevice *, int) = nullptr;
  CUresult (*DeviceGetAttribute)(int *, CUdevice_attribute, CUdevice) = nullptr;
  CUresult (*MulticastCreate)(CUmemGenericAllocationHandle *, const CUmulticastObjectProp *) = nullptr;
  CUresult (*MulticastGetGranularity)(size_t *, const CUmulticastObjectProp *,
                                      CUmulticastGranularity_flags) = nullptr;
  CUresult (*MulticastAddDevice)(CUmemGenericAllocationHandle, CUdevice) = nullptr;
  CUresult (*MulticastBindMem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle,
                               size_t, size_t, unsigned long long) = nullptr;
  CUresult (*MulticastUnbind)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t) = nullptr;
  CUresult (*MemCreate)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *,
                        unsigned long long) = nullptr;
  CUresult (*MemRelease)(CUmemGenericAllocationHandle) = nullptr;
  CUresult (*MemGetAllocationGranularity)(size_t *, const CUmemAllocationProp *,
                                          CUmemAllocationGranularity_flags) = nullptr;
  CUresult (*MemAddressReserve)(CUdeviceptr *, size_t, size_t, CUdeviceptr,
                                unsigned long long) = nullptr;
  CUresult (*MemAddressFree)(CUdeviceptr, size_t) = nullptr;
  CUresult (*MemMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle,
                     unsigned long long) = nullptr;
  CUresult (*MemUnmap)(CUdeviceptr, size_t) = nullptr;
  CUresult (*MemSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t) = nullptr;
  CUresult (*MemExportToShareableHandle)(void *, CUmemGenericAllocationHandle,
                                         CUmemAllocationHandleType, unsigned long long) = nullptr;
  CUresult (*MemImportFromShareableHandle)(CUmemGenericAllocationHandle *, void *,
                                           CUmemAllocationHandleType) = nullptr;
};

McApi g_mc;
std::mutex g_mc_mu;

template <class F>
bool entry(const char *name, F *out) {
  void *p = nullptr;
  cudaDriverEntryPointQueryResult q;
  // the multicast entry points first appeared in CUDA 12.1: ask for the
  // versions of the toolkit this library was built with
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &p, CUDA_VERSION, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) return false;
  *out = reinterpret_cast<F>(p);
  return true;
}

int mc_api(McApi **api) {
  std::lock_guard<std::mutex> lk(g_mc_mu);
  if (!g_mc.loaded) {
    g_mc.loaded = true;
    bool ok = true;
    ok &= entry("cuGetErrorName", &g_mc.GetErrorName);
    ok &= entry("cuDeviceGet", &g_mc.DeviceGet);
    ok &= entry("cuDeviceGetAttribute", &g_mc.DeviceGetAttribute);
    ok &= entry("cuMulticastCreate", &g_mc.MulticastCreate);
    ok &= entry("cuMulticastGetGranularity", &g_mc.MulticastGetGranularity);
    ok &= entry("cuMulticastAddDevice", &g_mc.MulticastAddDevice);
    ok &= entry("cuMulticastBindMem", &g_mc.MulticastBindMem);
    ok &= entry("cuMulticastUnbind", &g_mc.MulticastUnbind);
    ok &= entry("cuMemCreate", &g_mc.MemCreate);
    ok &= entry("cuMemRelease", &g_mc.MemRelease);
    ok &= entry("cuMemGetAllocationGranularity", &g_mc.MemGetAllocationGranularity);
    ok &= entry("cuMemAddressReserve", &g_mc.MemAddressReserve);
    ok &= entry("cuMemAddressFree", &g_mc.MemAddressFree);
    ok &= entry("cuMemMap", &g_mc.MemMap);
    ok &= entry("cuMemUnmap", &g_mc.MemUnmap);
    ok &= entry("cuMemSetAccess", &g_mc.MemSetAccess);
    ok &= entry("cuMemExportToShareableHandle", &g_mc.MemExportToShareableHandle);
    ok &= entry("cuMemImportFromShareableHandle", &g_mc.MemImportFromShareableHandle);
    g_mc.ok = ok;
  }
  if (!g_mc.ok) {
    g_mc.loaded = false;
    return thork_set_error(THORK_ERR_UNAVAILABLE,
                           "CUDA multicast / VMM entry points unavailable (no driver or too old)");
  }
  *api = &g_mc;
  return THORK_OK;
}

int mc_err(CUresult r, const char *what) {
  const char *name = "CUDA_ERROR_UNKNOWN";
  if (g_mc.GetErrorName) g_mc.GetErrorName(r, &name);
  return thork_set_error(THORK_ERR_CUDA, "CUDA error (%s): %s", what, name);
}

#define MC_TRY(call, what)                   \
  do {                                       \
    CUresult r_ = (call);                    \
    if (r_ != CUDA_SUCCESS) return mc_err(r_, what); \
  } while (0)

int current_cu_device(McApi *a, CUdevice *dev, int *ordinal) {
  cudaError_t e = cudaGetDevice(ordinal);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaGetDevice");
  e = cudaFree(nullptr);  // the primary context is current from here on
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaFree(0)");
  MC_TRY(a->DeviceGet(dev, *ordinal), "cuDeviceGet");
  return THORK_OK;
}

// One rank's view of a multicast buffer.
struct McBuffer {
  CUmemGenericAllocationHandle mc = 0;    // the multicast object
  CUmemGenericAllocationHandle phys = 0;  // this GPU's memory bound to it
  size_t bytes = 0;
  size_t gran = 0;
  CUdevice dev = 0;
  int fd = -1;                 // exported descriptor (creator only)
  CUdeviceptr local = 0;       // this GPU's memory, ordinary (unicast) view
  CUdeviceptr multi = 0;       // the multicast view: stores reach every GPU
  bool added = false, bound = false;
};

CUmulticastObjectProp mc_prop(int ndev, size_t bytes) {
  CUmulticastObjectProp p = {};
  p.numDevices = static_cast<unsigned>(ndev);
  p.size = bytes;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  p.flags = 0;
  return p;
}

// Memory bound to a multicast object must be shareable with the object's
// handle type (measured: cuMulticastBindMem refuses memory created without
// it with CUDA_ERROR_INVALID_VALUE).
CUmemAllocationProp phys_prop(CUdevice dev) {
  CUmemAllocationProp p = {};
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = static_cast<int>(dev);
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

}  // namespace

extern "C" int thork_mc_supported(int *supported) {
  if (!supported) return thork_set_error(THORK_ERR_INVALID, "mc_supported: NULL output");
  *supported = 0;
  McApi *a;
  int rc, ord;
  if ((rc = mc_api(&a))) return rc;
  CUdevice dev;
  if ((rc = current_cu_device(a, &dev, &ord))) return rc;
  int mc = 0, fd = 0;
  MC_TRY(a->DeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev),
         "cuDeviceGetAttribute(multicast)");
  MC_TRY(a->DeviceGetAttribute(&fd, CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR_SUPPORTED,
                               dev),
         "cuDeviceGetAttribute(posix fd handles)");
  *supported = (mc && fd) ? 1 : 0;
  return THORK_OK;
}

extern "C" int thork_mc_create(size_t bytes, int ndev, void **obj, int *fd, size_t *bytes_rounded) {
  if (!obj || !fd || !bytes_rounded || bytes == 0 || ndev < 1 || ndev > 8)
    return thork_set_error(THORK_ERR_INVALID, "mc_create: bad arguments (bytes=%zu ndev=%d)", bytes,
                           ndev);
  McApi *a;
  int rc, ord;
  if ((rc = mc_api(&a))) return rc;
  CUdevice dev;
  if ((rc = current_cu_device(a, &dev, &ord))) return rc;
  CUmulticastObjectProp p = mc_prop(ndev, bytes);
  size_t g_mc = 0, g_ph = 0;
  MC_TRY(a->MulticastGetGranularity(&g_mc, &p, CU_MULTICAST_GRANULARITY_RECOMMENDED),
         "cuMulticastGetGranularity");
  CUmemAllocationProp pp = phys_prop(dev);
  MC_TRY(a->MemGetAllocationGranularity(&g_ph, &pp, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED),
         "cuMemGetAllocationGranularity");
  const size_t gran = g_mc > g_ph ? g_mc : g_ph;
  p.size = (bytes + gran - 1) / gran * gran;
  McBuffer *b = new McBuffer;
  b->bytes = p.size;
  b->gran = gran;
  b->dev = dev;
  CUresult r = a->MulticastCreate(&b->mc, &p);
  if (r != CUDA_SUCCESS) {
    delete b;
    return mc_err(r, "cuMulticastCreate");
  }
  r = a->MemExportToShareableHandle(&b->fd, b->mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    a->MemRelease(b->mc);
    delete b;
    return mc_err(r, "cuMemExportToShareableHandle(multicast)");
  }
  *obj = b;
  *fd = b->fd;
  *bytes_rounded = b->bytes;
  return THORK_OK;
}

extern "C" int thork_mc_import(int fd, size_t bytes_rounded, void **obj) {
  if (!obj || fd < 0 || bytes_rounded == 0)
    return thork_set_error(THORK_ERR_INVALID, "mc_import: bad arguments");
  McApi *a;
  int rc, ord;
  if ((rc = mc_api(&a))) return rc;
  CUdevice dev;
  if ((rc = current_cu_device(a, &dev, &ord))) return rc;
  McBuffer *b = new McBuffer;
  b->bytes = bytes_rounded;
  b->dev = dev;
  CUmemAllocationProp pp = phys_prop(dev);
  CUresult r = a->MemGetAllocationGranularity(&b->gran, &pp, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
  if (r == CUDA_SUCCESS)
    r = a->MemImportFromShareableHandle(&b->mc, reinterpret_cast<void *>(static_cast<intptr_t>(fd)),
                                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  if (r != CUDA_SUCCESS) {
    delete b;
    return mc_err(r, "cuMemImportFromShareableHandle(multicast)");
  }
  if (b->bytes % b->gran) {
    a->MemRelease(b->mc);
    delete b;
    return thork_set_error(THORK_ERR_INVALID, "mc_import: size %zu is not a multiple of %zu",
                           bytes_rounded, b->gran);
  }
  *obj = b;
  return THORK_OK;
}

extern "C" int thork_mc_add_device(void *obj) {
  McBuffer *b = static_cast<McBuffer *>(obj);
  if (!b) return thork_set_error(THORK_ERR_INVALID, "mc_add_device: NULL object");
  McApi *a;
  int rc;
  if ((rc = mc_api(&a))) return rc;
  MC_TRY(a->MulticastAddDevice(b->mc, b->dev), "cuMulticastAddDevice");
  b->added = true;
  return THORK_OK;
}

extern "C" int thork_mc_bind(void *obj, void **d_local, void **d_multicast) {
  McBuffer *b = static_cast<McBuffer *>(obj);
  if (!b || !d_local || !d_multicast || !b->added)
    return thork_set_error(THORK_ERR_INVALID, "mc_bind: NULL argument or device not added");
  McApi *a;
  int rc;
  if ((rc = mc_api(&a))) return rc;
  CUmemAllocationProp pp = phys_prop(b->dev);
  MC_TRY(a->MemCreate(&b->phys, b->bytes, &pp, 0), "cuMemCreate");
  MC_TRY(a->MulticastBindMem(b->mc, 0, b->phys, 0, b->bytes, 0), "cuMulticastBindMem");
  b->bound = true;
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = static_cast<int>(b->dev);
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  MC_TRY(a->MemAddressReserve(&b->local, b->bytes, b->gran, 0, 0), "cuMemAddressReserve(local)");
  MC_TRY(a->MemMap(b->local, b->bytes, 0, b->phys, 0), "cuMemMap(local)");
  MC_TRY(a->MemSetAccess(b->local, b->bytes, &acc, 1), "cuMemSetAccess(local)");
  MC_TRY(a->MemAddressReserve(&b->multi, b->bytes, b->gran, 0, 0), "cuMemAddressReserve(multicast)");
  MC_TRY(a->MemMap(b->multi, b->bytes, 0, b->mc, 0), "cuMemMap(multicast)");
  MC_TRY(a->MemSetAccess(b->multi, b->bytes, &acc, 1), "cuMemSetAccess(multicast)");
  *d_local = reinterpret_cast<void *>(b->local);
  *d_multicast = reinterpret_cast<void *>(b->multi);
  return THORK_OK;
}

extern "C" int thork_mc_release(void *obj) {
  McBuffer *b = static_cast<McBuffer *>(obj);
  if (!b) return THORK_OK;
  McApi *a;
  int rc;
  if ((rc = mc_api(&a))) return rc;
  cudaDeviceSynchronize();  // this GPU's stores through the multicast view are done
  int first = THORK_OK;
  auto note = [&](CUresult r, const char *what) {
    if (r != CUDA_SUCCESS && first == THORK_OK) first = mc_err(r, what);
  };
  if (b->multi) {
    note(a->MemUnmap(b->multi, b->bytes), "cuMemUnmap(multicast)");
    note(a->MemAddressFree(b->multi, b->bytes), "cuMemAddressFree(multicast)");
  }
  if (b->bound) note(a->MulticastUnbind(b->mc, b->dev, 0, b->bytes), "cuMulticastUnbind");
  if (b->local) {
    note(a->MemUnmap(b->local, b->bytes), "cuMemUnmap(local)");
    note(a->MemAddressFree(b->local, b->bytes), "cuMemAddressFree(local)");
  }
  if (b->phys) note(a->MemRelease(b->phys), "cuMemRelease(physical)");
  if (b->mc) note(a->MemRelease(b->mc), "cuMemRelease(multicast)");
  if (b->fd >= 0) close(b->fd);
  delete b;
  return first;
}
