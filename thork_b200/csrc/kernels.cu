// kernels.cu — the library kernels of libthork_rt.so and their C-ABI entry
// points (declared in include/thork_rt.h):
//   thork_matrix_add_f32    128-bit vectorised, grid-stride fp32 add
//   thork_gemm_bf16         tcgen05 GEMM, bf16 x bf16 -> fp32 -> bf16
//   thork_gemm_e4m3         tcgen05 GEMM, e4m3 x e4m3 -> fp32 -> scaled bf16
//   thork_skinny_gemm_bf16  swap-AB tcgen05 GEMM for M <= 256 (decode shapes)
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <utility>

#include "device/gemm_sm100.cuh"
#include "thork_internal.h"
#include "thork_rt.h"

using thork::dev::TensorMap;
using thork::dev::u32;

// ---------------------------------------------------------------------------
// per-device state: status word, SM count, smem opt-in flags
// ---------------------------------------------------------------------------
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
unsigned *g_status[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
uint64_t g_smem_set[kMaxDevices] = {};  // bit i: kernel i has its smem attribute set

int current_device(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices)
    return thork_set_error(THORK_ERR_INVALID, "device index %d too large", *dev);
  return THORK_OK;
}
}  // namespace

int thork_status_word(unsigned **d_status) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_status[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, 16);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaMalloc(status word)");
    e = cudaMemset(p, 0, 16);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaMemset(status word)");
    g_status[dev] = static_cast<unsigned *>(p);
  }
  *d_status = g_status[dev];
  return THORK_OK;
}

int thork_sm_count(int *n) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_sms[dev]) {
    cudaError_t e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaDeviceGetAttribute(SM count)");
  }
  *n = g_sms[dev];
  return THORK_OK;
}

static int ensure_smem(const void *kernel, int kernel_id, int bytes) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!(g_smem_set[dev] & (1ull << kernel_id))) {
    cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaFuncSetAttribute(max dynamic smem)");
    g_smem_set[dev] |= 1ull << kernel_id;
  }
  return THORK_OK;
}

extern "C" int thork_kernel_status(unsigned *status, int clear) {
  if (!status) return thork_set_error(THORK_ERR_INVALID, "status is NULL");
  unsigned *d;
  int rc = thork_status_word(&d);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaDeviceSynchronize");
  e = cudaMemcpy(status, d, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return thork_cuda_error(e, "read status word");
  if (clear) {
    e = cudaMemset(d, 0, 16);
    if (e != cudaSuccess) return thork_cuda_error(e, "clear status word");
  }
  return THORK_OK;
}

extern "C" int thork_status_pointer(void **d_status) {
  if (!d_status) return thork_set_error(THORK_ERR_INVALID, "d_status is NULL");
  unsigned *d;
  int rc = thork_status_word(&d);
  if (rc) return rc;
  *d_status = d;
  return THORK_OK;
}

static int launch_check(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return thork_cuda_error(e, what);
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// elementwise add
// ---------------------------------------------------------------------------
// Each thread keeps 4 float4 loads of each input in flight per iteration;
// loads and stores use the streaming (evict-first) cache policy because
// every byte is touched once.
__global__ void __launch_bounds__(256) add_f32_v4_kernel(float4 *__restrict__ out,
                                                         const float4 *__restrict__ a,
                                                         const float4 *__restrict__ b, size_t n4) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 x[4], y[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      x[u] = __ldcs(a + i + u * stride);
      y[u] = __ldcs(b + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float4 r;
      r.x = x[u].x + y[u].x;
      r.y = x[u].y + y[u].y;
      r.z = x[u].z + y[u].z;
      r.w = x[u].w + y[u].w;
      __stcs(out + i + u * stride, r);
    }
  }
  for (; i < n4; i += stride) {
    const float4 x = __ldcs(a + i), y = __ldcs(b + i);
    float4 r;
    r.x = x.x + y.x;
    r.y = x.y + y.y;
    r.z = x.z + y.z;
    r.w = x.w + y.w;
    __stcs(out + i, r);
  }
}

// Scalar grid-stride add for the ragged tail and for unaligned pointers.
__global__ void __launch_bounds__(256) add_f32_scalar_kernel(float *__restrict__ out,
                                                             const float *__restrict__ a,
                                                             const float *__restrict__ b, size_t n) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = a[i] + b[i];
}

extern "C" int thork_matrix_add_f32(float *d_out, const float *d_a, const float *d_b, size_t n,
                                    void *stream) {
  if (n == 0) return THORK_OK;
  if (!d_out || !d_a || !d_b) return thork_set_error(THORK_ERR_INVALID, "matrix_add: NULL pointer");
  int sms, rc;
  if ((rc = thork_sm_count(&sms))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(d_out) | reinterpret_cast<uintptr_t>(d_a) |
        reinterpret_cast<uintptr_t>(d_b)) & 15u) == 0;
  const size_t n4 = aligned ? n / 4 : 0;
  if (n4) {
    // 8 resident 256-thread blocks per SM, fewer when the array is small.
    size_t blocks = (n4 + 255) / 256;
    const size_t cap = static_cast<size_t>(sms) * 8;
    if (blocks > cap) blocks = cap;
    add_f32_v4_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        reinterpret_cast<float4 *>(d_out), reinterpret_cast<const float4 *>(d_a),
        reinterpret_cast<const float4 *>(d_b), n4);
    if ((rc = launch_check("add_f32_v4_kernel launch"))) return rc;
  }
  const size_t done = n4 * 4;
  if (done < n) {
    const size_t rest = n - done;
    size_t blocks = (rest + 255) / 256;
    const size_t cap = static_cast<size_t>(sms) * 8;
    if (blocks > cap) blocks = cap;
    add_f32_scalar_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(d_out + done, d_a + done,
                                                                         d_b + done, rest);
    if ((rc = launch_check("add_f32_scalar_kernel launch"))) return rc;
  }
  return THORK_OK;
}

// ---------------------------------------------------------------------------
// tcgen05 GEMMs
// ---------------------------------------------------------------------------
// Launch with programmatic stream serialisation (the kernel executes
// griddepcontrol.wait before touching global memory), an optional cluster
// of `cluster_x` CTAs, and optionally as a cooperative grid (all CTAs
// co-resident, for kernels whose CTAs wait on one another).
template <class... KArgs, class... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t s,
                      int cluster_x, bool cooperative, const char *name, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[3];
  int n = 0;
  if (cooperative) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return thork_cuda_error(e, name);
  return launch_check(name);
}

namespace {
using namespace thork::gemm;

// bf16 / e4m3 GEMM: A row-major [M,K] (K-major), B row-major [K,N] (MN-major)
using CfgBf16 = Config<KIND_BF16, 256, 4, false, true, false>;
using CfgE4m3 = Config<KIND_E4M3, 256, 4, false, true, false>;
// 2-CTA (cluster pair) variants: 256 x 256 tiles, 32 KiB stages per CTA
using Cfg2Bf16 = Config2<KIND_BF16, 256, 6>;
using Cfg2E4m3 = Config2<KIND_E4M3, 256, 6>;
// skinny (swap-AB): A = W row-major [K,N] (MN-major), B = X row-major [M,K]
// (K-major), output written transposed into Y[M,N].
// stream-K decode (M <= 32): 6 stages keep W streaming at the HBM rate and
// leave room for the next launch's CTAs to start their prologue on the same
// SM (measured: 3-10 stages within 2 %, M=32 11 % faster than with 10)
using CfgSkinny16 = Config<KIND_BF16, 16, 6, true, false, true>;
using CfgSkinny32 = Config<KIND_BF16, 32, 6, true, false, true>;
using CfgSkinny64 = Config<KIND_BF16, 64, 8, true, false, true>;
using CfgSkinny128 = Config<KIND_BF16, 128, 6, true, false, true>;
using CfgSkinny256 = Config<KIND_BF16, 256, 4, true, false, true>;

enum KernelId {
  K_GEMM_BF16 = 0, K_GEMM_E4M3, K_SKINNY64, K_SKINNY128, K_SKINNY256,
  K_GEMM2_BF16, K_GEMM2_E4M3, K_SKSK16, K_SKSK32, K_GEMM_BF16_SK, K_GEMM_E4M3_SK,
  K_AG_BF16, K_AGP_BF16, K_AG_E4M3, K_AGP_E4M3,  // fused all-gather: staged, push warps
  K_AGM_BF16, K_AGM_E4M3,                        // fused all-gather through a multicast view
  K_SKSK64,                                      // stream-K decode, M 33..64, few tiles
  K_SKINNY16, K_SKINNY32                         // one CTA per tile, M <= 32
};

template <class Cfg, int AG = AG_NONE>
int run_gemm(int kernel_id, const TensorMap &ta, const TensorMap &tb, const Params &prm,
             cudaStream_t s, const char *name) {
  int rc, sms;
  auto kern = gemm_kernel<Cfg, AG>;
  constexpr int smem = gemm_smem_bytes<Cfg, AG>();
  static_assert(smem <= 232448, "shared memory budget exceeded");
  if ((rc = ensure_smem(reinterpret_cast<const void *>(kern), kernel_id, smem))) return rc;
  if ((rc = thork_sm_count(&sms))) return rc;
  const int ntiles = ((prm.GM + Cfg::BM - 1) / Cfg::BM) * ((prm.GN + Cfg::BN - 1) / Cfg::BN);
  const int grid = ntiles < sms ? ntiles : sms;
  // push warps wait on tiles of other CTAs: launch the grid co-resident
  return launch_pdl(kern, dim3(grid), gemm_threads<Cfg, AG>(), smem, s, 1, AG == AG_PUSH, name, ta,
                    tb, prm);
}

// Cluster-pair launch: grid = 2 x (pairs), cluster (2,1,1).
template <class Cfg>
int run_gemm2(int kernel_id, const TensorMap &ta, const TensorMap &tb, const Params &prm,
              cudaStream_t s, const char *name) {
  int rc, sms;
  auto kern = gemm2_kernel<Cfg>;
  if ((rc = ensure_smem(reinterpret_cast<const void *>(kern), kernel_id, Cfg::SMEM_BYTES))) return rc;
  if ((rc = thork_sm_count(&sms))) return rc;
  const int ntiles = ((prm.GM + 2 * Cfg::BM - 1) / (2 * Cfg::BM)) * ((prm.GN + Cfg::BN - 1) / Cfg::BN);
  const int pairs = ntiles < sms / 2 ? ntiles : sms / 2;
  return launch_pdl(kern, dim3(2 * pairs), Cfg::THREADS, Cfg::SMEM_BYTES, s, 2, false, name, ta, tb,
                    prm);
}

template <class Cfg>
int run_gemm_sk(int kernel_id, const TensorMap &ta, const TensorMap &tb, const Params &prm,
                cudaStream_t s);
bool prefer_stream_k(long long tiles, int sms);

int check_dims(int M, int N, int K, int align, const char *what) {
  if (M <= 0 || N <= 0 || K <= 0)
    return thork_set_error(THORK_ERR_INVALID, "%s: dimensions must be positive (M=%d N=%d K=%d)",
                           what, M, N, K);
  if (K % align || N % align)
    return thork_set_error(THORK_ERR_INVALID,
                           "%s: K and N must be multiples of %d for 16-byte TMA row strides "
                           "(M=%d N=%d K=%d)",
                           what, align, M, N, K);
  return THORK_OK;
}

int check_ptrs(const void *a, const void *b, const void *c, const char *what) {
  if (!a || !b || !c) return thork_set_error(THORK_ERR_INVALID, "%s: NULL pointer", what);
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(c)) & 15u)
    return thork_set_error(THORK_ERR_INVALID, "%s: pointers must be 16-byte aligned", what);
  return THORK_OK;
}
}  // namespace

extern "C" int thork_gemm_bf16(const void *d_a, const void *d_b, void *d_c, int M, int N, int K,
                               int variant, void *stream) {
  int rc;
  if ((rc = check_dims(M, N, K, 8, "gemm_bf16"))) return rc;
  if ((rc = check_ptrs(d_a, d_b, d_c, "gemm_bf16"))) return rc;
  if (variant < 0 || variant > 3)
    return thork_set_error(THORK_ERR_INVALID, "gemm_bf16: unknown variant %d", variant);
  alignas(64) TensorMap ta, tb;
  using C = CfgBf16;
  // both variants read A in 128 x BK boxes and B in BK x 64 boxes
  if ((rc = thork_encode_tmap_2d(&ta, THORK_DT_BF16, d_a, M, K, (uint64_t)K * 2, C::BM, C::BK, 128)))
    return rc;
  if ((rc = thork_encode_tmap_2d(&tb, THORK_DT_BF16, d_b, K, N, (uint64_t)N * 2, C::BK, C::CHUNK, 128)))
    return rc;
  unsigned *status;
  if ((rc = thork_status_word(&status))) return rc;
  Params prm{d_c, M, N, K, N, M, N, 1.0f, status};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // automatic choice: stream-K when the 128 x 256 tiles would fill at most
  // half of the SMs; otherwise the 2-CTA kernel once a pair tile has work
  // for both CTAs (measured 8192^3: 1447 against 1414 TFLOP/s in bursts,
  // 1264-1269 against 1242-1249 over 2.5 s under the power cap; 4096^3:
  // 1360 against 1280)
  if (variant == 0) {
    int sms;
    if ((rc = thork_sm_count(&sms))) return rc;
    const long long tiles = static_cast<long long>((M + C::BM - 1) / C::BM) * ((N + C::BN - 1) / C::BN);
    variant = prefer_stream_k(tiles, sms) ? 3 : (M > 128 ? 2 : 1);
  }
  if (variant == 2) return run_gemm2<Cfg2Bf16>(K_GEMM2_BF16, ta, tb, prm, s, "gemm2_bf16 launch");
  if (variant == 3) return run_gemm_sk<C>(K_GEMM_BF16_SK, ta, tb, prm, s);
  return run_gemm<C>(K_GEMM_BF16, ta, tb, prm, s, "gemm_bf16 launch");
}

extern "C" int thork_gemm_e4m3(const void *d_a, const void *d_b, void *d_c, int M, int N, int K,
                               float scale_a, float scale_b, int variant, void *stream) {
  int rc;
  if ((rc = check_dims(M, N, K, 16, "gemm_e4m3"))) return rc;
  if ((rc = check_ptrs(d_a, d_b, d_c, "gemm_e4m3"))) return rc;
  if (variant < 0 || variant > 3)
    return thork_set_error(THORK_ERR_INVALID, "gemm_e4m3: unknown variant %d", variant);
  alignas(64) TensorMap ta, tb;
  using C = CfgE4m3;
  if ((rc = thork_encode_tmap_2d(&ta, THORK_DT_E4M3, d_a, M, K, (uint64_t)K, C::BM, C::BK, 128)))
    return rc;
  if ((rc = thork_encode_tmap_2d(&tb, THORK_DT_E4M3, d_b, K, N, (uint64_t)N, C::BK, C::CHUNK, 128)))
    return rc;
  unsigned *status;
  if ((rc = thork_status_word(&status))) return rc;
  Params prm{d_c, M, N, K, N, M, N, scale_a * scale_b, status};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // automatic choice: the 2-CTA kernel sustains ~1.6% more on e4m3 once a
  // pair tile has work for both CTAs
  if (variant == 0) variant = (M > 128) ? 2 : 1;
  if (variant == 2) return run_gemm2<Cfg2E4m3>(K_GEMM2_E4M3, ta, tb, prm, s, "gemm2_e4m3 launch");
  if (variant == 3) return run_gemm_sk<C>(K_GEMM_E4M3_SK, ta, tb, prm, s);
  return run_gemm<C>(K_GEMM_E4M3, ta, tb, prm, s, "gemm_e4m3 launch");
}

// ---------------------------------------------------------------------------
// Fused GEMM + all-gather over NVLink peer memory
// ---------------------------------------------------------------------------
namespace {
// Shared body of the fused GEMM + all-gather entry points: this rank's rows
// [row0, row0 + rows) of C go to d_c and to every peer buffer at the same
// offset.  Variant 1 stores to the peers from the epilogue (through a
// shared-memory staging tile); variant 2 leaves that to four push warps per
// CTA that share all (tile, peer) pushes of the grid; 0 chooses.
template <class Cfg>
int gemm_allgather(int kid_staged, int kid_push, int dt, int elem, const void *d_a_rows, const void *d_b, void *d_c,
                   void *const *d_peer_c, int n_peers, int rows, int N, int K, int row0,
                   unsigned *d_tile_flags, unsigned epoch, float alpha, int variant, void *stream,
                   const char *what) {
  int rc;
  if ((rc = check_dims(rows, N, K, 16 / elem, what))) return rc;
  if ((rc = check_ptrs(d_a_rows, d_b, d_c, what))) return rc;
  if (variant < 0 || variant > 2)
    return thork_set_error(THORK_ERR_INVALID, "%s: unknown variant %d", what, variant);
  if (n_peers < 0 || n_peers > 7 || (n_peers > 0 && !d_peer_c))
    return thork_set_error(THORK_ERR_INVALID, "%s: n_peers=%d must be 0..7", what, n_peers);
  if (row0 < 0) return thork_set_error(THORK_ERR_INVALID, "%s: row0 < 0", what);
  for (int g = 0; g < n_peers; ++g)
    if (!d_peer_c[g] || (reinterpret_cast<uintptr_t>(d_peer_c[g]) & 15u))
      return thork_set_error(THORK_ERR_INVALID,
                             "%s: peer buffer %d is NULL or not 16-byte aligned", what, g);
  if (variant == 0) variant = n_peers >= 3 ? 2 : 1;
  if (variant == 2 && (!d_tile_flags || (reinterpret_cast<uintptr_t>(d_tile_flags) & 3u)))
    return thork_set_error(THORK_ERR_INVALID, "%s: variant 2 needs 4-byte aligned tile flags",
                           what);
  alignas(64) TensorMap ta, tb;
  if ((rc = thork_encode_tmap_2d(&ta, dt, d_a_rows, rows, K, (uint64_t)K * elem, Cfg::BM, Cfg::BK,
                                 128)))
    return rc;
  if ((rc = thork_encode_tmap_2d(&tb, dt, d_b, K, N, (uint64_t)N * elem, Cfg::BK, Cfg::CHUNK, 128)))
    return rc;
  unsigned *status;
  if ((rc = thork_status_word(&status))) return rc;
  const size_t off = static_cast<size_t>(row0) * N * 2;  // bytes to this rank's bf16 rows
  Params prm{static_cast<char *>(d_c) + off, rows, N, K, N, rows, N, alpha, status};
  for (int g = 0; g < n_peers; ++g) prm.peer[g] = static_cast<char *>(d_peer_c[g]) + off;
  prm.npeer = n_peers;
  prm.tile_flags = d_tile_flags;
  prm.epoch = epoch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (variant == 2) return run_gemm<Cfg, AG_PUSH>(kid_push, ta, tb, prm, s, what);
  return run_gemm<Cfg, AG_STAGED>(kid_staged, ta, tb, prm, s, what);
}
}  // namespace

extern "C" int thork_gemm_bf16_allgather(const void *d_a_rows, const void *d_b, void *d_c,
                                        void *const *d_peer_c, int n_peers, int rows, int N, int K,
                                        int row0, unsigned *d_tile_flags, unsigned epoch,
                                        int variant, void *stream) {
  return gemm_allgather<CfgBf16>(
      K_AG_BF16, K_AGP_BF16, THORK_DT_BF16, 2, d_a_rows, d_b, d_c, d_peer_c, n_peers, rows, N, K, row0,
      d_tile_flags, epoch, 1.0f, variant, stream, "gemm_bf16_allgather");
}

extern "C" int thork_gemm_e4m3_allgather(const void *d_a_rows, const void *d_b, void *d_c,
                                        void *const *d_peer_c, int n_peers, int rows, int N, int K,
                                        int row0, unsigned *d_tile_flags, unsigned epoch,
                                        float scale_a, float scale_b, int variant, void *stream) {
  return gemm_allgather<CfgE4m3>(
      K_AG_E4M3, K_AGP_E4M3, THORK_DT_E4M3, 1, d_a_rows, d_b, d_c, d_peer_c, n_peers, rows, N, K, row0,
      d_tile_flags, epoch, scale_a * scale_b, variant, stream, "gemm_e4m3_allgather");
}

namespace {
// Fused GEMM + all-gather through a multicast view: this rank's rows are
// stored once, with multimem.st, at their offset of the gathered C.
template <class Cfg>
int gemm_allgather_mc(int kid, int dt, int elem, const void *d_a_rows, const void *d_b, void *d_c_mc,
                      int rows, int N, int K, int row0, float alpha, void *stream, const char *what) {
  int rc;
  if ((rc = check_dims(rows, N, K, 16 / elem, what))) return rc;
  if ((rc = check_ptrs(d_a_rows, d_b, d_c_mc, what))) return rc;
  if (row0 < 0) return thork_set_error(THORK_ERR_INVALID, "%s: row0 < 0", what);
  if (reinterpret_cast<uintptr_t>(d_c_mc) & 15u)
    return thork_set_error(THORK_ERR_INVALID, "%s: multicast view not 16-byte aligned", what);
  alignas(64) TensorMap ta, tb;
  if ((rc = thork_encode_tmap_2d(&ta, dt, d_a_rows, rows, K, (uint64_t)K * elem, Cfg::BM, Cfg::BK,
                                 128)))
    return rc;
  if ((rc = thork_encode_tmap_2d(&tb, dt, d_b, K, N, (uint64_t)N * elem, Cfg::BK, Cfg::CHUNK, 128)))
    return rc;
  unsigned *status;
  if ((rc = thork_status_word(&status))) return rc;
  const size_t off = static_cast<size_t>(row0) * N * 2;
  Params prm{static_cast<char *>(d_c_mc) + off, rows, N, K, N, rows, N, alpha, status};
  return run_gemm<Cfg, AG_MULTIMEM>(kid, ta, tb, prm, static_cast<cudaStream_t>(stream), what);
}
}  // namespace

extern "C" int thork_gemm_bf16_allgather_mc(const void *d_a_rows, const void *d_b, void *d_c_mc,
                                           int rows, int N, int K, int row0, void *stream) {
  return gemm_allgather_mc<CfgBf16>(K_AGM_BF16, THORK_DT_BF16, 2, d_a_rows, d_b, d_c_mc, rows, N, K,
                                    row0, 1.0f, stream, "gemm_bf16_allgather_mc");
}

extern "C" int thork_gemm_e4m3_allgather_mc(const void *d_a_rows, const void *d_b, void *d_c_mc,
                                           int rows, int N, int K, int row0, float scale_a,
                                           float scale_b, void *stream) {
  return gemm_allgather_mc<CfgE4m3>(K_AGM_E4M3, THORK_DT_E4M3, 1, d_a_rows, d_b, d_c_mc, rows, N, K,
                                    row0, scale_a * scale_b, stream, "gemm_e4m3_allgather_mc");
}

namespace {
// Flag barrier between the ranks of a fused all-gather.  Rank r stores
// `epoch` into flags[r] of every peer (release at system scope, after a
// system fence that orders this GPU's earlier peer stores), then waits, at
// most THORK_WAIT_TIMEOUT_NS, until its own flags[q] reach `epoch` for every
// peer q (acquire).  Flags compare by wrapping difference.
struct PeerFlagPtrs {
  unsigned *p[8];
};

// Launched with programmatic stream serialisation: the block is resident
// while the GEMM before it runs and starts signalling the moment that grid
// completes, and the next launch may begin its prologue meanwhile.
__global__ void peer_barrier_kernel(const PeerFlagPtrs peers, unsigned *flags, int world, int rank,
                                    unsigned epoch, unsigned *status) {
  thork::dev::pdl_launch_dependents();
  thork::dev::pdl_wait();  // the previous grid's stores are complete and visible from here on
  const int t = threadIdx.x;
  if (t < world && t != rank) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.p[t] + rank), "r"(epoch)
                 : "memory");
    const uint64_t t0 = thork::dev::globaltimer();
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + t) : "memory");
      if (static_cast<int>(v - epoch) >= 0) break;
      if (thork::dev::globaltimer() - t0 > THORK_WAIT_TIMEOUT_NS) {
        thork::dev::report_status(status, thork::dev::STATUS_WAIT_TIMEOUT, 20);
        break;
      }
      __nanosleep(64);
    }
  }
  // what the peers stored through a multicast view is read through this
  // GPU's ordinary view after the barrier
  thork::dev::fence_proxy_alias();
  __syncthreads();
}
}  // namespace

extern "C" int thork_peer_barrier(void *d_flags, void *const *d_peer_flags, int world, int rank,
                                  unsigned epoch, void *stream) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return thork_set_error(THORK_ERR_INVALID, "peer_barrier: rank %d / world %d (at most 8)", rank,
                           world);
  if (!d_flags || (world > 1 && !d_peer_flags))
    return thork_set_error(THORK_ERR_INVALID, "peer_barrier: NULL flags");
  PeerFlagPtrs peers = {};
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    if (!d_peer_flags[q] || (reinterpret_cast<uintptr_t>(d_peer_flags[q]) & 3u))
      return thork_set_error(THORK_ERR_INVALID, "peer_barrier: flags of rank %d NULL or unaligned",
                             q);
    peers.p[q] = static_cast<unsigned *>(d_peer_flags[q]);
  }
  if (world == 1) return THORK_OK;
  unsigned *status;
  int rc;
  if ((rc = thork_status_word(&status))) return rc;
  return launch_pdl(peer_barrier_kernel, dim3(1), 32, 0, static_cast<cudaStream_t>(stream), 1, false,
                    "peer_barrier launch", peers, static_cast<unsigned *>(d_flags), world, rank,
                    epoch, status);
}

namespace {
// ---- stream-K GEMM ----------------------------------------------------------
struct SkPlan {
  int grid, base, extra, tiles, dp_tiles;
  size_t partial_bytes, counter_bytes;
};

// Work split for a GEMM in MMA space GM x GN x GK.  With `data_parallel`,
// the whole waves of tiles go one tile per CTA (in raster order, so the
// tiles in flight share operand panels in L2) and only the tiles of the
// last, partial wave are split into equal contiguous ranges of (tile,
// k-block) units; otherwise every tile is.  Each CTA owns two partial slots.
template <class Cfg>
SkPlan sk_plan(int GM, int GN, int GK, int sms, bool data_parallel = false) {
  SkPlan pl;
  pl.tiles = ((GM + Cfg::BM - 1) / Cfg::BM) * ((GN + Cfg::BN - 1) / Cfg::BN);
  const int nkb = (GK + Cfg::BK - 1) / Cfg::BK;
  pl.dp_tiles = data_parallel && pl.tiles > sms ? (pl.tiles - 1) / sms * sms : 0;
  const long long units = static_cast<long long>(pl.tiles - pl.dp_tiles) * nkb;
  pl.grid = pl.dp_tiles ? sms : static_cast<int>(units < sms ? units : sms);
  pl.base = static_cast<int>(units / pl.grid);
  pl.extra = static_cast<int>(units % pl.grid);
  pl.partial_bytes = static_cast<size_t>(pl.grid) * 2 * Cfg::BM * Cfg::BN * sizeof(float);
  pl.counter_bytes = static_cast<size_t>(pl.tiles) * sizeof(unsigned);
  return pl;
}

// Stream-K splits the k-loop of the tiles over all SMs at the cost of a
// partial write and a fixup per split tile.  Measured on B200, that only
// pays when whole tiles would leave most SMs idle (4096^3, 3.46 waves:
// stream-K 5 % slower than whole tiles); it is chosen automatically when
// the tiles fill at most half of the SMs.
bool prefer_stream_k(long long tiles, int sms) { return tiles * 2 <= sms; }

// Per-device workspaces of the stream-K path: the partial slots, and the
// per-tile arrival counters in a buffer of their own (zeroed when allocated
// or grown; every launch returns the counters it uses to zero), so the
// counters never land on memory an earlier plan used for partials.
std::mutex g_ws_mu;
void *g_part[kMaxDevices] = {};
size_t g_part_bytes[kMaxDevices] = {};
void *g_cnt[kMaxDevices] = {};
size_t g_cnt_bytes[kMaxDevices] = {};

int grow(void **buf, size_t *have, size_t need, bool zero, const char *what) {
  if (*have >= need) return THORK_OK;
  if (*buf) cudaFree(*buf);
  *buf = nullptr;
  *have = 0;
  cudaError_t e = cudaMalloc(buf, need);
  if (e != cudaSuccess) return thork_cuda_error(e, what);
  if (zero) {
    e = cudaMemset(*buf, 0, need);
    if (e != cudaSuccess) return thork_cuda_error(e, what);
  }
  *have = need;
  return THORK_OK;
}

int sk_workspace(size_t partial_bytes, size_t counter_bytes, void **partial, void **counters) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  if ((rc = grow(&g_part[dev], &g_part_bytes[dev], partial_bytes, false, "cudaMalloc(stream-K partials)")))
    return rc;
  if ((rc = grow(&g_cnt[dev], &g_cnt_bytes[dev], counter_bytes, true, "cudaMalloc(stream-K counters)")))
    return rc;
  *partial = g_part[dev];
  *counters = g_cnt[dev];
  return THORK_OK;
}

template <class Cfg>
int launch_sk(int kernel_id, const TensorMap &ta, const TensorMap &tb, const Params &prm,
              const SkPlan &pl, void *partial, void *counters, cudaStream_t s,
              bool w_static = false) {
  int rc;
  auto kern = sk_kernel<Cfg>;
  if ((rc = ensure_smem(reinterpret_cast<const void *>(kern), kernel_id, Cfg::SMEM_BYTES))) return rc;
  SkParams sp;
  sp.p = prm;
  sp.partial = static_cast<float *>(partial);
  sp.counters = static_cast<unsigned *>(counters);
  sp.base = pl.base;
  sp.extra = pl.extra;
  sp.dp_tiles = pl.dp_tiles;
  sp.w_static = w_static ? 1 : 0;
  return launch_pdl(kern, dim3(pl.grid), Cfg::THREADS, Cfg::SMEM_BYTES, s, 1, false, "sk_kernel launch",
                    ta, tb, sp);
}

// Stream-K form of the 128 x 256-tile GEMM (A K-major, B MN-major).
template <class Cfg>
int run_gemm_sk(int kernel_id, const TensorMap &ta, const TensorMap &tb, const Params &prm,
                cudaStream_t s) {
  int rc, sms;
  if ((rc = thork_sm_count(&sms))) return rc;
  const SkPlan pl = sk_plan<Cfg>(prm.GM, prm.GN, prm.GK, sms, true);
  void *part, *cnt;
  if ((rc = sk_workspace(pl.partial_bytes, pl.counter_bytes, &part, &cnt))) return rc;
  return launch_sk<Cfg>(kernel_id, ta, tb, prm, pl, part, cnt, s);
}

template <class Cfg>
int encode_skinny_maps(TensorMap &ta, TensorMap &tb, const void *d_x, const void *d_w, int M, int N,
                       int K) {
  int rc;
  // A operand = W [K, N] (MN-major), B operand = X [M, K] (K-major, rows >= M read as zero)
  if ((rc = thork_encode_tmap_2d(&ta, THORK_DT_BF16, d_w, K, N, (uint64_t)N * 2, Cfg::BK, Cfg::CHUNK, 128)))
    return rc;
  return thork_encode_tmap_2d(&tb, THORK_DT_BF16, d_x, M, K, (uint64_t)K * 2, Cfg::BN, Cfg::BK, 128);
}

template <class Cfg>
int run_skinny_sk(int kernel_id, const void *d_x, const void *d_w, void *d_y, int M, int N, int K,
                  cudaStream_t s, bool w_static) {
  int rc, sms;
  alignas(64) TensorMap ta, tb;
  if ((rc = encode_skinny_maps<Cfg>(ta, tb, d_x, d_w, M, N, K))) return rc;
  if ((rc = thork_sm_count(&sms))) return rc;
  const SkPlan pl = sk_plan<Cfg>(N, M, K, sms);
  void *part, *cnt;
  if ((rc = sk_workspace(pl.partial_bytes, pl.counter_bytes, &part, &cnt))) return rc;
  unsigned *status;
  if ((rc = thork_status_word(&status))) return rc;
  Params prm{d_y, N, M, K, N, M, N, 1.0f, status};
  return launch_sk<Cfg>(kernel_id, ta, tb, prm, pl, part, cnt, s, w_static);
}

template <class Cfg>
int run_skinny(int kernel_id, const void *d_x, const void *d_w, void *d_y, int M, int N, int K,
               cudaStream_t s) {
  int rc;
  alignas(64) TensorMap ta, tb;
  // A operand = W [K, N] (MN-major), B operand = X [M, K] (K-major, rows >= M read as zero)
  if ((rc = thork_encode_tmap_2d(&ta, THORK_DT_BF16, d_w, K, N, (uint64_t)N * 2, Cfg::BK, Cfg::CHUNK, 128)))
    return rc;
  if ((rc = thork_encode_tmap_2d(&tb, THORK_DT_BF16, d_x, M, K, (uint64_t)K * 2, Cfg::BN, Cfg::BK, 128)))
    return rc;
  unsigned *status;
  if ((rc = thork_status_word(&status))) return rc;
  // MMA space: GM = N (W columns), GN = M (X rows); output Y [M, N] written transposed.
  Params prm{d_y, N, M, K, N, M, N, 1.0f, status};
  return run_gemm<Cfg>(kernel_id, ta, tb, prm, s, "skinny_gemm_bf16 launch");
}
}  // namespace

extern "C" int thork_skinny_gemm_bf16_ex(const void *d_x, const void *d_w, void *d_y, int M, int N,
                                         int K, int flags, void *stream) {
  int rc;
  if ((rc = check_dims(M, N, K, 8, "skinny_gemm_bf16"))) return rc;
  if ((rc = check_ptrs(d_x, d_w, d_y, "skinny_gemm_bf16"))) return rc;
  if (flags & ~THORK_SKINNY_W_STATIC)
    return thork_set_error(THORK_ERR_INVALID, "skinny_gemm_bf16: unknown flags 0x%x", flags);
  const bool w_static = (flags & THORK_SKINNY_W_STATIC) != 0;
  if (M > 256)
    return thork_set_error(THORK_ERR_INVALID, "skinny_gemm_bf16: M must be <= 256 (M=%d)", M);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // One CTA per 128-column tile of W, except that M <= 64 takes stream-K
  // when the tiles fill at most half of the SMs (W split over GPUs).
  // Measured K=4096 (static weights): N=14336 one CTA per tile 23.2-23.6 /
  // 23.5 / 22.8 us at M=1 / 16 / 32 against 23.9 / 24.1 / 24.9 stream-K;
  // M=64 at N=3584 / 1792 stream-K 17.6 / 19.9 against 20.8 / 20.7; M=128
  // at N=7168 / 3584 one CTA per tile 22.4 / 21.6 against 24.9 / 24.3.
  int sms;
  if ((rc = thork_sm_count(&sms))) return rc;
  const bool few_tiles = prefer_stream_k((N + CfgSkinny16::BM - 1) / CfgSkinny16::BM, sms);
  if (M <= 16) {
    if (few_tiles) return run_skinny_sk<CfgSkinny16>(K_SKSK16, d_x, d_w, d_y, M, N, K, s, w_static);
    return run_skinny<CfgSkinny16>(K_SKINNY16, d_x, d_w, d_y, M, N, K, s);
  }
  if (M <= 32) {
    if (few_tiles) return run_skinny_sk<CfgSkinny32>(K_SKSK32, d_x, d_w, d_y, M, N, K, s, w_static);
    return run_skinny<CfgSkinny32>(K_SKINNY32, d_x, d_w, d_y, M, N, K, s);
  }
  if (M <= 64) {
    if (few_tiles) return run_skinny_sk<CfgSkinny64>(K_SKSK64, d_x, d_w, d_y, M, N, K, s, w_static);
    return run_skinny<CfgSkinny64>(K_SKINNY64, d_x, d_w, d_y, M, N, K, s);
  }
  if (M <= 128) return run_skinny<CfgSkinny128>(K_SKINNY128, d_x, d_w, d_y, M, N, K, s);
  return run_skinny<CfgSkinny256>(K_SKINNY256, d_x, d_w, d_y, M, N, K, s);
}

extern "C" int thork_skinny_gemm_bf16(const void *d_x, const void *d_w, void *d_y, int M, int N,
                                      int K, void *stream) {
  return thork_skinny_gemm_bf16_ex(d_x, d_w, d_y, M, N, K, 0, stream);
}

// ---------------------------------------------------------------------------
// allocation-free decode GEMM (thork_skinny_gemm_bf16_noalloc)
// ---------------------------------------------------------------------------
// Scratch layout: [status word, 256 B][tile counters, 64 KiB][partial slots].
// The array is zero when the library's module loads.  Each call clears the
// counters it will use before launching; the status word is sticky: kernels
// only OR a code into it, and only thork_skinny_gemm_bf16_noalloc_status
// (clear != 0) resets it, so an expired wait stays visible until read.
namespace {
constexpr size_t kNoAllocBytes = 8u << 20;
constexpr size_t kNoAllocStatusBytes = 256;
constexpr size_t kNoAllocCounterBytes = 64u << 10;
constexpr size_t kNoAllocPartialBytes = kNoAllocBytes - kNoAllocStatusBytes - kNoAllocCounterBytes;
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_na_mu;
unsigned char *g_na_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once
// per device; the host-side name is only a stand-in for it).
int noalloc_scratch(unsigned char **addr) {
  int dev, rc;
  if ((rc = current_device(&dev))) return rc;
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (!g_na_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_na_addr[dev] = static_cast<unsigned char *>(p);
  }
  *addr = g_na_addr[dev];
  return THORK_OK;
}

template <class Cfg>
int run_skinny_noalloc(int kernel_id, const void *d_x, const void *d_w, void *d_y, int M, int N, int K,
                       cudaStream_t s) {
  int rc, sms;
  if ((rc = thork_sm_count(&sms))) return rc;
  const SkPlan pl = sk_plan<Cfg>(N, M, K, sms);
  if (pl.partial_bytes > kNoAllocPartialBytes)
    return thork_set_error(THORK_ERR_INVALID,
                           "skinny_gemm_bf16_noalloc: M=%d N=%d K=%d needs %zu bytes of split-tile "
                           "partials; the scratch array holds %zu",
                           M, N, K, pl.partial_bytes, kNoAllocPartialBytes);
  unsigned char *base;
  if ((rc = noalloc_scratch(&base))) return rc;
  unsigned char *counters = base + kNoAllocStatusBytes;
  unsigned char *partial = counters + kNoAllocCounterBytes;
  // this plan's tile counters must start at zero (the status word is left
  // as it is: it keeps any earlier call's expired-wait code until read)
  cudaError_t e = cudaMemsetAsync(counters, 0, pl.counter_bytes, s);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaMemsetAsync(no-alloc scratch)");
  alignas(64) TensorMap ta, tb;
  if ((rc = encode_skinny_maps<Cfg>(ta, tb, d_x, d_w, M, N, K))) return rc;
  Params prm{d_y, N, M, K, N, M, N, 1.0f, reinterpret_cast<unsigned *>(base)};
  return launch_sk<Cfg>(kernel_id, ta, tb, prm, pl, partial, counters, s);
}
}  // namespace

extern "C" int thork_skinny_gemm_bf16_noalloc(const void *d_x, const void *d_w, void *d_y, int M,
                                              int N, int K, void *stream) {
  int rc;
  if ((rc = check_dims(M, N, K, 8, "skinny_gemm_bf16_noalloc"))) return rc;
  if (M > 32)
    return thork_set_error(THORK_ERR_INVALID,
                           "skinny_gemm_bf16_noalloc: M must be <= 32 (M=%d); use "
                           "thork_skinny_gemm_bf16 for larger M",
                           M);
  if (static_cast<size_t>((N + 127) / 128) * sizeof(unsigned) > kNoAllocCounterBytes)
    return thork_set_error(THORK_ERR_INVALID,
                           "skinny_gemm_bf16_noalloc: N=%d gives %d output tiles; at most %zu fit the "
                           "scratch array",
                           N, (N + 127) / 128, kNoAllocCounterBytes / sizeof(unsigned));
  if ((rc = check_ptrs(d_x, d_w, d_y, "skinny_gemm_bf16_noalloc"))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M <= 16) return run_skinny_noalloc<CfgSkinny16>(K_SKSK16, d_x, d_w, d_y, M, N, K, s);
  return run_skinny_noalloc<CfgSkinny32>(K_SKSK32, d_x, d_w, d_y, M, N, K, s);
}

extern "C" int thork_skinny_gemm_bf16_noalloc_status(unsigned *status, int clear, void *stream) {
  if (!status) return thork_set_error(THORK_ERR_INVALID, "noalloc_status: status is NULL");
  unsigned char *base;
  int rc;
  if ((rc = noalloc_scratch(&base))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // a 4-byte copy into the caller's host word and an optional 4-byte clear:
  // neither allocates device or pinned memory
  cudaError_t e = cudaMemcpyAsync(status, base, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return thork_cuda_error(e, "read no-alloc status word");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaStreamSynchronize(no-alloc status)");
  if (clear) {
    e = cudaMemsetAsync(base, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return thork_cuda_error(e, "clear no-alloc status word");
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaStreamSynchronize(no-alloc status)");
  }
  return THORK_OK;
}
