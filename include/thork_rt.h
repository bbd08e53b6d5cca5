/*
 * thork_rt.h — C-ABI of libthork_rt.so, the B200 (sm_100a) runtime and kernel
 * library behind the thork_b200 Python package.
 *
 * The reference (save-buffer/thork, a Python tracing DSL) reaches the GPU
 * through two foreign interfaces, and this library replaces both:
 *
 *   1. cuda-python driver/NVRTC bindings called from src/thork/runtime.py
 *      (cuInit/cuCtxCreate, cuMemAlloc, cuMemcpyHtoD/DtoH, nvrtcCompileProgram,
 *      cuModuleLoadData, cuModuleGetFunction, cuLaunchKernel, cuCtxSynchronize,
 *      cuMemFree).  Each entry point below names the runtime.py lines it
 *      stands in for.
 *   2. the per-kernel host launcher `extern "C" void thork_launch_<name>(grid,
 *      block, smem, stream, args...)` that src/thork/codegen.py:416-469 emits
 *      for ThunderKittens kernels and src/thork/runtime.py:534-622 calls through
 *      ctypes.  Traced kernels here launch through thork_launch(); the
 *      library kernels (tk.kernels.matrix_add / matmul) have fixed entry
 *      points (thork_matrix_add_f32, thork_gemm_*, thork_skinny_gemm_bf16).
 *
 * Conventions: every function returns an int status (THORK_OK == 0).  On any
 * other status thork_last_error() returns a thread-local message.  Pointers
 * named d_* are device pointers, h_* host pointers; `stream` is a cudaStream_t
 * (NULL = the legacy default stream).  No function takes or returns a torch
 * or Python type.
 */
#ifndef THORK_RT_H
#define THORK_RT_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define THORK_API __attribute__((visibility("default")))
#else
#define THORK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
enum {
  THORK_OK = 0,
  THORK_ERR_CUDA = 1,        /* a CUDA runtime/driver call failed            */
  THORK_ERR_NVRTC = 2,       /* NVRTC failed (compile log in the out param)  */
  THORK_ERR_NCCL = 3,        /* an NCCL call failed                          */
  THORK_ERR_INVALID = 4,     /* bad argument (shape, alignment, null, ...)   */
  THORK_ERR_KERNEL = 5,      /* a kernel reported a bounded-wait timeout     */
  THORK_ERR_UNAVAILABLE = 6  /* a dependency (driver, NVRTC, NCCL) missing   */
};

/* Element types for thork_tensor_map_2d and the NCCL wrappers. */
enum {
  THORK_DT_U8 = 0,
  THORK_DT_U16 = 1,
  THORK_DT_U32 = 2,
  THORK_DT_F32 = 3,
  THORK_DT_BF16 = 4,
  THORK_DT_F16 = 5,
  THORK_DT_E4M3 = 6
};

/* Attributes for thork_device_attr. */
enum {
  THORK_ATTR_CC_MAJOR = 0,
  THORK_ATTR_CC_MINOR = 1,
  THORK_ATTR_SM_COUNT = 2,
  THORK_ATTR_SMEM_OPTIN = 3,      /* max dynamic smem per block (opt-in)   */
  THORK_ATTR_L2_BYTES = 4,
  THORK_ATTR_CLOCK_KHZ = 5,
  THORK_ATTR_MEM_CLOCK_KHZ = 6,
  THORK_ATTR_PCI_DOMAIN = 7,      /* PCI location: identifies the physical GPU */
  THORK_ATTR_PCI_BUS = 8,
  THORK_ATTR_PCI_DEVICE = 9
};

/* ---- library / errors ----------------------------------------------- */
/* Library ABI version (major*100 + minor).  No reference counterpart.     */
THORK_API int thork_version(void);
/* Copies the calling thread's last error message into buf (NUL-terminated).
 * Replaces the message text of runtime.py:_check (runtime.py:53-77).       */
THORK_API int thork_last_error(char *buf, size_t n);

/* ---- devices -------------------------------------------------------- */
/* Number of visible CUDA devices (0 when no driver is present).           */
THORK_API int thork_device_count(int *count);
/* Makes `dev` current on this thread and initialises its primary context.
 * Replaces runtime.get_device (runtime.py:85-105), which hard-codes device
 * 0 and calls cuInit/cuDeviceGet/cuCtxCreate.                              */
THORK_API int thork_init(int dev);
/* Queries one THORK_ATTR_* value.  Replaces the cuDeviceGetAttribute calls
 * of runtime.py:97-104 (compute capability) and runtime.py:172-186
 * (CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN).                 */
THORK_API int thork_device_attr(int dev, int attr, int *value);
/* Blocks until all work on the current device is done.  Replaces
 * cuCtxSynchronize (runtime.py:618, runtime.py:691).                       */
THORK_API int thork_device_synchronize(void);

/* ---- memory --------------------------------------------------------- */
/* Device allocation / free.  Replace cuMemAlloc (runtime.py:577, 657) and
 * cuMemFree (runtime.py:622, 700).                                         */
THORK_API int thork_malloc(size_t nbytes, void **d_ptr);
THORK_API int thork_free(void *d_ptr);
/* Page-locked host memory, used for the end-to-end copy path.  No
 * reference counterpart (the reference copies from pageable numpy memory). */
THORK_API int thork_host_alloc(size_t nbytes, void **h_ptr);
THORK_API int thork_host_free(void *h_ptr);
/* Copies.  stream == NULL and sync != 0 gives the blocking semantics of
 * cuMemcpyHtoD / cuMemcpyDtoH (runtime.py:578, 620, 659, 695); otherwise
 * the copy is queued on `stream`.                                          */
THORK_API int thork_memcpy_htod(void *d_dst, const void *h_src, size_t nbytes, void *stream, int sync);
THORK_API int thork_memcpy_dtoh(void *h_dst, const void *d_src, size_t nbytes, void *stream, int sync);
THORK_API int thork_memcpy_dtod(void *d_dst, const void *d_src, size_t nbytes, void *stream);
THORK_API int thork_memset(void *d_ptr, int value, size_t nbytes, void *stream);
/* Free and total device memory of the current device (cudaMemGetInfo).  No
 * reference counterpart; tests use it to show an entry point allocates
 * nothing.                                                                 */
THORK_API int thork_mem_info(size_t *free_bytes, size_t *total_bytes);

/* ---- streams and events (no reference counterpart: it uses stream 0) --- */
THORK_API int thork_stream_create(void **stream);
THORK_API int thork_stream_destroy(void *stream);
THORK_API int thork_stream_synchronize(void *stream);
THORK_API int thork_event_create(void **event);
THORK_API int thork_event_destroy(void *event);
THORK_API int thork_event_record(void *event, void *stream);
THORK_API int thork_event_synchronize(void *event);
THORK_API int thork_event_elapsed_ms(void *start, void *end, float *ms);
/* Make `stream` wait for `event` (cross-stream ordering for the pipelined
 * copy-in / compute / copy-out path).                                      */
THORK_API int thork_stream_wait_event(void *stream, void *event);

/* ---- NVRTC ---------------------------------------------------------- */
/* NVRTC version linked at run time (dlopen of libnvrtc.so.12).            */
THORK_API int thork_nvrtc_version(int *major, int *minor);
/* Compiles CUDA C++ `source` to a cubin for `arch` (e.g. "sm_100a").
 * `opts` are extra NVRTC options.  On success *cubin/*cubin_size hold a
 * buffer owned by the caller (release with thork_buffer_free).  The compile
 * log is always returned in *log (caller frees; may be NULL if empty).
 * Replaces runtime.compile_source (runtime.py:373-421), which produces PTX
 * for compute_<cap> and lets the driver JIT it.                           */
THORK_API int thork_nvrtc_compile(const char *source, const char *name, const char *arch,
                        const char **opts, int n_opts,
                        void **cubin, size_t *cubin_size, char **log);
THORK_API int thork_buffer_free(void *buf);

/* ---- modules and launches -------------------------------------------- */
/* Loads a cubin into the current context.  Replaces cuModuleLoadData
 * (runtime.py:420).                                                        */
THORK_API int thork_module_load(const void *image, void **module);
THORK_API int thork_module_unload(void *module);
/* Replaces runtime.get_function / cuModuleGetFunction (runtime.py:424-428). */
THORK_API int thork_module_get_function(void *module, const char *name, void **function);
/* Replaces set_max_dynamic_shared_size (runtime.py:189-200) and the
 * cudaFuncSetAttribute line of the generated launcher (codegen.py:459-462). */
THORK_API int thork_function_set_max_dynamic_smem(void *function, int nbytes);
/* Launches `function` with kernel-parameter pointers `args` (the
 * cuLaunchKernel convention).  cluster may be NULL or {1,1,1} for no
 * cluster.  Replaces cuLaunchKernel (runtime.py:682-690) and the
 * `<<<grid, block, smem, stream>>>` launch of codegen.py:463-467.          */
THORK_API int thork_launch(void *function, const unsigned grid[3], const unsigned block[3],
                 const unsigned cluster[3], unsigned smem_bytes, void *stream,
                 void **args);

/* ---- TMA ------------------------------------------------------------- */
/* Encodes a 2-D tiled TMA descriptor (128 bytes, written to out128, which
 * must be 64-byte aligned) for a row-major rows x cols matrix at d_base.
 * box_rows x box_cols is the copied box; swizzle_bytes is 0, 32, 64 or
 * 128.  Stands in for the descriptor that ThunderKittens' gl<> constructor
 * builds inside the generated launcher (codegen.py:447-455).               */
THORK_API int thork_tensor_map_2d(void *out128, int dtype, const void *d_base,
                        uint64_t rows, uint64_t cols, uint64_t row_stride_bytes,
                        uint32_t box_rows, uint32_t box_cols, int swizzle_bytes);

/* ---- kernel status --------------------------------------------------- */
/* Reads (and with clear != 0 resets) the current device's status word.
 * Kernels of this library and traced tile kernels set it when a bounded
 * wait gives up (code in bits 0-7, site in bits 8-15).  No reference
 * counterpart (the reference has no bounded waits).                       */
THORK_API int thork_kernel_status(unsigned *status, int clear);
/* Device address of the current device's status word, passed to traced tile
 * kernels as their hidden last parameter.                                  */
THORK_API int thork_status_pointer(void **d_status);

/* ---- library kernels --------------------------------------------------
 * All of these queue work on `stream` and return without synchronising.
 * Inputs and outputs are device pointers to dense row-major storage.      */

/* out[i] = a[i] + b[i] for i < n, fp32, bit-exact with IEEE addition.
 * Replaces the kernel of tk.kernels.matrix_add
 * (src/thork/kernels/matrix_add.py:15-52) and the traced README example
 * (README.md:54-85).                                                       */
THORK_API int thork_matrix_add_f32(float *d_out, const float *d_a, const float *d_b,
                         size_t n, void *stream);

/* C[M,N] = A[M,K] . B[K,N], bf16 in, fp32 accumulate (tcgen05, TMEM),
 * bf16 out.  Requires K % 8 == 0 and N % 8 == 0 (16-byte TMA strides).
 * `variant` 0 = automatic, 1 = 1-CTA 128x256 tiles, 2 = 2-CTA 256x256,
 * 3 = stream-K over 128x256 tiles (whole waves one tile per CTA, the tiles
 * of the last wave split into equal k-loop shares over all SMs).  The
 * automatic choice is 3 when the tiles fill at most half of the SMs, else
 * 2 when M > 128, else 1.
 * Replaces tk.kernels.matmul (src/thork/kernels/matmul.py:17-71, fp32 SIMT
 * only) for dtype=bfloat16, and the level-06 tcgen05 matmul that
 * tests/test_kittens.py:187-274 can only compile.                          */
THORK_API int thork_gemm_bf16(const void *d_a, const void *d_b, void *d_c,
                    int M, int N, int K, int variant, void *stream);

/* C[M,N] = (scale_a*scale_b) * (A[M,K] . B[K,N]) with A, B float8 e4m3
 * (bytes), fp32 accumulate, bf16 out.  Requires K % 16 == 0, N % 16 == 0.
 * Variants as for thork_gemm_bf16 (0 = 2-CTA above M=128, else 1-CTA).
 * No reference counterpart (the reference has no FP8 dtype,
 * src/thork/dtypes.py:18-36); it is tk.kernels.matmul(dtype=float8_e4m3). */
THORK_API int thork_gemm_e4m3(const void *d_a, const void *d_b, void *d_c,
                    int M, int N, int K, float scale_a, float scale_b,
                    int variant, void *stream);

/* Y[M,N] = X[M,K] . W[K,N] for small M (1..256), bf16 in/out, fp32
 * accumulate; memory-bound on W.  Requires K % 8 == 0 and N % 8 == 0.
 * Decode-shaped variant of tk.kernels.matmul(dtype=bfloat16)
 * (src/thork/kernels/matmul.py:17-71).                                     */
THORK_API int thork_skinny_gemm_bf16(const void *d_x, const void *d_w, void *d_y,
                           int M, int N, int K, void *stream);

/* C[M,N] rows [row0, row0+rows) = A_rows . B, written both to d_c (this
 * GPU's full M x N result buffer) and, over NVLink, to the same rows of each
 * peer's result buffer d_peer_c[0..n_peers) (pointers opened with
 * thork_ipc_open).  This fuses the GEMM with the all-gather of C: once every
 * rank's launch is complete (thork_peer_barrier), every rank holds the full
 * C.  bf16 in/out, K and N multiples of 8, at most 7 peers.
 * variant 1: the epilogue stores each tile to the peers itself;
 * variant 2: four extra warps per CTA share all (tile, peer) pushes of the
 *   grid (cooperative launch); needs d_tile_flags, ceil(rows/128) *
 *   ceil(N/64) zero-initialised words owned by this GPU, and `epoch` =
 *   1, 2, 3, ... for successive calls on the same flags (every variant
 *   counts on the flags when they are given, so calls may mix variants);
 * variant 0: 2 when n_peers >= 3, else 1.
 * No reference counterpart (the reference is single-GPU,
 * src/thork/runtime.py:85-105).                                            */
THORK_API int thork_gemm_bf16_allgather(const void *d_a_rows, const void *d_b, void *d_c,
                                        void *const *d_peer_c, int n_peers, int rows, int N, int K,
                                        int row0, unsigned *d_tile_flags, unsigned epoch,
                                        int variant, void *stream);
/* FP8 form of thork_gemm_bf16_allgather: e4m3 A rows and B (K, N multiples
 * of 16), C = scale_a * scale_b * A.B in bf16 rows on this GPU and every
 * peer.  No reference counterpart.                                         */
THORK_API int thork_gemm_e4m3_allgather(const void *d_a_rows, const void *d_b, void *d_c,
                                        void *const *d_peer_c, int n_peers, int rows, int N, int K,
                                        int row0, unsigned *d_tile_flags, unsigned epoch,
                                        float scale_a, float scale_b, int variant, void *stream);
/* Fused GEMM + all-gather through an NVLink multicast buffer: rows
 * [row0, row0+rows) of C = A_rows . B are written once, with multimem
 * stores, to d_c_multicast (the multicast view, thork_mc_bind, of a full
 * M x N bf16 result), which places them in every member GPU's memory.
 * Pair with thork_peer_barrier as for thork_gemm_bf16_allgather.  bf16:
 * K, N multiples of 8; e4m3: multiples of 16, C scaled by scale_a*scale_b.
 * No reference counterpart.                                                */
THORK_API int thork_gemm_bf16_allgather_mc(const void *d_a_rows, const void *d_b, void *d_c_multicast,
                                           int rows, int N, int K, int row0, void *stream);
THORK_API int thork_gemm_e4m3_allgather_mc(const void *d_a_rows, const void *d_b, void *d_c_multicast,
                                           int rows, int N, int K, int row0, float scale_a,
                                           float scale_b, void *stream);
/* Device-side barrier of the fused all-gather: this rank stores `epoch` into
 * slot `rank` of every peer's flag array (d_peer_flags[q], q != rank, each
 * `world` unsigned words in the peer's memory opened with thork_ipc_open)
 * after a system-scope fence, then waits until its own d_flags[q] reach
 * `epoch` for all q != rank.  The wait is bounded (1 s); on expiry the
 * kernel status word records it and the barrier returns.  One rank per GPU,
 * world <= 8.  No reference counterpart.                                   */
THORK_API int thork_peer_barrier(void *d_flags, void *const *d_peer_flags, int world, int rank,
                                 unsigned epoch, void *stream);
/* CUDA IPC for the fused all-gather: export a cudaMalloc'd buffer (64-byte
 * handle), open a peer's handle in this process, close it.                 */
THORK_API int thork_ipc_handle(const void *d_ptr, void *handle64);
THORK_API int thork_ipc_open(const void *handle64, void **d_ptr);
THORK_API int thork_ipc_close(void *d_ptr);

/* thork_skinny_gemm_bf16 with flags.  THORK_SKINNY_W_STATIC promises that
 * no kernel launched earlier on the stream writes W (decode weights): the
 * stream-K kernels (M <= 64 when the 128-column tiles fill at most half
 * of the SMs) then fetch W for their opening pipeline stages before the
 * programmatic-dependent-launch wait, overlapping the previous kernel's
 * tail.  X and Y keep the full stream ordering.  The one-CTA-per-tile
 * kernel of the other shapes ignores the flag (measured no faster).  No reference
 * counterpart.                                                            */
#define THORK_SKINNY_W_STATIC 1
THORK_API int thork_skinny_gemm_bf16_ex(const void *d_x, const void *d_w, void *d_y, int M, int N,
                                        int K, int flags, void *stream);

/* Allocation-free form of thork_skinny_gemm_bf16 for 1 <= M <= 32 (the
 * stream-K decode path).  No reference counterpart: it exists for callers
 * that must not allocate device memory, directly or through this library --
 * for example a serving process whose memory pool owns the whole GPU
 * budget, or a latency-critical path that cannot afford the device-wide
 * synchronisation cudaMalloc/cudaFree imply.  thork_skinny_gemm_bf16
 * allocates its workspace (and status word) on first use; this entry point
 * instead uses a fixed 8 MiB scratch array compiled into the library, which
 * every GPU that loads the library holds until the process exits.
 *   - The first call on a device looks up that device's address of the array;
 *     make that first call before any stream capture.
 *   - The scratch is shared by every call and keeps the last call's contents:
 *     each call clears the parts that must start at zero, and calls that can
 *     overlap on the GPU (different streams, other threads) race on it.
 *   - Limits: M <= 32 and ceil(N/128) <= 16384 output tiles (the split-tile
 *     partials, two slots per CTA, always fit); larger requests return
 *     THORK_ERR_INVALID with the sizes in the message.  Inputs, output and
 *     stream are as for thork_skinny_gemm_bf16; no cudaMalloc, cudaFree or
 *     other allocating call is made.
 *   - Failures: a bounded wait that expires inside this kernel is recorded
 *     in a status word inside the same scratch array, NOT in the word that
 *     thork_kernel_status reads.  Read it with
 *     thork_skinny_gemm_bf16_noalloc_status; it is sticky (later calls do
 *     not clear it), so a non-zero value means some call since the last
 *     clearing read may have left Y incomplete.                            */
THORK_API int thork_skinny_gemm_bf16_noalloc(const void *d_x, const void *d_w, void *d_y,
                                            int M, int N, int K, void *stream);
/* Status word of thork_skinny_gemm_bf16_noalloc on the current device: waits
 * for `stream`, copies the word into *status (0 = every call since the last
 * clear finished its waits; else code in bits 0-7, wait site in bits 8-15)
 * and resets it when clear != 0.  Allocates nothing.  No reference
 * counterpart.                                                             */
THORK_API int thork_skinny_gemm_bf16_noalloc_status(unsigned *status, int clear, void *stream);

/* ---- NVLink multicast buffers (no reference counterpart) ---------------
 * For the fused GEMM + all-gather over NVSwitch multicast ("NVLS"): every
 * GPU of a group binds memory of its own to one multicast object, and a
 * `multimem.st` to the multicast view from any GPU lands at the same offset
 * in every GPU's memory.  One process per GPU:
 *   1. one rank: thork_mc_create (the object and a POSIX descriptor to hand
 *      to the others, e.g. over a Unix socket); the others: thork_mc_import
 *      (the caller closes its received descriptor afterwards);
 *   2. every rank: thork_mc_add_device; then a host barrier;
 *   3. every rank: thork_mc_bind -> this GPU's ordinary (unicast) view and
 *      the multicast view; then a host barrier before any store;
 *   4. every rank, after a host barrier that no kernel is still storing:
 *      thork_mc_release (unmaps, unbinds and frees; closes the creator's
 *      descriptor).
 * A rank should not exit while its memory is bound: release it first.      */
/* *supported = 1 when the current device can join multicast objects shared
 * through POSIX file descriptors.                                          */
THORK_API int thork_mc_supported(int *supported);
/* Creates an object for `ndev` GPUs of at least `bytes` (rounded up to the
 * multicast granularity: *bytes_rounded).  *fd is owned by the object.     */
THORK_API int thork_mc_create(size_t bytes, int ndev, void **obj, int *fd, size_t *bytes_rounded);
/* Imports an object from a descriptor; `bytes_rounded` as reported by the
 * creator.                                                                 */
THORK_API int thork_mc_import(int fd, size_t bytes_rounded, void **obj);
/* Adds the current device to the object.                                  */
THORK_API int thork_mc_add_device(void *obj);
/* Allocates the current device's memory, binds it and maps both views.    */
THORK_API int thork_mc_bind(void *obj, void **d_local, void **d_multicast);
THORK_API int thork_mc_release(void *obj);

/* ---- NCCL (dlopen of libnccl.so.2; no reference counterpart) ---------- */
/* Writes a 128-byte ncclUniqueId into id128.                              */
THORK_API int thork_nccl_get_unique_id(void *id128);
/* One rank of a multi-process communicator (one process per GPU).  When
 * the environment variable THORK_FAULT_NCCL_INIT=1 is set, returns
 * THORK_ERR_NCCL before touching NCCL (host-side fault injection).        */
THORK_API int thork_nccl_comm_init_rank(void **comm, int nranks, const void *id128, int rank);
THORK_API int thork_nccl_comm_destroy(void *comm);
/* recv[r*count .. (r+1)*count) = send of rank r (ncclAllGather).          */
THORK_API int thork_nccl_allgather(const void *d_send, void *d_recv, size_t count, int dtype,
                         void *comm, void *stream);
/* In-place sum all-reduce of `count` elements (used for barriers).        */
THORK_API int thork_nccl_allreduce_sum(void *d_buf, size_t count, int dtype, void *comm, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* THORK_RT_H */
