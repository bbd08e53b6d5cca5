// sm100.cuh — sm_100a device primitives written as inline PTX from the PTX ISA:
// mbarriers with bounded waits, TMA (cp.async.bulk.tensor) loads and stores,
// tcgen05 TMEM allocation / MMA / commit / loads, and the shared-memory and
// instruction descriptors tcgen05.mma consumes.
//
// The header compiles under both nvcc (the prebuilt library kernels of
// libthork_rt.so) and NVRTC (traced @tk.jit tile kernels), so it includes no
// standard headers.  No TMA load here uses cluster multicast: the same kernels
// run in multi-GPU configurations.
#pragma once

#ifndef THORK_WAIT_TIMEOUT_NS
// Bound on any single wait inside a kernel.  A correct kernel never waits
// more than microseconds; on expiry the wait records a status code and the
// kernel unwinds instead of hanging the GPU.
#define THORK_WAIT_TIMEOUT_NS 1000000000ull
#endif

namespace thork {
namespace dev {

typedef unsigned int u32;
typedef unsigned long long u64;

// Status codes written to the status word (bits 0-7); the site id of the
// wait that expired goes to bits 8-15.
enum : u32 { STATUS_WAIT_TIMEOUT = 1u, STATUS_BAD_CONFIG = 2u };

struct alignas(64) TensorMap {  // opaque CUtensorMap (128 bytes)
  u64 opaque[16];
};

__device__ __forceinline__ u32 smem_u32(const void *p) {
  return static_cast<u32>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ u64 globaltimer() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ u32 lane_id() {
  u32 l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ void report_status(u32 *status, u32 code, u32 site) {
  if (status) atomicOr(status, code | (site << 8));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(u32 bar, u32 count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(u32 bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on a barrier of another CTA of the cluster (`cta` = its rank).
__device__ __forceinline__ void mbar_arrive_cluster(u32 bar, u32 cta) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(bar),
      "r"(cta)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(u32 bar, u32 bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(u32 bar, u32 bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(u32 bar, u32 parity) {
  u32 ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with parity `parity` to complete.  Returns false (and
// records STATUS_WAIT_TIMEOUT | site) if that takes longer than
// THORK_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool mbar_wait(u32 bar, u32 parity, u32 *status, u32 site) {
  if (mbar_try_wait(bar, parity)) return true;
  const u64 t0 = globaltimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > THORK_WAIT_TIMEOUT_NS) {
      report_status(status, STATUS_WAIT_TIMEOUT, site);
      return false;
    }
  }
}

// ---------------------------------------------------------------- dependent launch
// Allow the next kernel of the stream (launched with programmatic stream
// serialisation) to start its prologue on SMs this grid frees.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Wait until the preceding grid has completed and its writes are visible;
// returns at once when the launch had no programmatic dependency.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const TensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<u64>(m)) : "memory");
}

// 2-D tiled load of the box at element coordinates (x = inner/column,
// y = row) into shared memory; completion is signalled on `bar`.
__device__ __forceinline__ void tma_load_2d(u32 dst, const TensorMap *m, u32 bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<u64>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled store of a shared-memory box to global memory (bulk group).
// 2-D tiled load into this CTA's shared memory whose completion is counted
// on a barrier of either CTA of a cluster pair (cta_group::2 form;
// `bar_cluster` is a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(u32 dst, const TensorMap *m, u32 bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<u64>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const TensorMap *m, u32 src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::
                   "l"(reinterpret_cast<u64>(m)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups are still reading their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation is warp-collective; the address lands in shared memory.
template <int CTA_GROUP>
__device__ __forceinline__ void tmem_alloc(u32 dst_smem, u32 ncols) {
  if (CTA_GROUP == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

template <int CTA_GROUP>
__device__ __forceinline__ void tmem_relinquish() {
  if (CTA_GROUP == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CTA_GROUP>
__device__ __forceinline__ void tmem_dealloc(u32 taddr, u32 ncols) {
  if (CTA_GROUP == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]; kind::f16 (bf16/fp16 operands, fp32 accum).
__device__ __forceinline__ void mma_f16_ss(u32 d_tmem, u64 a_desc, u64 b_desc, u32 idesc,
                                           u32 accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f8f6f4 (e4m3/e5m2/... operands, fp32 accum).
__device__ __forceinline__ void mma_f8f6f4_ss(u32 d_tmem, u64 a_desc, u64 b_desc, u32 idesc,
                                              u32 accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2-CTA (cta_group::2) forms, issued by the even CTA of a cluster pair.
__device__ __forceinline__ void mma2_f16_ss(u32 d_tmem, u64 a_desc, u64 b_desc, u32 idesc,
                                            u32 accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma2_f8f6f4_ss(u32 d_tmem, u64 a_desc, u64 b_desc, u32 idesc,
                                               u32 accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all tcgen05 ops issued so far by this thread are
// complete.
__device__ __forceinline__ void tc_commit(u32 bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 2-CTA commit: `bar` is a shared::cluster address (may be the peer CTA's).
__device__ __forceinline__ void tc_commit2(u32 bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

__device__ __forceinline__ u32 mapa_cluster(u32 smem_addr, u32 cta) {
  u32 r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(cta));
  return r;
}

__device__ __forceinline__ u32 cluster_ctarank() {
  u32 r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// row (lane base + i), columns [col, col+32) of the TMEM address.
__device__ __forceinline__ void tmem_ld_32x32b_x32(u32 taddr, u32 (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(u32 taddr, u32 (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05 "version 1" format):
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4
//   bits 32-45  stride-dimension byte offset >> 4
//   bits 46-47  version = 1
//   bits 49-51  base offset (0: every tile here is 1024-byte aligned)
//   bit  52     LBO mode (0)
//   bits 61-63  layout: 2 = 128-byte swizzle
// For the 128-byte-swizzled canonical layouts used here:
//   K-major : rows of 128 bytes, 8-row groups SBO = 1024 bytes apart; LBO unused (16).
//   MN-major: 64-element (128-byte) MN chunks LBO bytes apart, 8-row K groups
//             SBO = 1024 bytes apart.
__device__ __forceinline__ u64 smem_desc_sw128(u32 addr, u32 lbo_bytes, u32 sbo_bytes) {
  u64 d = 0;
  d |= static_cast<u64>((addr >> 4) & 0x3FFFu);
  d |= static_cast<u64>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<u64>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for dense tcgen05.mma with fp32 accumulation:
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format,
//   bit 15 A major (1 = MN), bit 16 B major (1 = MN), 17-22 N>>3, 24-28 M>>4.
// Formats: kind::f16 -> 0 = f16, 1 = bf16; kind::f8f6f4 -> 0 = e4m3, 1 = e5m2.
__host__ __device__ constexpr u32 make_idesc(u32 a_fmt, u32 b_fmt, bool a_mn, bool b_mn, u32 M,
                                             u32 N) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ---------------------------------------------------------------- conversions
__device__ __forceinline__ u32 pack_bf16x2(float lo, float hi) {
  u32 r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 16-byte store to a multicast (NVLS) address: the NVSwitch writes it to the
// same offset in every member GPU's memory, this one included.
__device__ __forceinline__ void multimem_st_v4(void *p, u32 a, u32 b, u32 c, u32 d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a),
               "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Orders this thread's accesses through a multicast view before later ones
// through an ordinary view of the same memory (and the reverse).
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

__device__ __forceinline__ void st_global_v4(void *p, u32 a, u32 b, u32 c, u32 d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

}  // namespace dev
}  // namespace thork
