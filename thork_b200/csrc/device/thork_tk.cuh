// thork_tk.cuh — tile library behind the `tk.kittens` front end: the target of
// traced tile kernels (compiled by NVRTC for sm_100a).
//
// Provides, in the ThunderKittens vocabulary the front end exposes:
//   gl<T, TR, TC>   global tile view passed by value (__grid_constant__): a TMA
//                   tensor map for TR x TC boxes plus pointer/rows/cols
//   st<T, R, C>     shared tile, stored as column chunks of one swizzle width
//                   (128/64/32 bytes), each R rows deep; the same layout TMA
//                   writes and tcgen05.mma reads (K-major or MN-major)
//   rt<T, R, C, L>  register tile of one warp, 16x16 sub-tiles in mma.sync
//                   fragment order (L = 0 row layout, 1 column layout)
//   tt<T, R, C>     tensor-memory (TMEM) accumulator tile
//   semaphore       an mbarrier
// and the warp / warpgroup / tma / tcgen05 operations on them.  Every wait is
// bounded (THORK_WAIT_TIMEOUT_NS) and reports to the launch's status word.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace thork {
namespace tk {

using namespace thork::dev;
typedef __nv_bfloat16 bf16;
typedef __half half;

struct coord {
  int r, c;
};

// ------------------------------------------------------------------ globals
template <class T, int TR, int TC>
struct gl {
  TensorMap tmap;  // valid when the parameter was declared with a tile shape
  T *ptr;
  unsigned long long rows;
  unsigned long long cols;
};

// ------------------------------------------------------------------ shared tiles
template <class T, int R, int C>
struct st {
  static constexpr int E = sizeof(T);
  static constexpr int RB = C * E;  // bytes of one logical row
  static constexpr int SW = (RB % 128 == 0) ? 128 : (RB % 64 == 0) ? 64 : (RB % 32 == 0) ? 32 : 0;
  static constexpr int CC = SW ? SW / E : C;  // columns per chunk
  static constexpr int NCH = C / CC;          // chunks
  static constexpr int ROWB = SW ? SW : RB;   // bytes of one chunk row
  static constexpr int CHB = R * ROWB;        // bytes of one chunk
  static constexpr int BYTES = R * C * E;
  static constexpr int rows = R, cols = C;
  static_assert(R % 8 == 0, "shared tile rows must be a multiple of 8");
  static_assert(RB % 16 == 0, "shared tile rows must be a multiple of 16 bytes");
  unsigned char raw[BYTES];

  __device__ __forceinline__ u32 base() const { return smem_u32(raw); }
  // byte offset of element (r, c): chunk, row, column, then the swizzle XOR of
  // address bits [4, 4+log2(SW/16)) with bits [7, ...), as TMA applies it
  static __device__ __forceinline__ u32 offset(int r, int c) {
    u32 off = (c / CC) * CHB + r * ROWB + (c % CC) * E;
    if (SW) off ^= ((off >> 7) & (SW / 16 - 1)) << 4;
    return off;
  }
};

// ------------------------------------------------------------------ register tiles
template <class T>
struct frag {  // one 16x16 sub-tile of a 16-bit type: 4 packed pairs
  u32 v[4];
};
template <>
struct frag<float> {  // fp32 accumulator sub-tile
  float v[8];
};

// Row layout (16-bit): v[q], quadrant q = (row block q&1, column block q>>1);
//   lane holds row 8*(q&1) + lane/4, columns 8*(q>>1) + 2*(lane%4) + {0,1}.
// Column layout (16-bit): v[q] holds the transpose of the same quadrant:
//   lane holds column 8*(q>>1) + lane/4, rows 8*(q&1) + 2*(lane%4) + {0,1}.
// fp32 (row layout only): v[4h + i]: columns 8h + 2*(lane%4) + {0,1} (i&1),
//   row lane/4 (i < 2) or 8 + lane/4 (i >= 2) — the mma C fragment.
template <class T, int R, int C, int L = 0>
struct rt {
  static_assert(R % 16 == 0 && C % 16 == 0, "register tile dims must be multiples of 16");
  static constexpr int rows = R, cols = C, SR = R / 16, SC = C / 16, layout = L;
  frag<T> t[SR][SC];
};

template <class T>
__device__ __forceinline__ u32 pack2(float lo, float hi);
template <>
__device__ __forceinline__ u32 pack2<bf16>(float lo, float hi) {
  return pack_bf16x2(lo, hi);
}
template <>
__device__ __forceinline__ u32 pack2<half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<u32 *>(&h);
}
template <class T>
__device__ __forceinline__ void unpack2(u32 v, float &lo, float &hi);
template <>
__device__ __forceinline__ void unpack2<bf16>(u32 v, float &lo, float &hi) {
  lo = __uint_as_float(v << 16);
  hi = __uint_as_float(v & 0xFFFF0000u);
}
template <>
__device__ __forceinline__ void unpack2<half>(u32 v, float &lo, float &hi) {
  __half2 h = *reinterpret_cast<__half2 *>(&v);
  float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}

template <class T>
__device__ __forceinline__ float to_f(T x) {
  return static_cast<float>(x);
}
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f<half>(half x) {
  return __half2float(x);
}
template <class T>
__device__ __forceinline__ T from_f(float x) {
  return static_cast<T>(x);
}
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ half from_f<half>(float x) {
  return __float2half_rn(x);
}

// element (r, c) of a sub-tile position: helpers for the scalar paths
__device__ __forceinline__ int lane_g() { return static_cast<int>(lane_id()) >> 2; }
__device__ __forceinline__ int lane_t() { return static_cast<int>(lane_id()) & 3; }

// ------------------------------------------------------------------ per-CTA state
__device__ __forceinline__ volatile int &abort_flag() {
  __shared__ int flag;
  return flag;
}

__device__ __forceinline__ void kernel_begin() {
  if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) abort_flag() = 0;
  __syncthreads();
}

__device__ __forceinline__ void kernel_end() {
  bulk_wait<0>();  // outstanding TMA stores of this thread complete
}

// ------------------------------------------------------------------ semaphores
struct alignas(8) semaphore {
  unsigned long long bar;
};

__device__ __forceinline__ u32 sem_addr(semaphore &s) { return smem_u32(&s.bar); }

__device__ __forceinline__ void init_semaphore(semaphore &s, int thread_count, int tx_count) {
  mbar_init(sem_addr(s), static_cast<u32>(thread_count + tx_count));
  fence_mbar_init();
}

__device__ __forceinline__ void wait(semaphore &s, int phase, u32 *status) {
  if (abort_flag()) return;
  if (!mbar_wait(sem_addr(s), static_cast<u32>(phase & 1), status, 0x40)) abort_flag() = 1;
}

// Also orders this thread's earlier tensor-memory accesses (tcgen05.ld of an
// accumulator being handed back) before the arrival.
__device__ __forceinline__ void arrive(semaphore &s) {
  tc_fence_before();
  mbar_arrive(sem_addr(s));
}

// ------------------------------------------------------------------ warp scope
namespace warp {

template <class T, int R, int C, int L>
__device__ __forceinline__ void zero(rt<T, R, C, L> &x) {
#pragma unroll
  for (int i = 0; i < R / 16; ++i)
#pragma unroll
    for (int j = 0; j < C / 16; ++j)
#pragma unroll
      for (int k = 0; k < (int)(sizeof(x.t[0][0].v) / sizeof(x.t[0][0].v[0])); ++k) x.t[i][j].v[k] = 0;
}

// shared -> register (16-bit types), ldmatrix.x4 per sub-tile; the column
// layout uses the transposing form.  row0 offsets into the shared tile.
template <class T, int R, int C, int L, int SR_, int SC_>
__device__ __forceinline__ void load(rt<T, R, C, L> &dst, const st<T, SR_, SC_> &src, int row0 = 0) {
  static_assert(sizeof(T) == 2, "ldmatrix path is for 16-bit tiles");
  const int lane = lane_id();
  const int j = lane >> 3;  // matrix index supplied by this lane's address
#pragma unroll
  for (int i = 0; i < R / 16; ++i)
#pragma unroll
    for (int k = 0; k < C / 16; ++k) {
      const int r = row0 + 16 * i + 8 * (j & 1) + (lane & 7);
      const int c = 16 * k + 8 * (j >> 1);
      const u32 a = src.base() + st<T, SR_, SC_>::offset(r, c);
      u32 *v = dst.t[i][k].v;
      if (L == 0)
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                     : "r"(a));
      else
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                     : "r"(a));
    }
}

// register -> shared; fp32 tiles are converted to the shared tile's type.
// Ends with a proxy fence so a TMA store issued after the next barrier sees it.
template <class TS, class TR, int R, int C, int SR_, int SC_>
__device__ __forceinline__ void store(st<TS, SR_, SC_> &dst, const rt<TR, R, C, 0> &src, int row0 = 0) {
  const int g = lane_g(), t = lane_t();
  unsigned char *base = dst.raw;
#pragma unroll
  for (int i = 0; i < R / 16; ++i)
#pragma unroll
    for (int k = 0; k < C / 16; ++k)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = row0 + 16 * i + 8 * (q & 1) + g;
        const int c = 16 * k + 8 * (q >> 1) + 2 * t;
        float lo, hi;
        if constexpr (sizeof(TR) == 4) {
          // fp32 fragment: quadrant q -> (row half q&1, column half q>>1)
          lo = src.t[i][k].v[4 * (q >> 1) + 2 * (q & 1)];
          hi = src.t[i][k].v[4 * (q >> 1) + 2 * (q & 1) + 1];
        } else {
          unpack2<TR>(src.t[i][k].v[q], lo, hi);
        }
        if constexpr (sizeof(TS) == 2) {
          *reinterpret_cast<u32 *>(base + st<TS, SR_, SC_>::offset(r, c)) = pack2<TS>(lo, hi);
        } else {
          *reinterpret_cast<TS *>(base + st<TS, SR_, SC_>::offset(r, c)) = from_f<TS>(lo);
          *reinterpret_cast<TS *>(base + st<TS, SR_, SC_>::offset(r, c + 1)) = from_f<TS>(hi);
        }
      }
  fence_proxy_async_smem();
}

// register -> global at tile coordinate (rows of R, columns of C), bounds-checked
template <class TG, int GR, int GC, class TR, int R, int C>
__device__ __forceinline__ void store(const gl<TG, GR, GC> &dst, const rt<TR, R, C, 0> &src, coord at,
                                      int row0 = 0, int tile_rows = R) {
  const int g = lane_g(), t = lane_t();
#pragma unroll
  for (int i = 0; i < R / 16; ++i)
#pragma unroll
    for (int k = 0; k < C / 16; ++k)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const long long r = (long long)at.r * tile_rows + row0 + 16 * i + 8 * (q & 1) + g;
        const long long c = (long long)at.c * C + 16 * k + 8 * (q >> 1) + 2 * t;
        float lo, hi;
        if constexpr (sizeof(TR) == 4) {
          lo = src.t[i][k].v[4 * (q >> 1) + 2 * (q & 1)];
          hi = src.t[i][k].v[4 * (q >> 1) + 2 * (q & 1) + 1];
        } else {
          unpack2<TR>(src.t[i][k].v[q], lo, hi);
        }
        if (r < (long long)dst.rows) {
          TG *p = dst.ptr + r * (long long)dst.cols + c;
          if (c < (long long)dst.cols) p[0] = from_f<TG>(lo);
          if (c + 1 < (long long)dst.cols) p[1] = from_f<TG>(hi);
        }
      }
}

// global -> register at tile coordinate (scalar loads, zero outside)
template <class T, int R, int C, class TG, int GR, int GC>
__device__ __forceinline__ void load(rt<T, R, C, 0> &dst, const gl<TG, GR, GC> &src, coord at) {
  const int g = lane_g(), t = lane_t();
#pragma unroll
  for (int i = 0; i < R / 16; ++i)
#pragma unroll
    for (int k = 0; k < C / 16; ++k)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const long long r = (long long)at.r * R + 16 * i + 8 * (q & 1) + g;
        const long long c = (long long)at.c * C + 16 * k + 8 * (q >> 1) + 2 * t;
        float lo = 0.f, hi = 0.f;
        if (r < (long long)src.rows) {
          const TG *p = src.ptr + r * (long long)src.cols + c;
          if (c < (long long)src.cols) lo = to_f<TG>(p[0]);
          if (c + 1 < (long long)src.cols) hi = to_f<TG>(p[1]);
        }
        if constexpr (sizeof(T) == 4) {
          dst.t[i][k].v[4 * (q >> 1) + 2 * (q & 1)] = lo;
          dst.t[i][k].v[4 * (q >> 1) + 2 * (q & 1) + 1] = hi;
        } else {
          dst.t[i][k].v[q] = pack2<T>(lo, hi);
        }
      }
}

// global -> shared (cooperative over `nthreads` threads starting at `tid0`),
// 16-byte pieces, zero outside the matrix
template <class T, int R, int C, class TG, int GR, int GC>
__device__ __forceinline__ void load(st<T, R, C> &dst, const gl<TG, GR, GC> &src, coord at,
                                     int tid = -1, int nthreads = 32) {
  static_assert(sizeof(T) == sizeof(TG), "shared and global element sizes differ");
  constexpr int PER = 16 / sizeof(T);  // elements per 16-byte piece
  if (tid < 0) tid = lane_id();
  for (int idx = tid; idx < R * C / PER; idx += nthreads) {
    const int r = idx / (C / PER);
    const int c = (idx % (C / PER)) * PER;
    const long long gr = (long long)at.r * R + r;
    const long long gc = (long long)at.c * C + c;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (gr < (long long)src.rows) {
      const T *p = reinterpret_cast<const T *>(src.ptr) + gr * (long long)src.cols + gc;
      if (gc + PER <= (long long)src.cols && ((reinterpret_cast<unsigned long long>(p) & 15) == 0)) {
        v = *reinterpret_cast<const uint4 *>(p);
      } else {
        T tmp[PER];
        for (int e = 0; e < PER; ++e) tmp[e] = (gc + e < (long long)src.cols) ? p[e] : T();
        v = *reinterpret_cast<uint4 *>(tmp);
      }
    }
    *reinterpret_cast<uint4 *>(dst.raw + st<T, R, C>::offset(r, c)) = v;
  }
  fence_proxy_async_smem();
}

// shared -> global (cooperative), bounds-checked
template <class TG, int GR, int GC, class T, int R, int C>
__device__ __forceinline__ void store(const gl<TG, GR, GC> &dst, const st<T, R, C> &src, coord at,
                                      int tid = -1, int nthreads = 32) {
  static_assert(sizeof(T) == sizeof(TG), "shared and global element sizes differ");
  constexpr int PER = 16 / sizeof(T);
  if (tid < 0) tid = lane_id();
  for (int idx = tid; idx < R * C / PER; idx += nthreads) {
    const int r = idx / (C / PER);
    const int c = (idx % (C / PER)) * PER;
    const long long gr = (long long)at.r * R + r;
    const long long gc = (long long)at.c * C + c;
    if (gr >= (long long)dst.rows) continue;
    const uint4 v = *reinterpret_cast<const uint4 *>(src.raw + st<T, R, C>::offset(r, c));
    T *p = reinterpret_cast<T *>(dst.ptr) + gr * (long long)dst.cols + gc;
    if (gc + PER <= (long long)dst.cols && ((reinterpret_cast<unsigned long long>(p) & 15) == 0)) {
      *reinterpret_cast<uint4 *>(p) = v;
    } else {
      const T *tmp = reinterpret_cast<const T *>(&v);
      for (int e = 0; e < PER; ++e)
        if (gc + e < (long long)dst.cols) p[e] = tmp[e];
    }
  }
}

// row <-> column layout of a 16-bit register tile (movmatrix per quadrant)
template <class T, int R, int C, int L1, int L2>
__device__ __forceinline__ void swap_layout(rt<T, R, C, L1> &dst, const rt<T, R, C, L2> &src) {
  static_assert(sizeof(T) == 2 && L1 != L2, "swap_layout converts 16-bit tiles between layouts");
#pragma unroll
  for (int i = 0; i < R / 16; ++i)
#pragma unroll
    for (int k = 0; k < C / 16; ++k)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;"
                     : "=r"(dst.t[i][k].v[q])
                     : "r"(src.t[i][k].v[q]));
}

template <class T>
__device__ __forceinline__ void mma16816(float (&d)[4], const u32 (&a)[4], u32 b0, u32 b1, const float (&c)[4]);
template <>
__device__ __forceinline__ void mma16816<bf16>(float (&d)[4], const u32 (&a)[4], u32 b0, u32 b1,
                                               const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}
template <>
__device__ __forceinline__ void mma16816<half>(float (&d)[4], const u32 (&a)[4], u32 b0, u32 b1,
                                               const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}

// D = A . B + C_in with B in column layout (K x N)
template <class T, int M, int N, int K>
__device__ __forceinline__ void mma_AB(rt<float, M, N, 0> &d, const rt<T, M, K, 0> &a,
                                       const rt<T, K, N, 1> &b, const rt<float, M, N, 0> &c) {
#pragma unroll
  for (int i = 0; i < M / 16; ++i)
#pragma unroll
    for (int j = 0; j < N / 16; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float acc[4] = {c.t[i][j].v[4 * h], c.t[i][j].v[4 * h + 1], c.t[i][j].v[4 * h + 2],
                        c.t[i][j].v[4 * h + 3]};
#pragma unroll
        for (int k = 0; k < K / 16; ++k) {
          const u32 av[4] = {a.t[i][k].v[0], a.t[i][k].v[1], a.t[i][k].v[2], a.t[i][k].v[3]};
          float out[4];
          mma16816<T>(out, av, b.t[k][j].v[2 * h], b.t[k][j].v[2 * h + 1], acc);
          acc[0] = out[0], acc[1] = out[1], acc[2] = out[2], acc[3] = out[3];
        }
        d.t[i][j].v[4 * h] = acc[0];
        d.t[i][j].v[4 * h + 1] = acc[1];
        d.t[i][j].v[4 * h + 2] = acc[2];
        d.t[i][j].v[4 * h + 3] = acc[3];
      }
}

// D = A . B^T + C_in with B (N x K) in row layout
template <class T, int M, int N, int K>
__device__ __forceinline__ void mma_AB_t(rt<float, M, N, 0> &d, const rt<T, M, K, 0> &a,
                                         const rt<T, N, K, 0> &b, const rt<float, M, N, 0> &c) {
#pragma unroll
  for (int i = 0; i < M / 16; ++i)
#pragma unroll
    for (int j = 0; j < N / 16; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float acc[4] = {c.t[i][j].v[4 * h], c.t[i][j].v[4 * h + 1], c.t[i][j].v[4 * h + 2],
                        c.t[i][j].v[4 * h + 3]};
#pragma unroll
        for (int k = 0; k < K / 16; ++k) {
          const u32 av[4] = {a.t[i][k].v[0], a.t[i][k].v[1], a.t[i][k].v[2], a.t[i][k].v[3]};
          float out[4];
          mma16816<T>(out, av, b.t[j][k].v[h], b.t[j][k].v[h + 2], acc);
          acc[0] = out[0], acc[1] = out[1], acc[2] = out[2], acc[3] = out[3];
        }
        d.t[i][j].v[4 * h] = acc[0];
        d.t[i][j].v[4 * h + 1] = acc[1];
        d.t[i][j].v[4 * h + 2] = acc[2];
        d.t[i][j].v[4 * h + 3] = acc[3];
      }
}

}  // namespace warp

// ------------------------------------------------------------------ TMEM
template <class T, int R, int C>
struct tt {
  static constexpr int rows = R, cols = C;
  u32 addr;  // lane << 16 | column
};

template <int NCOLS>
__device__ __forceinline__ void tmem_acquire(u32 *slot) {
  if (threadIdx.x / 32 == 0) {
    tmem_alloc<1>(smem_u32(slot), NCOLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

template <int NCOLS>
__device__ __forceinline__ void tmem_release(u32 *slot) {
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x / 32 == 0) tmem_dealloc<1>(*slot, NCOLS);
}

// ------------------------------------------------------------------ clusters
// A pair of CTAs (cluster (2,1,1)) shares one tcgen05 MMA of M = 256: rank 0
// (the leader) issues it, each CTA holds 128 rows of A, half of B's columns
// and its 128 accumulator rows in its own TMEM.
__device__ __forceinline__ int cluster_ctarank() { return static_cast<int>(dev::cluster_ctarank()); }
__device__ __forceinline__ void cluster_sync() { dev::cluster_sync(); }

// TMEM for a CTA pair: warp 0 of both CTAs allocates with cta_group::2 (the
// same columns in both); released after a cluster barrier, so neither CTA
// frees its columns while the leader's MMAs may still write them.
template <int NCOLS>
__device__ __forceinline__ void tmem_acquire2(u32 *slot) {
  if (threadIdx.x / 32 == 0) {
    tmem_alloc<2>(smem_u32(slot), NCOLS);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  __syncthreads();
  dev::cluster_sync();  // both CTAs' semaphores are initialised before remote use
  tc_fence_after();
}

template <int NCOLS>
__device__ __forceinline__ void tmem_release2(u32 *slot) {
  tc_fence_before();
  __syncthreads();
  dev::cluster_sync();
  tc_fence_after();
  if (threadIdx.x / 32 == 0) tmem_dealloc<2>(*slot, NCOLS);
}

template <class TT>
__device__ __forceinline__ TT tensor_alloc(u32 slot, int col_offset) {
  TT t;
  t.addr = slot + static_cast<u32>(col_offset);
  return t;
}

template <int SW>
__device__ __forceinline__ u64 smem_desc(u32 addr, u32 lbo, u32 sbo) {
  static_assert(SW == 128 || SW == 64 || SW == 32, "tcgen05 operands need a swizzled shared tile");
  u64 d = 0;
  d |= static_cast<u64>((addr >> 4) & 0x3FFFu);
  d |= static_cast<u64>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<u64>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<u64>(SW == 128 ? 2 : SW == 64 ? 4 : 6) << 61;
  return d;
}

// K-major operand (rows = M or N, columns = K) for the UMMA_K-wide step `kk`
template <class T, int R, int C>
__device__ __forceinline__ u64 desc_kmajor(const st<T, R, C> &s, int kk) {
  using S = st<T, R, C>;
  const int k0 = kk * (32 / (int)sizeof(T));
  const u32 a = s.base() + (k0 / S::CC) * S::CHB + (k0 % S::CC) * sizeof(T);
  return smem_desc<S::SW>(a, 16, 8 * S::SW);
}

// MN-major operand (rows = K, columns = M or N) for step `kk`
template <class T, int R, int C>
__device__ __forceinline__ u64 desc_mnmajor(const st<T, R, C> &s, int kk) {
  using S = st<T, R, C>;
  const int k0 = kk * (32 / (int)sizeof(T));
  return smem_desc<S::SW>(s.base() + k0 * S::ROWB, S::CHB, 8 * S::SW);
}

template <class T>
struct umma_fmt;
template <>
struct umma_fmt<bf16> {
  static constexpr u32 v = 1;
};
template <>
struct umma_fmt<half> {
  static constexpr u32 v = 0;
};

// D(tt) (+)= A(st, M x K) . B(st, K x N), one thread issues; `sem` is signalled
// by tcgen05.commit when the operands have been consumed.
template <bool ACC, class T, int M, int N, int K, int KB, int NB>
__device__ __forceinline__ void umma_ab(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, KB, NB> &b,
                                        semaphore &sem) {
  tc_fence_after();  // after the semaphore wait that handed this thread the operands
  static_assert(KB == K && NB == N, "tcgen05 operand shapes disagree");
  static_assert(M == 64 || M == 128, "tcgen05 (one CTA) needs M = 64 or 128");
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "tcgen05 N must be 16..256, a multiple of 16");
  constexpr u32 idesc = make_idesc(umma_fmt<T>::v, umma_fmt<T>::v, false, true, M, N);
#pragma unroll
  for (int kk = 0; kk < K / 16; ++kk)
    mma_f16_ss(d.addr, desc_kmajor(a, kk), desc_mnmajor(b, kk), idesc, (ACC || kk > 0) ? 1u : 0u);
  tc_commit(sem_addr(sem));
}

// D(tt) (+)= A(st, M x K) . B(st, N x K)^T
template <bool ACC, class T, int M, int N, int K, int NB, int KB>
__device__ __forceinline__ void umma_abt(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, NB, KB> &b,
                                         semaphore &sem) {
  tc_fence_after();  // after the semaphore wait that handed this thread the operands
  static_assert(KB == K && NB == N, "tcgen05 operand shapes disagree");
  static_assert(M == 64 || M == 128, "tcgen05 (one CTA) needs M = 64 or 128");
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "tcgen05 N must be 16..256, a multiple of 16");
  constexpr u32 idesc = make_idesc(umma_fmt<T>::v, umma_fmt<T>::v, false, false, M, N);
#pragma unroll
  for (int kk = 0; kk < K / 16; ++kk)
    mma_f16_ss(d.addr, desc_kmajor(a, kk), desc_kmajor(b, kk), idesc, (ACC || kk > 0) ? 1u : 0u);
  tc_commit(sem_addr(sem));
}

// 2-CTA forms (issued by the leader CTA of a pair): D (+)= A . B with
// M = 256.  Each CTA passes its own tiles at the same shared offsets: A is
// its 128 rows (128 x K), B its half of the columns (K x N/2); D is each
// CTA's 128 x N accumulator.  `sem` is signalled in both CTAs.
__device__ __forceinline__ void commit_pair(semaphore &sem) {
  tc_commit2(mapa_cluster(sem_addr(sem), 0));
  tc_commit2(mapa_cluster(sem_addr(sem), 1));
}

template <bool ACC, class T, int M, int N, int K, int KB, int NH>
__device__ __forceinline__ void umma2_ab(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, KB, NH> &b,
                                         semaphore &sem) {
  tc_fence_after();  // after the semaphore wait that handed this thread the operands
  static_assert(KB == K && 2 * NH == N, "2-CTA tcgen05: B holds K x N/2 per CTA");
  static_assert(M == 128, "2-CTA tcgen05: 128 rows per CTA (M = 256 per pair)");
  static_assert(N % 32 == 0 && N >= 32 && N <= 256, "2-CTA tcgen05 N must be 32..256, a multiple of 32");
  constexpr u32 idesc = make_idesc(umma_fmt<T>::v, umma_fmt<T>::v, false, true, 2 * M, N);
#pragma unroll
  for (int kk = 0; kk < K / 16; ++kk)
    mma2_f16_ss(d.addr, desc_kmajor(a, kk), desc_mnmajor(b, kk), idesc, (ACC || kk > 0) ? 1u : 0u);
  commit_pair(sem);
}

template <bool ACC, class T, int M, int N, int K, int NH, int KB>
__device__ __forceinline__ void umma2_abt(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, NH, KB> &b,
                                          semaphore &sem) {
  tc_fence_after();  // after the semaphore wait that handed this thread the operands
  static_assert(KB == K && 2 * NH == N, "2-CTA tcgen05: B holds N/2 x K per CTA");
  static_assert(M == 128, "2-CTA tcgen05: 128 rows per CTA (M = 256 per pair)");
  static_assert(N % 32 == 0 && N >= 32 && N <= 256, "2-CTA tcgen05 N must be 32..256, a multiple of 32");
  constexpr u32 idesc = make_idesc(umma_fmt<T>::v, umma_fmt<T>::v, false, false, 2 * M, N);
#pragma unroll
  for (int kk = 0; kk < K / 16; ++kk)
    mma2_f16_ss(d.addr, desc_kmajor(a, kk), desc_kmajor(b, kk), idesc, (ACC || kk > 0) ? 1u : 0u);
  commit_pair(sem);
}

template <int NCTA>
__device__ __forceinline__ void tcgen05_commit(semaphore &sem) {
  static_assert(NCTA == 1 || NCTA == 2, "tcgen05 commits span one CTA or a pair");
  if constexpr (NCTA == 1)
    tc_commit(sem_addr(sem));
  else
    commit_pair(sem);
}

__device__ __forceinline__ void tensor_load_wait() { tmem_wait_ld(); }

// ------------------------------------------------------------------ warpgroup scope
namespace warpgroup {

__device__ __forceinline__ int laneid() { return static_cast<int>(threadIdx.x & 127); }
__device__ __forceinline__ int warpid() { return static_cast<int>((threadIdx.x >> 5) & 3); }

__device__ __forceinline__ void sync(int id) {
  asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory");
}

template <class T, int R, int C, int L>
__device__ __forceinline__ void zero(rt<T, R, C, L> &x) {
  warp::zero(x);
}

// each warp moves its R-row slice (rows warpid*R ...) of the shared tile
template <class T, int R, int C, int L, int SR_, int SC_>
__device__ __forceinline__ void load(rt<T, R, C, L> &dst, const st<T, SR_, SC_> &src) {
  warp::load(dst, src, warpid() * R);
}

template <class TS, class TR, int R, int C, int SR_, int SC_>
__device__ __forceinline__ void store(st<TS, SR_, SC_> &dst, const rt<TR, R, C, 0> &src) {
  warp::store(dst, src, warpid() * R);
}

template <class TG, int GR, int GC, class TR, int R, int C>
__device__ __forceinline__ void store(const gl<TG, GR, GC> &dst, const rt<TR, R, C, 0> &src, coord at) {
  warp::store(dst, src, at, warpid() * R, 4 * R);
}

template <class T, int R, int C, class TG, int GR, int GC>
__device__ __forceinline__ void load(st<T, R, C> &dst, const gl<TG, GR, GC> &src, coord at) {
  warp::load(dst, src, at, laneid(), 128);
}

template <class TG, int GR, int GC, class T, int R, int C>
__device__ __forceinline__ void store(const gl<TG, GR, GC> &dst, const st<T, R, C> &src, coord at) {
  warp::store(dst, src, at, laneid(), 128);
}

template <class T, int M, int N, int K>
__device__ __forceinline__ void mma_AB(rt<float, M, N, 0> &d, const rt<T, M, K, 0> &a,
                                       const rt<T, K, N, 1> &b, const rt<float, M, N, 0> &c) {
  warp::mma_AB(d, a, b, c);
}

template <class T, int M, int N, int K>
__device__ __forceinline__ void mma_AB_t(rt<float, M, N, 0> &d, const rt<T, M, K, 0> &a,
                                         const rt<T, N, K, 0> &b, const rt<float, M, N, 0> &c) {
  warp::mma_AB_t(d, a, b, c);
}

template <class T, int M, int N, int K, int KB, int NB>
__device__ __forceinline__ void mm_AB(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, KB, NB> &b,
                                      semaphore &sem) {
  umma_ab<false>(d, a, b, sem);
}
template <class T, int M, int N, int K, int KB, int NB>
__device__ __forceinline__ void mma_AB(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, KB, NB> &b,
                                       semaphore &sem) {
  umma_ab<true>(d, a, b, sem);
}
template <class T, int M, int N, int K, int NB, int KB>
__device__ __forceinline__ void mm_ABt(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, NB, KB> &b,
                                       semaphore &sem) {
  umma_abt<false>(d, a, b, sem);
}
template <class T, int M, int N, int K, int NB, int KB>
__device__ __forceinline__ void mma_AB_t(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, NB, KB> &b,
                                         semaphore &sem) {
  umma_abt<true>(d, a, b, sem);
}

template <class T, int M, int N, int K, int KB, int NH>
__device__ __forceinline__ void mm2_AB(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, KB, NH> &b,
                                       semaphore &sem) {
  umma2_ab<false>(d, a, b, sem);
}
template <class T, int M, int N, int K, int KB, int NH>
__device__ __forceinline__ void mma2_AB(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, KB, NH> &b,
                                        semaphore &sem) {
  umma2_ab<true>(d, a, b, sem);
}
template <class T, int M, int N, int K, int NH, int KB>
__device__ __forceinline__ void mm2_ABt(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, NH, KB> &b,
                                        semaphore &sem) {
  umma2_abt<false>(d, a, b, sem);
}
template <class T, int M, int N, int K, int NH, int KB>
__device__ __forceinline__ void mma2_AB_t(tt<float, M, N> &d, const st<T, M, K> &a, const st<T, NH, KB> &b,
                                          semaphore &sem) {
  umma2_abt<true>(d, a, b, sem);
}

// TMEM -> shared without a register tile: thread i of warp w takes TMEM lane
// 32 (w % 4) + i (accumulator row 32 (w % 4) + i), converts 32 columns at a
// time and writes them as 16-byte pieces into the swizzled shared tile.
// Ends with a proxy fence so a TMA store issued after the next barrier sees
// the data.
template <class TS, int SR_, int SC_, int M, int N>
__device__ __forceinline__ void store(st<TS, SR_, SC_> &dst, const tt<float, M, N> &src) {
  static_assert(sizeof(TS) == 2, "TMEM -> shared stores 16-bit tiles");
  static_assert(SR_ == M && SC_ <= N && SC_ % 32 == 0, "shared tile must cover the accumulator rows");
  using S = st<TS, SR_, SC_>;
  const int row = warpid() * 32 + static_cast<int>(lane_id());
  const u32 taddr = src.addr + (static_cast<u32>(warpid() * 32) << 16);
  tc_fence_after();  // the MMAs' completion was observed through a semaphore
#pragma unroll 1
  for (int c0 = 0; c0 < SC_; c0 += 32) {
    u32 v[32];
    tmem_ld_32x32b_x32(taddr + c0, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      u32 w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h)
        w[h] = pack2<TS>(__uint_as_float(v[8 * j + 2 * h]), __uint_as_float(v[8 * j + 2 * h + 1]));
      *reinterpret_cast<uint4 *>(dst.raw + S::offset(row, c0 + 8 * j)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  fence_proxy_async_smem();
}

// TMEM -> global at tile coordinate `at` (tiles of the accumulator's M x N):
// thread i of warp w writes accumulator row 32 (w % 4) + i, 16 bytes at a
// time where the row and columns are in bounds and aligned, element by
// element at a ragged edge.
template <class TG, int GR, int GC, int M, int N>
__device__ __forceinline__ void store(const gl<TG, GR, GC> &dst, const tt<float, M, N> &src, coord at) {
  static_assert(sizeof(TG) == 2 || sizeof(TG) == 4, "TMEM -> global stores 16- or 32-bit elements");
  static_assert(N % 32 == 0, "accumulator columns must be a multiple of 32");
  const long long row = (long long)at.r * M + warpid() * 32 + static_cast<int>(lane_id());
  const u32 taddr = src.addr + (static_cast<u32>(warpid() * 32) << 16);
  tc_fence_after();
#pragma unroll 1
  for (int c0 = 0; c0 < N; c0 += 32) {
    u32 v[32];
    tmem_ld_32x32b_x32(taddr + c0, v);
    tmem_wait_ld();
    if (row >= (long long)dst.rows) continue;
    const long long col0 = (long long)at.c * N + c0;
    TG *p = dst.ptr + row * (long long)dst.cols + col0;
    constexpr int PER = 16 / sizeof(TG);  // elements per 16-byte store
    const bool vec = col0 + 32 <= (long long)dst.cols && ((reinterpret_cast<unsigned long long>(p) & 15) == 0) &&
                     ((dst.cols * sizeof(TG)) % 16 == 0);
#pragma unroll
    for (int j = 0; j < 32 / PER; ++j) {
      if (vec) {
        u32 w[4];
        if constexpr (sizeof(TG) == 2) {
#pragma unroll
          for (int h = 0; h < 4; ++h)
            w[h] = pack2<TG>(__uint_as_float(v[8 * j + 2 * h]), __uint_as_float(v[8 * j + 2 * h + 1]));
        } else {
#pragma unroll
          for (int h = 0; h < 4; ++h) w[h] = v[4 * j + h];
        }
        st_global_v4(p + PER * j, w[0], w[1], w[2], w[3]);
      } else {
#pragma unroll
        for (int e = 0; e < PER; ++e)
          if (col0 + PER * j + e < (long long)dst.cols) p[PER * j + e] = from_f<TG>(__uint_as_float(v[PER * j + e]));
      }
    }
  }
}

// TMEM -> registers: this warp's 32 TMEM lanes (quadrant warpid) become the
// R = 32 rows of the register tile.  tcgen05.ld hands each thread one row;
// shuffles move the values into mma fragment positions.
template <class T, int R, int C, int M, int N>
__device__ __forceinline__ void load_async(rt<T, R, C, 0> &dst, const tt<float, M, N> &src) {
  static_assert(R == 32 && C <= N && C % 32 == 0, "load_async reads 32 TMEM lanes per warp");
  const int lane = lane_id();
  const int g = lane >> 2, t = lane & 3;
  const u32 taddr = src.addr + (static_cast<u32>(warpid() * 32) << 16);
  tc_fence_after();  // the MMAs' completion was observed through a semaphore
#pragma unroll 1
  for (int c0 = 0; c0 < C; c0 += 32) {
    u32 row[32];
    tmem_ld_32x32b_x32(taddr + c0, row);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)  // 16-column sub-tile within the 32-column chunk
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int src_lane = 16 * i + 8 * (q & 1) + g;
          float pair[2];
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            float v = 0.f;
#pragma unroll
            for (int tq = 0; tq < 4; ++tq) {
              const float x = __shfl_sync(0xffffffffu, __uint_as_float(row[16 * kb + 8 * (q >> 1) + 2 * tq + p]),
                                          src_lane);
              if (t == tq) v = x;
            }
            pair[p] = v;
          }
          auto &f = dst.t[i][c0 / 16 + kb];
          if constexpr (sizeof(T) == 4) {
            f.v[4 * (q >> 1) + 2 * (q & 1)] = pair[0];
            f.v[4 * (q >> 1) + 2 * (q & 1) + 1] = pair[1];
          } else {
            f.v[q] = pack2<T>(pair[0], pair[1]);
          }
        }
  }
}

}  // namespace warpgroup

// ------------------------------------------------------------------ TMA
namespace tma {

__device__ __forceinline__ void expect_bytes(semaphore &s, int bytes) {
  mbar_arrive_expect_tx(sem_addr(s), static_cast<u32>(bytes));
}

template <class T, int R, int C, class TG, int GR, int GC>
__device__ __forceinline__ void load_async(st<T, R, C> &dst, const gl<TG, GR, GC> &src, coord at,
                                           semaphore &sem) {
  using S = st<T, R, C>;
  static_assert(GR == R && GC == C, "TMA box (global tile shape) differs from the shared tile");
  static_assert(sizeof(T) == sizeof(TG), "shared and global element sizes differ");
  constexpr int BOX_R = R < 256 ? R : 256;
#pragma unroll
  for (int ch = 0; ch < S::NCH; ++ch)
#pragma unroll
    for (int r0 = 0; r0 < R; r0 += BOX_R)
      tma_load_2d(dst.base() + ch * S::CHB + r0 * S::ROWB, &src.tmap, sem_addr(sem),
                  at.c * C + ch * S::CC, at.r * R + r0);
}

template <class TG, int GR, int GC, class T, int R, int C>
__device__ __forceinline__ void store_async(const gl<TG, GR, GC> &dst, const st<T, R, C> &src, coord at) {
  using S = st<T, R, C>;
  static_assert(GR == R && GC == C, "TMA box (global tile shape) differs from the shared tile");
  constexpr int BOX_R = R < 256 ? R : 256;
  fence_proxy_async_smem();
#pragma unroll
  for (int ch = 0; ch < S::NCH; ++ch)
#pragma unroll
    for (int r0 = 0; r0 < R; r0 += BOX_R)
      tma_store_2d(&dst.tmap, src.base() + ch * S::CHB + r0 * S::ROWB, at.c * C + ch * S::CC,
                   at.r * R + r0);
  bulk_commit();
}

__device__ __forceinline__ void store_async_read_wait() { bulk_wait_read<0>(); }

// Loads into this CTA's shared tile whose bytes are counted on `sem` of
// cluster CTA `dst_cta` (the pair leader's copy, for a 2-CTA MMA).  The
// leader expects both CTAs' bytes (expect_bytes on its own semaphore).  No
// multicast: every CTA fetches its own tiles.
namespace pair {
__device__ __forceinline__ void expect_bytes(semaphore &s, int bytes) {
  mbar_arrive_expect_tx(sem_addr(s), static_cast<u32>(bytes));
}

template <class T, int R, int C, class TG, int GR, int GC>
__device__ __forceinline__ void load_async(st<T, R, C> &dst, const gl<TG, GR, GC> &src, coord at,
                                           semaphore &sem, int dst_cta) {
  using S = st<T, R, C>;
  static_assert(GR == R && GC == C, "TMA box (global tile shape) differs from the shared tile");
  static_assert(sizeof(T) == sizeof(TG), "shared and global element sizes differ");
  constexpr int BOX_R = R < 256 ? R : 256;
  const u32 bar = mapa_cluster(sem_addr(sem), static_cast<u32>(dst_cta));
#pragma unroll
  for (int ch = 0; ch < S::NCH; ++ch)
#pragma unroll
    for (int r0 = 0; r0 < R; r0 += BOX_R)
      tma_load_2d_pair(dst.base() + ch * S::CHB + r0 * S::ROWB, &src.tmap, bar, at.c * C + ch * S::CC,
                       at.r * R + r0);
}
}  // namespace pair

}  // namespace tma

}  // namespace tk
}  // namespace thork
