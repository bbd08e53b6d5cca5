// gemm_sm100.cuh — persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[GM, GN] = alpha * (A . B),  fp32 accumulation in tensor memory (TMEM),
//   bf16 output written row-major (or transposed, for the swap-AB skinny path).
//
// One CTA per SM loops over output tiles.  Warp roles (192 threads):
//   warp 0    TMA producer: fills a STAGES-deep ring of shared-memory stages.
//   warp 1    MMA issuer: allocates TMEM, issues tcgen05.mma (one thread) and
//             tcgen05.commit to release stages / publish accumulators.
//   warps 2-5 epilogue: tcgen05.ld TMEM -> registers -> bf16 -> 128-bit
//             global stores; TMEM lane quadrant = warp_id % 4.
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns), so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Operand layouts in shared memory are the 128-byte-swizzled canonical
// layouts that TMA (CU_TENSOR_MAP_SWIZZLE_128B) writes:
//   K-major operand (row-major A[M,K]):  BM rows x 128 bytes of K.
//   MN-major operand (row-major B[K,N]):  chunks of 128 bytes of N, each
//     BK rows deep; chunk c at c * BK * 128 bytes.
// BK is one 128-byte swizzle atom of K (64 bf16 or 128 e4m3 elements).
#pragma once
#include "sm100.cuh"

namespace thork {
namespace gemm {

using namespace thork::dev;

enum : int { KIND_BF16 = 0, KIND_E4M3 = 1 };

__host__ __device__ constexpr int ceil_pow2_cols(int n) {
  return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : n <= 256 ? 256 : 512;
}

template <int KIND_, int BN_, int STAGES_, bool A_MN_, bool B_MN_, bool TRANS_OUT_, int GROUP_M_ = 16>
struct Config {
  static constexpr int GROUP_M = GROUP_M_;  // tile rows per raster group
  static constexpr int KIND = KIND_;
  static constexpr int ELEM = KIND == KIND_BF16 ? 2 : 1;  // bytes per operand element
  static constexpr int BM = 128;                           // UMMA M (one CTA)
  static constexpr int BN = BN_;                           // UMMA N
  static constexpr int BK = 128 / ELEM;                    // one swizzle atom of K
  static constexpr int UMMA_K = 32 / ELEM;                 // K per tcgen05.mma
  static constexpr int CHUNK = 128 / ELEM;                 // MN elements per 128-byte chunk
  static constexpr int STAGES = STAGES_;
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr bool TRANS_OUT = TRANS_OUT_;
  static constexpr int A_BYTES = BM * BK * ELEM;
  static constexpr int B_BYTES = BN * BK * ELEM;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = ceil_pow2_cols(2 * BN);
  static constexpr int THREADS = 192;
  // stages + barriers (full/empty per stage, tmem full/empty x2, teardown) + tmem slot
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  // staged all-gather epilogue: each epilogue warp stages 32 rows x EPI_COLS
  // bf16 in shared memory so that its global stores are whole 128-byte lines
  static constexpr int EPI_COLS = 64;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES + ((BAR_BYTES + 127) & ~127);
  static constexpr int EPI_WARP_BYTES = 32 * EPI_COLS * 2;
  static constexpr int SMEM_BYTES_STAGED = 1024 + EPI_OFF + 4 * EPI_WARP_BYTES;
  static constexpr u32 IDESC =
      make_idesc(KIND == KIND_BF16 ? 1u : 0u, KIND == KIND_BF16 ? 1u : 0u, A_MN, B_MN, BM, BN);

  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N must be 16..256, multiple of 16");
  static_assert(!A_MN || BM % CHUNK == 0, "MN-major A needs BM multiple of the 128-byte chunk");
  static_assert(!B_MN || BN % CHUNK == 0, "MN-major B needs BN multiple of the 128-byte chunk");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

struct Params {
  void *out;      // bf16 output
  int GM, GN, GK; // MMA-space extents
  int ldo;        // output leading dimension (elements)
  int out_rows;   // rows of the output matrix (bounds for stores)
  int out_cols;   // cols of the output matrix
  float alpha;
  u32 *status;
  // fused all-gather: the same output rows are also stored at the same
  // offsets of up to 7 peer GPUs' buffers (P2P stores over NVLink)
  void *peer[7];
  int npeer;
  u32 *tile_flags;  // fused all-gather: completion counts per 128 x 64 unit of C
  u32 epoch;        // this call's number: a unit is done once its count is 4 * epoch
};

// Modes of the fused all-gather inside gemm_kernel: staged peer stores, push
// warps, or one multicast (NVLS) store per line through `out`, the
// multicast view of the gathered C.
enum : int { AG_NONE = 0, AG_STAGED = 1, AG_PUSH = 2, AG_MULTIMEM = 3 };

template <class Cfg, int AG>
constexpr int gemm_smem_bytes() {
  return (AG == AG_STAGED || AG == AG_MULTIMEM || (Cfg::TRANS_OUT && Cfg::BN % 64 == 0))
             ? Cfg::SMEM_BYTES_STAGED
             : Cfg::SMEM_BYTES;
}
template <class Cfg, int AG>
constexpr int gemm_threads() {
  return AG == AG_PUSH ? Cfg::THREADS + 128 : Cfg::THREADS;
}

// Output-tile order: groups of GROUP_M tile-rows walked column by column, so
// the ~SM-count tiles in flight share A rows and B columns in L2.
template <int GROUP_M>
__device__ __forceinline__ void tile_coords(int t, int ntm, int ntn, int &tm, int &tn) {
  const int per_group = GROUP_M * ntn;
  const int g = t / per_group;
  const int first = g * GROUP_M;
  const int gsize = min(ntm - first, GROUP_M);
  const int r = t - g * per_group;
  tm = first + r % gsize;
  tn = r / gsize;
}

template <class Cfg>
__device__ __forceinline__ void load_operand(u32 dst, const TensorMap *tm, u32 bar, bool mn_major,
                                             int extent, int mn0, int k0) {
  if (mn_major) {
    // global tensor is [K rows, MN cols]; one box per 128-byte MN chunk
#pragma unroll
    for (int c = 0; c < extent / Cfg::CHUNK; ++c)
      tma_load_2d(dst + c * Cfg::BK * 128, tm, bar, mn0 + c * Cfg::CHUNK, k0);
  } else {
    // global tensor is [MN rows, K cols]; one box of extent rows x 128 bytes
    tma_load_2d(dst, tm, bar, k0, mn0);
  }
}

template <class Cfg>
__device__ __forceinline__ u64 operand_desc(u32 base, bool mn_major, int kstep) {
  if (mn_major) return smem_desc_sw128(base + kstep * Cfg::UMMA_K * 128, Cfg::BK * 128, 1024);
  return smem_desc_sw128(base + kstep * 32, 16, 1024);
}

__device__ __forceinline__ void st_global_b16(void *p, u32 v) {
  asm volatile("st.global.b16 [%0], %1;" ::"l"(p), "h"(static_cast<unsigned short>(v & 0xFFFFu))
               : "memory");
}

// Epilogue for one accumulator row slice: TMEM lane row_mma of the tile,
// columns [col0, col0 + BN) -> bf16.  Non-transposed output writes row
// `row_mma` of D with 16-byte vector stores; transposed output (swap-AB
// skinny path) writes column `row_mma` of D^T.
template <class Cfg>
__device__ __forceinline__ void bf16_store_tile(const Params &p, u32 t_row, int row_mma, int col0) {
  constexpr int CH = (Cfg::BN % 32 == 0) ? 32 : 16;
  unsigned short *out = static_cast<unsigned short *>(p.out);
#pragma unroll 1
  for (int c0 = 0; c0 < Cfg::BN; c0 += CH) {
    u32 r[CH];
    if constexpr (CH == 32)
      tmem_ld_32x32b_x32(t_row + c0, r);
    else
      tmem_ld_32x32b_x16(t_row + c0, r);
    tmem_wait_ld();
    if (!Cfg::TRANS_OUT) {
      if (row_mma < p.out_rows) {
        unsigned short *dst = out + static_cast<long long>(row_mma) * p.ldo + col0 + c0;
#pragma unroll
        for (int j = 0; j < CH / 8; ++j) {
          if (col0 + c0 + 8 * j < p.out_cols) {
            u32 w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h)
              w[h] = pack_bf16x2(__uint_as_float(r[8 * j + 2 * h]) * p.alpha,
                                 __uint_as_float(r[8 * j + 2 * h + 1]) * p.alpha);
            st_global_v4(dst + 8 * j, w[0], w[1], w[2], w[3]);
          }
        }
      }
    } else {
      if (row_mma < p.out_cols) {
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int orow = col0 + c0 + i;
          if (orow < p.out_rows)
            st_global_b16(out + static_cast<long long>(orow) * p.ldo + row_mma,
                          pack_bf16x2(__uint_as_float(r[i]) * p.alpha, 0.0f));
        }
      }
    }
  }
}

// Named barrier 1 over the 128 epilogue threads.
__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Same barrier, returning whether any of the 128 threads passed `v` = true,
// so all epilogue warps take the same branch.
__device__ __forceinline__ bool epi_vote_any(bool v) {
  u32 r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, 1, 128, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}

// Transposed (swap-AB) epilogue of one tile, shared by the four epilogue
// warps: TMEM lane n holds W column n0 + n, and its BN accumulator columns
// are the tile's rows of Y.  Per 64-row slice, the two lanes of a pair swap
// one value (shfl) so that each thread writes two adjacent columns of one
// row as one 4-byte word into a [64][128] bf16 staging slice (256-byte
// rows; on odd rows the 16-byte chunks are XOR 4, so a warp's even and odd
// lanes write different banks).  After a barrier of the 128 epilogue
// threads each warp stores 16 whole rows of the slice, two 256-byte row
// segments per instruction, instead of one 64-byte piece of a row per
// instruction.
template <class Cfg>
__device__ __forceinline__ void bf16_store_tile_trans(const Params &p, u32 t_lane, int n0, int m0,
                                                      unsigned char *stg, int q, int lane) {
  static_assert(Cfg::TRANS_OUT && Cfg::BM == 128 && Cfg::BN % 64 == 0, "transposed staging layout");
  static_assert(4 * Cfg::EPI_WARP_BYTES >= 64 * 256, "staging slice is 64 rows of 256 bytes");
  unsigned short *out = static_cast<unsigned short *>(p.out);
  const bool odd = lane & 1;
  const int nw = q * 32 + (lane & ~1);  // first of the two columns this thread writes
  const int wchunk = nw >> 3;           // its 16-byte chunk of the 256-byte row
  const int wbyte = (nw & 7) * 2;       // and the byte within the chunk
#pragma unroll 1
  for (int c0 = 0; c0 < Cfg::BN; c0 += 64) {
#pragma unroll
    for (int h = 0; h < 64; h += 32) {
      u32 r[32];
      tmem_ld_32x32b_x32(t_lane + c0 + h, r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        // even lane: row i, columns (own, partner); odd lane: row i + 1, (partner, own)
        const u32 got = __shfl_xor_sync(0xffffffffu, odd ? r[i] : r[i + 1], 1);
        const float lo = __uint_as_float(odd ? got : r[i]);
        const float hi = __uint_as_float(odd ? r[i + 1] : got);
        const int row = h + i + (odd ? 1 : 0);
        *reinterpret_cast<u32 *>(stg + row * 256 + ((wchunk ^ ((row & 1) << 2)) * 16) + wbyte) =
            pack_bf16x2(lo * p.alpha, hi * p.alpha);
      }
    }
    epi_bar();  // the slice is complete
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int row = q * 16 + 2 * j + (lane >> 4);
      const int chunk = lane & 15;
      const uint4 v =
          *reinterpret_cast<const uint4 *>(stg + row * 256 + ((chunk ^ ((row & 1) << 2)) * 16));
      const int orow = m0 + c0 + row, ocol = n0 + chunk * 8;
      // N is a multiple of 8, so a 16-byte chunk is wholly in or out
      if (orow < p.out_rows && ocol < p.out_cols)
        st_global_v4(out + static_cast<long long>(orow) * p.ldo + ocol, v.x, v.y, v.z, v.w);
    }
    epi_bar();  // every warp has read the slice before the next one is written
  }
}

// Epilogue of the fused all-gather for one warp's 32 accumulator rows
// (TMEM lanes of t_row, output rows row0..row0+31, columns col0..col0+BN):
// each EPI_COLS-wide slice goes TMEM -> registers -> bf16 -> this warp's
// staging buffer (row = lane, 16-byte chunks XOR-swizzled by row so both
// directions are bank-conflict free), then back out with lanes covering
// consecutive 16-byte chunks of a row: every warp store writes whole
// 128-byte lines, to this GPU's C and to each peer's C at the same offset.
// MC: `p.out` is a multicast view; each line is stored once with
// multimem.st and the NVSwitch delivers it to every GPU of the group.
template <class Cfg, bool MC = false>
__device__ __forceinline__ void bf16_store_tile_peers(const Params &p, u32 t_row, int row0,
                                                      int col0, unsigned char *stg, int lane) {
  constexpr int EC = Cfg::EPI_COLS;
  constexpr int RB = EC * 2;     // staged bytes per row
  constexpr int CPR = RB / 16;   // 16-byte chunks per row
  constexpr int RPI = 32 / CPR;  // rows per warp store instruction
  static_assert(CPR == 8 && Cfg::BN % EC == 0, "staging assumes 128-byte rows");
  unsigned short *out = static_cast<unsigned short *>(p.out);
#pragma unroll 1
  for (int c0 = 0; c0 < Cfg::BN; c0 += EC) {
#pragma unroll
    for (int h = 0; h < EC; h += 32) {
      u32 r[32];
      tmem_ld_32x32b_x32(t_row + c0 + h, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        u32 w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          w[q] = pack_bf16x2(__uint_as_float(r[8 * j + 2 * q]) * p.alpha,
                             __uint_as_float(r[8 * j + 2 * q + 1]) * p.alpha);
        const int chunk = h / 8 + j;
        *reinterpret_cast<uint4 *>(stg + lane * RB + ((chunk ^ (lane & (CPR - 1))) * 16)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncwarp();
#pragma unroll 2
    for (int it = 0; it < 32 / RPI; ++it) {
      const int r = it * RPI + lane / CPR;
      const int chunk = lane % CPR;
      const uint4 v = *reinterpret_cast<const uint4 *>(stg + r * RB + ((chunk ^ (r & (CPR - 1))) * 16));
      const int row = row0 + r, col = col0 + c0 + chunk * 8;
      if (row < p.out_rows && col < p.out_cols) {
        const long long off = static_cast<long long>(row) * p.ldo + col;
        if constexpr (MC) {
          multimem_st_v4(out + off, v.x, v.y, v.z, v.w);
        } else {
          st_global_v4(out + off, v.x, v.y, v.z, v.w);
#pragma unroll
          for (int g = 0; g < 7; ++g)  // constant indices keep p.peer in parameter space
            if (g < p.npeer)
              st_global_v4(static_cast<unsigned short *>(p.peer[g]) + off, v.x, v.y, v.z, v.w);
        }
      }
    }
    __syncwarp();
  }
}

// Push warps of the AG_PUSH all-gather (warps 6..9).  The (tile, peer)
// pushes of the whole grid, in tile order, are dealt round-robin to the
// CTAs, so every SM carries an equal share of the NVLink traffic whichever
// SM computed the tile.  A push waits (bounded) until the four epilogue
// warps of the tile's CTA have stored it to this GPU's C (the count of its
// first 128 x 64 unit reaches 4 * epoch), reads it back from L2 and stores it to the peer's C
// at the same offset, one 512-byte row segment per warp instruction.  The
// epilogue never waits for the pushes.  All CTAs are co-resident (a
// cooperative launch), so a wait on another CTA's tile always ends.
template <class Cfg>
__device__ __forceinline__ void push_tasks(const Params &p, int ntm, int ntn, int ntiles,
                                           volatile u32 *abort_flag, int pw, int lane) {
  constexpr int LPR = Cfg::BN / 8;  // lanes per tile row (16 bytes each)
  constexpr int RPI = 32 / LPR;     // tile rows per warp instruction
  static_assert(LPR * RPI == 32 && Cfg::BM % (4 * RPI * 8) == 0, "push layout");
  const unsigned short *out = static_cast<const unsigned short *>(p.out);
  const int ntasks = ntiles * p.npeer;
  const u32 need = 4u * p.epoch;
  for (int j = blockIdx.x; j < ntasks; j += gridDim.x) {
    const int t = j / p.npeer, g = j - t * p.npeer;
    int tm, tn;
    tile_coords<Cfg::GROUP_M>(t, ntm, ntn, tm, tn);
    const u32 *flag = p.tile_flags + tm * ((p.GN + 63) / 64) + tn * (Cfg::BN / 64);
    int ok = 1;
    if (lane == 0) {
      const u64 t0 = globaltimer();
      for (;;) {
        u32 v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (static_cast<int>(v - need) >= 0) break;
        if (*abort_flag) { ok = 0; break; }
        if (globaltimer() - t0 > THORK_WAIT_TIMEOUT_NS) {
          report_status(p.status, STATUS_WAIT_TIMEOUT, 7);
          *abort_flag = 1;
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    const int col = tn * Cfg::BN + (lane % LPR) * 8;
    // N is a multiple of 8, so a lane's 16-byte chunk is wholly in or out
    const int row_end = col < p.out_cols ? min(tm * Cfg::BM + Cfg::BM, p.out_rows) : 0;
    unsigned short *dst = nullptr;
#pragma unroll
    for (int q = 0; q < 7; ++q)  // constant indices keep p.peer in parameter space
      if (q == g) dst = static_cast<unsigned short *>(p.peer[q]);
    // warp pw takes row groups pw, pw + 4, ... of RPI consecutive rows
    const int row_first = tm * Cfg::BM + pw * RPI + lane / LPR;
#pragma unroll 1
    for (int r0 = row_first; r0 < tm * Cfg::BM + Cfg::BM; r0 += 32 * RPI) {
      uint4 v[8];  // eight row groups in flight
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = r0 + 4 * RPI * i;
        if (row < row_end) {
          const unsigned short *src = out + static_cast<long long>(row) * p.ldo + col;
          asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(v[i].x), "=r"(v[i].y), "=r"(v[i].z), "=r"(v[i].w)
                       : "l"(src));
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = r0 + 4 * RPI * i;
        if (row < row_end)
          st_global_v4(dst + static_cast<long long>(row) * p.ldo + col, v[i].x, v[i].y, v[i].z,
                       v[i].w);
      }
    }
  }
  // these stores are ordered before anything a later kernel signals to the
  // peers (the fused all-gather's flag barrier)
  __threadfence_system();
}

template <class Cfg, int AG = AG_NONE>
__global__ void __launch_bounds__(gemm_threads<Cfg, AG>(), 1)
    gemm_kernel(const __grid_constant__ TensorMap tmap_a, const __grid_constant__ TensorMap tmap_b,
                const Params p) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  const u32 raw = smem_u32(smem_raw);
  const u32 base = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (base - raw);
  const u32 stage0 = base;
  const u32 bars = base + Cfg::STAGES * Cfg::STAGE_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (Cfg::STAGES + s); };
  auto tfull_bar = [&](int a) { return bars + 8u * (2 * Cfg::STAGES + a); };
  auto tempty_bar = [&](int a) { return bars + 8u * (2 * Cfg::STAGES + 2 + a); };
  const u32 drain_bar = bars + 8u * (2 * Cfg::STAGES + 4);
  u32 *tmem_slot = reinterpret_cast<u32 *>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + (2 * Cfg::STAGES + 5) * 8);
  volatile u32 *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  const int ntm = (p.GM + Cfg::BM - 1) / Cfg::BM;
  const int ntn = (p.GN + Cfg::BN - 1) / Cfg::BN;
  const int ntiles = ntm * ntn;
  const int nkb = (p.GK + Cfg::BK - 1) / Cfg::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const u32 tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel of the stream is complete from here on

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      u32 ph = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x) {
        int tm, tn;
        tile_coords<Cfg::GROUP_M>(t, ntm, ntn, tm, tn);
        const int m0 = tm * Cfg::BM, n0 = tn * Cfg::BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(empty_bar(s), ph ^ 1u, p.status, 1)) {
            *abort_flag = 1;
            break;
          }
          const u32 sa = stage0 + s * Cfg::STAGE_BYTES;
          const u32 sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(full_bar(s), Cfg::STAGE_BYTES);
          load_operand<Cfg>(sa, &tmap_a, full_bar(s), Cfg::A_MN, Cfg::BM, m0, kb * Cfg::BK);
          load_operand<Cfg>(sb, &tmap_b, full_bar(s), Cfg::B_MN, Cfg::BN, n0, kb * Cfg::BK);
          if (++s == Cfg::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Drain: wait until every issued load has landed before the CTA may exit.
      // The stage about to be reused was released by the MMA warp, so waiting
      // on the empty barriers of the last STAGES slots covers every copy.
      for (int i = 0; i < Cfg::STAGES; ++i) {
        if (!mbar_wait(empty_bar(s), ph ^ 1u, p.status, 2)) break;
        if (++s == Cfg::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    // The whole loop runs in lane 0: a warp-wide reconvergence (shuffle,
    // __syncwarp) per k-block delayed each stage's MMAs enough to idle the
    // tensor pipe (measured 8192^3 bf16: 1336 -> 1420 TFLOP/s without it).
    if (lane == 0) {
      int s = 0;
      u32 ph = 0;
      int it = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const u32 acc_ph = (it >> 1) & 1;
        const u32 d_tmem = tmem_base + acc * Cfg::BN;
        if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, p.status, 3)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(full_bar(s), ph, p.status, 4)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const u32 sa = stage0 + s * Cfg::STAGE_BYTES;
          const u32 sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
            const u64 ad = operand_desc<Cfg>(sa, Cfg::A_MN, k);
            const u64 bd = operand_desc<Cfg>(sb, Cfg::B_MN, k);
            const u32 accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (Cfg::KIND == KIND_BF16)
              mma_f16_ss(d_tmem, ad, bd, Cfg::IDESC, accum);
            else
              mma_f8f6f4_ss(d_tmem, ad, bd, Cfg::IDESC, accum);
          }
          tc_commit(empty_bar(s));  // stage s free once these MMAs have read it
          if (++s == Cfg::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok || *abort_flag) break;
        tc_commit(tfull_bar(acc));  // accumulator ready for the epilogue
      }
      // Teardown: make sure every MMA this thread issued has completed before
      // TMEM is released.
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.status, 5);
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ------------------------------------------------ NVLink push (warps 6..9)
    if constexpr (AG == AG_PUSH) push_tasks<Cfg>(p, ntm, ntn, ntiles, abort_flag, warp - 6, lane);
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    // the transposed store synchronises the four epilogue warps, so they
    // leave the tile loop together: the abort decision is a vote of all 128
    constexpr bool kVote = Cfg::TRANS_OUT && Cfg::BN % 64 == 0 && AG == AG_NONE;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      if (!kVote && *abort_flag) break;
      int tm, tn;
      tile_coords<Cfg::GROUP_M>(t, ntm, ntn, tm, tn);
      const int acc = it & 1;
      const u32 acc_ph = (it >> 1) & 1;
      bool ok = kVote ? !*abort_flag : true;
      if (lane == 0 && ok) ok = mbar_wait(tfull_bar(acc), acc_ph, p.status, 6);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if constexpr (kVote) ok = !epi_vote_any(!ok);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row_mma = tm * Cfg::BM + q * 32 + lane;  // MMA-space row owned by this thread
      const u32 t_row = tmem_base + ((u32)(q * 32) << 16) + acc * Cfg::BN;
      if constexpr (AG == AG_STAGED || AG == AG_MULTIMEM)
        bf16_store_tile_peers<Cfg, AG == AG_MULTIMEM>(p, t_row, tm * Cfg::BM + q * 32, tn * Cfg::BN,
                                                      smem + Cfg::EPI_OFF + q * Cfg::EPI_WARP_BYTES,
                                                      lane);
      else if constexpr (Cfg::TRANS_OUT && Cfg::BN % 64 == 0)
        bf16_store_tile_trans<Cfg>(p, t_row, tm * Cfg::BM, tn * Cfg::BN, smem + Cfg::EPI_OFF, q, lane);
      else
        bf16_store_tile<Cfg>(p, t_row, row_mma, tn * Cfg::BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      if constexpr (AG != AG_NONE) {
        // the warp's rows of this tile are in C: publish them to the push
        // warps (counted in both modes, so epochs stay in step when calls
        // on the same flags mix the variants)
        if (lane == 0 && p.tile_flags) {
          __threadfence();
          // one count per 128 x 64 unit of C, whatever the tile width, so
          // calls with different tile widths keep the same epochs
          const int upr = (p.GN + 63) / 64;
          const int u0 = tn * (Cfg::BN / 64);
#pragma unroll
          for (int u = 0; u < (Cfg::BN + 63) / 64; ++u)
            if (u0 + u < upr)
              asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.tile_flags + tm * upr + u0 + u)
                           : "memory");
        }
      }
    }
    // staged peer stores (or multicast stores) are ordered before anything a
    // later kernel signals to the peers (the fused all-gather's flag barrier)
    if constexpr (AG == AG_MULTIMEM) fence_proxy_alias();
    if constexpr (AG == AG_STAGED || AG == AG_MULTIMEM) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<1>(tmem_base, Cfg::TMEM_COLS);
}

// ===========================================================================
// Stream-K decode GEMM (swap-AB skinny shapes).  The (tile, k-block) units of
// the whole problem are split into gridDim.x contiguous, equal ranges, so
// every SM streams the same share of W however few output tiles there are.
// A tile covered by one CTA is stored directly; a tile split across CTAs has
// each CTA write its fp32 partial to a workspace slot, and the CTA that
// completes the tile's arrival counter sums the slots in slot order
// (deterministic), writes the bf16 output and resets the counter to zero.
// ===========================================================================
struct SkParams {
  Params p;
  float *partial;       // [grid][2][BN/4][BM] float4: a CTA's first and last segment
  unsigned *counters;   // [tiles], zero between launches
  int base, extra;      // CTA c owns base + (c < extra) stream-K units
  int dp_tiles;         // leading tiles done whole, CTA c taking c, c + grid, ...
  int w_static;         // A is written by no earlier launch: prefetch it before the dependency wait
};



// A CTA's unit range is contiguous, so only its first and last segments can
// be part of a tile; slot 0 holds the first, slot 1 the last.
__device__ __forceinline__ int sk_slot(int c, int tile, int nkb, int base, int extra) {
  return (c * base + min(c, extra)) / nkb == tile ? 0 : 1;
}

__device__ __forceinline__ int sk_first_unit(int c, int base, int extra) {
  return c * base + min(c, extra);
}

__device__ __forceinline__ int sk_cta_of_unit(int u, int base, int extra) {
  const int big = extra * (base + 1);
  return u < big ? u / (base + 1) : extra + (u - big) / base;
}

// Next tile segment [k0, k1) of this CTA's unit range; false when done.
__device__ __forceinline__ bool sk_next(int &u, int end, int nkb, int &tile, int &k0, int &k1) {
  if (u >= end) return false;
  tile = u / nkb;
  k0 = u - tile * nkb;
  const int e = min(end, (tile + 1) * nkb);
  k1 = k0 + (e - u);
  u = e;
  return true;
}

// The CTA's work in order: its whole data-parallel tiles, then the
// segments of its stream-K unit range (units count from tile dp_tiles on).
struct SkIter {
  int t_dp, u;
  __device__ __forceinline__ bool next(const SkParams &sp, int u_end, int nkb, int &tile, int &k0,
                                       int &k1) {
    if (t_dp < sp.dp_tiles) {
      tile = t_dp;
      k0 = 0;
      k1 = nkb;
      t_dp += gridDim.x;
      return true;
    }
    if (!sk_next(u, u_end, nkb, tile, k0, k1)) return false;
    tile += sp.dp_tiles;
    return true;
  }
};

template <class Cfg>
__global__ void __launch_bounds__(192, 1)
    sk_kernel(const __grid_constant__ TensorMap tmap_a, const __grid_constant__ TensorMap tmap_b,
              const SkParams sp) {
  pdl_launch_dependents();
  const Params &p = sp.p;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const u32 raw = smem_u32(smem_raw);
  const u32 base = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (base - raw);
  const u32 stage0 = base;
  const u32 bars = base + Cfg::STAGES * Cfg::STAGE_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (Cfg::STAGES + s); };
  auto tfull_bar = [&](int a) { return bars + 8u * (2 * Cfg::STAGES + a); };
  auto tempty_bar = [&](int a) { return bars + 8u * (2 * Cfg::STAGES + 2 + a); };
  const u32 drain_bar = bars + 8u * (2 * Cfg::STAGES + 4);
  u32 *tmem_slot = reinterpret_cast<u32 *>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + (2 * Cfg::STAGES + 5) * 8);
  volatile u32 *abort_flag = tmem_slot + 1;
  volatile u32 *last_flag = tmem_slot + 2;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int nkb = (p.GK + Cfg::BK - 1) / Cfg::BK;
  const int ntm = (p.GM + Cfg::BM - 1) / Cfg::BM;
  const int ntn = (p.GN + Cfg::BN - 1) / Cfg::BN;
  const int u_begin = sk_first_unit(blockIdx.x, sp.base, sp.extra);
  const int u_end = sk_first_unit(blockIdx.x + 1, sp.base, sp.extra);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const u32 tmem_base = *tmem_slot;
  // the previous kernel of the stream is complete from pdl_wait() on; the
  // producer may first fetch W for its opening stages when W is static
  if (warp != 0) pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // Static W: the opening STAGES stages get their W tiles while the
      // previous kernel still runs; X follows after the dependency wait.
      int npre = 0;
      if (sp.w_static) {
        SkIter pre{static_cast<int>(blockIdx.x), u_begin};
        int tile, k0, k1;
        while (npre < Cfg::STAGES && pre.next(sp, u_end, nkb, tile, k0, k1)) {
          int tm, tn;
          tile_coords<Cfg::GROUP_M>(tile, ntm, ntn, tm, tn);
          for (int kb = k0; kb < k1 && npre < Cfg::STAGES; ++kb, ++npre) {
            const u32 sa = stage0 + npre * Cfg::STAGE_BYTES;
            mbar_arrive_expect_tx(full_bar(npre), Cfg::STAGE_BYTES);
            load_operand<Cfg>(sa, &tmap_a, full_bar(npre), Cfg::A_MN, Cfg::BM, tm * Cfg::BM,
                              kb * Cfg::BK);
          }
        }
      }
      pdl_wait();
      int s = 0;
      u32 ph = 0;
      int issued = 0;
      SkIter itr{static_cast<int>(blockIdx.x), u_begin};
      int tile, k0, k1;
      while (!*abort_flag && itr.next(sp, u_end, nkb, tile, k0, k1)) {
        int tm, tn;
        tile_coords<Cfg::GROUP_M>(tile, ntm, ntn, tm, tn);
        for (int kb = k0; kb < k1; ++kb, ++issued) {
          const u32 sa = stage0 + s * Cfg::STAGE_BYTES;
          const u32 sb = sa + Cfg::A_BYTES;
          if (issued >= npre) {
            if (!mbar_wait(empty_bar(s), ph ^ 1u, p.status, 0x21)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(full_bar(s), Cfg::STAGE_BYTES);
            load_operand<Cfg>(sa, &tmap_a, full_bar(s), Cfg::A_MN, Cfg::BM, tm * Cfg::BM, kb * Cfg::BK);
          }
          load_operand<Cfg>(sb, &tmap_b, full_bar(s), Cfg::B_MN, Cfg::BN, tn * Cfg::BN, kb * Cfg::BK);
          if (++s == Cfg::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      for (int i = 0; i < Cfg::STAGES; ++i) {
        if (!mbar_wait(empty_bar(s), ph ^ 1u, p.status, 0x22)) break;
        if (++s == Cfg::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      u32 ph = 0;
      int it = 0;
      SkIter itr{static_cast<int>(blockIdx.x), u_begin};
      int tile, k0, k1;
      while (!*abort_flag && itr.next(sp, u_end, nkb, tile, k0, k1)) {
        const int acc = it & 1;
        const u32 acc_ph = (it >> 1) & 1;
        const u32 d_tmem = tmem_base + acc * Cfg::BN;
        if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, p.status, 0x23)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int kb = k0; kb < k1; ++kb) {
          if (!mbar_wait(full_bar(s), ph, p.status, 0x24)) {
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const u32 sa = stage0 + s * Cfg::STAGE_BYTES;
          const u32 sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
            const u64 ad = operand_desc<Cfg>(sa, Cfg::A_MN, k), bd = operand_desc<Cfg>(sb, Cfg::B_MN, k);
            const u32 accum = (kb > k0 || k > 0) ? 1u : 0u;
            if constexpr (Cfg::KIND == KIND_BF16)
              mma_f16_ss(d_tmem, ad, bd, Cfg::IDESC, accum);
            else
              mma_f8f6f4_ss(d_tmem, ad, bd, Cfg::IDESC, accum);
          }
          tc_commit(empty_bar(s));
          if (++s == Cfg::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (*abort_flag) break;
        tc_commit(tfull_bar(acc));
        ++it;
      }
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.status, 0x25);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;  // TMEM lane: MMA-space row within the tile
    unsigned short *out = static_cast<unsigned short *>(p.out);
    int it = 0;
    SkIter itr{static_cast<int>(blockIdx.x), u_begin};
    int tile, k0, k1;
    while (itr.next(sp, u_end, nkb, tile, k0, k1)) {
      const int acc = it & 1;
      const u32 acc_ph = (it >> 1) & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(tfull_bar(acc), acc_ph, p.status, 0x26);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      // one decision for all four warps: the partial path below has barriers
      if (epi_vote_any(!ok || *abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const u32 t_row = tmem_base + ((u32)(q * 32) << 16) + acc * Cfg::BN;
      int tm, tn;
      tile_coords<Cfg::GROUP_M>(tile, ntm, ntn, tm, tn);
      // MMA-space row: the output column n (swap-AB) or the output row m
      const int n = tm * Cfg::BM + row;
      if (k0 == 0 && k1 == nkb) {
        bf16_store_tile<Cfg>(p, t_row, n, tn * Cfg::BN);
      } else {
        const int lt = tile - sp.dp_tiles;  // tile index within the stream-K units
        const int first = sk_cta_of_unit(lt * nkb, sp.base, sp.extra);
        const int nseg = sk_cta_of_unit((lt + 1) * nkb - 1, sp.base, sp.extra) - first + 1;
        constexpr int V = Cfg::BN / 4;
        constexpr int VC = V < 8 ? V : 8;  // float4 per chunk: 16 or 32 columns
        constexpr int CH = 4 * VC;
        if (k0 != 0) {
          // not the tile's head segment: this CTA's fp32 partial goes to its
          // slot ([BN/4][BM] float4: a warp's 32 rows of one 4-column chunk
          // are 512 contiguous bytes), then it counts itself in
          const int slot = sk_slot(blockIdx.x, lt, nkb, sp.base, sp.extra);
          float4 *mine = reinterpret_cast<float4 *>(sp.partial) +
                         (static_cast<long long>(blockIdx.x) * 2 + slot) * V * Cfg::BM + row;
#pragma unroll 1
          for (int c0 = 0; c0 < Cfg::BN; c0 += CH) {
            u32 r[CH];
            if constexpr (CH == 32)
              tmem_ld_32x32b_x32(t_row + c0, r);
            else
              tmem_ld_32x32b_x16(t_row + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < CH / 4; ++j)
              mine[(c0 / 4 + j) * Cfg::BM] =
                  make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                              __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          }
          __threadfence();
          epi_bar();
          if (threadIdx.x == 64) atomicAdd(sp.counters + tile, 1u);
        } else {
          // the head segment (k-blocks from 0) is the last range its CTA
          // works on, so it sums the tile: once the other nseg - 1 segments
          // have counted themselves in (bounded wait), its own accumulator
          // from TMEM plus their slots in CTA order -- the order every split
          // tile has always been summed in
          if (threadIdx.x == 64) {
            u32 ok = 1;
            const u64 t0 = globaltimer();
            for (;;) {
              unsigned v;
              asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(sp.counters + tile)
                           : "memory");
              if (v >= static_cast<unsigned>(nseg - 1)) break;
              if (*abort_flag || globaltimer() - t0 > THORK_WAIT_TIMEOUT_NS) {
                if (!*abort_flag) report_status(p.status, STATUS_WAIT_TIMEOUT, 0x27);
                ok = 0;
                break;
              }
            }
            *last_flag = ok;
          }
          epi_bar();
          if (!*last_flag) {
            *abort_flag = 1;
          } else {
            __threadfence();
#pragma unroll 1
            for (int c = 0; c < V; c += VC) {
              u32 r[CH];
              if constexpr (CH == 32)
                tmem_ld_32x32b_x32(t_row + 4 * c, r);
              else
                tmem_ld_32x32b_x16(t_row + 4 * c, r);
              tmem_wait_ld();
              float4 sum[VC];
#pragma unroll
              for (int j = 0; j < VC; ++j)
                sum[j] = make_float4(0.f + __uint_as_float(r[4 * j]), 0.f + __uint_as_float(r[4 * j + 1]),
                                     0.f + __uint_as_float(r[4 * j + 2]),
                                     0.f + __uint_as_float(r[4 * j + 3]));
              for (int sgi = 1; sgi < nseg; ++sgi) {
                const int cta = first + sgi;
                const float4 *slot4 =
                    reinterpret_cast<const float4 *>(sp.partial) +
                    (static_cast<long long>(cta) * 2 + sk_slot(cta, lt, nkb, sp.base, sp.extra)) * V * Cfg::BM +
                    row;
                float4 v[VC];
#pragma unroll
                for (int j = 0; j < VC; ++j) v[j] = __ldcg(slot4 + (c + j) * Cfg::BM);
#pragma unroll
                for (int j = 0; j < VC; ++j) {
                  sum[j].x += v[j].x;
                  sum[j].y += v[j].y;
                  sum[j].z += v[j].z;
                  sum[j].w += v[j].w;
                }
              }
              const float *f = reinterpret_cast<const float *>(sum);
              if constexpr (Cfg::TRANS_OUT) {
                if (n < p.out_cols) {
#pragma unroll
                  for (int m = 0; m < 4 * VC; ++m)
                    if (4 * c + m < p.out_rows)
                      st_global_b16(out + static_cast<long long>(4 * c + m) * p.ldo + n,
                                    pack_bf16x2(f[m] * p.alpha, 0.0f));
                }
              } else if (n < p.out_rows) {
                // row n of C, columns tn*BN + 4c .. + 4 VC, 16-byte stores
#pragma unroll
                for (int g = 0; g < VC / 2; ++g) {
                  const int col = tn * Cfg::BN + 4 * c + 8 * g;
                  if (col < p.out_cols) {
                    u32 w[4];
#pragma unroll
                    for (int h = 0; h < 4; ++h)
                      w[h] = pack_bf16x2(f[8 * g + 2 * h] * p.alpha, f[8 * g + 2 * h + 1] * p.alpha);
                    st_global_v4(out + static_cast<long long>(n) * p.ldo + col, w[0], w[1], w[2], w[3]);
                  }
                }
              }
            }
            if (threadIdx.x == 64) sp.counters[tile] = 0u;  // ready for the next launch
          }
        }
        epi_bar();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      ++it;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<1>(tmem_base, Cfg::TMEM_COLS);
}

// ===========================================================================
// 2-CTA variant: a cluster of two CTAs computes a 256 x BN tile with
// tcgen05.mma.cta_group::2 (M = 256).  CTA rank r loads rows [128r, 128r+128)
// of the A tile and columns [BN/2*r, BN/2*(r+1)) of the B tile into its own
// shared memory (no multicast); both CTAs' TMA loads complete on the leader's
// (rank 0) full barrier.  The leader's MMA thread reads both CTAs' operands
// and writes each CTA's 128 accumulator rows into that CTA's TMEM; its
// commits release the stage / publish the accumulator in both CTAs.
// ===========================================================================
template <int KIND_, int BN_, int STAGES_, int GROUP_M_ = 16>
struct Config2 {
  static constexpr int GROUP_M = GROUP_M_;  // pair-tile rows per raster group
  static constexpr int KIND = KIND_;
  static constexpr int ELEM = KIND == KIND_BF16 ? 2 : 1;
  static constexpr int BM = 128;       // rows per CTA (pair tile: 256)
  static constexpr int BN = BN_;       // pair tile columns (UMMA N)
  static constexpr int BNH = BN / 2;   // B columns held per CTA
  static constexpr int BK = 128 / ELEM;
  static constexpr int UMMA_K = 32 / ELEM;
  static constexpr int CHUNK = 128 / ELEM;
  static constexpr int STAGES = STAGES_;
  static constexpr int A_BYTES = BM * BK * ELEM;
  static constexpr int B_BYTES = BNH * BK * ELEM;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // per CTA
  static constexpr int TMEM_COLS = ceil_pow2_cols(2 * BN);
  static constexpr int THREADS = 192;
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static constexpr u32 IDESC =
      make_idesc(KIND == KIND_BF16 ? 1u : 0u, KIND == KIND_BF16 ? 1u : 0u, false, true, 256, BN);
  static_assert(BN % 32 == 0 && BN <= 256, "pair tile N must be a multiple of 32, at most 256");
  static_assert(BNH % CHUNK == 0, "per-CTA B columns must be whole 128-byte chunks");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

template <class Cfg>
__global__ void __launch_bounds__(192, 1)
    gemm2_kernel(const __grid_constant__ TensorMap tmap_a, const __grid_constant__ TensorMap tmap_b,
                 const Params p) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const u32 raw = smem_u32(smem_raw);
  const u32 base = (raw + 1023u) & ~1023u;
  unsigned char *smem = smem_raw + (base - raw);
  const u32 stage0 = base;
  const u32 bars = base + Cfg::STAGES * Cfg::STAGE_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (Cfg::STAGES + s); };
  auto tfull_bar = [&](int a) { return bars + 8u * (2 * Cfg::STAGES + a); };
  auto tempty_bar = [&](int a) { return bars + 8u * (2 * Cfg::STAGES + 2 + a); };
  const u32 drain_bar = bars + 8u * (2 * Cfg::STAGES + 4);
  u32 *tmem_slot =
      reinterpret_cast<u32 *>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + (2 * Cfg::STAGES + 5) * 8);
  volatile u32 *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const u32 rank = cluster_ctarank();
  const int pair = blockIdx.x / 2;
  const int npairs = gridDim.x / 2;

  const int ntm = (p.GM + 2 * Cfg::BM - 1) / (2 * Cfg::BM);
  const int ntn = (p.GN + Cfg::BN - 1) / Cfg::BN;
  const int ntiles = ntm * ntn;
  const int nkb = (p.GK + Cfg::BK - 1) / Cfg::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(full_bar(s), 1);   // leader: its producer's arrive.expect_tx
      mbar_init(empty_bar(s), 1);  // leader MMA thread's commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps in each CTA (leader's copy used)
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc<2>(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish<2>();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any remote use
  tc_fence_after();
  const u32 tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel of the stream is complete from here on

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int s = 0;
      u32 ph = 0;
      for (int t = pair; t < ntiles && !*abort_flag; t += npairs) {
        int tm, tn;
        tile_coords<Cfg::GROUP_M>(t, ntm, ntn, tm, tn);
        const int m0 = tm * 2 * Cfg::BM + rank * Cfg::BM;
        const int n0 = tn * Cfg::BN + rank * Cfg::BNH;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(empty_bar(s), ph ^ 1u, p.status, 0x11)) {
            *abort_flag = 1;
            break;
          }
          const u32 sa = stage0 + s * Cfg::STAGE_BYTES;
          const u32 sb = sa + Cfg::A_BYTES;
          const u32 fb = mapa_cluster(full_bar(s), 0);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(s), 2 * Cfg::STAGE_BYTES);
          tma_load_2d_pair(sa, &tmap_a, fb, kb * Cfg::BK, m0);
#pragma unroll
          for (int c = 0; c < Cfg::BNH / Cfg::CHUNK; ++c)
            tma_load_2d_pair(sb + c * Cfg::BK * 128, &tmap_b, fb, n0 + c * Cfg::CHUNK, kb * Cfg::BK);
          if (++s == Cfg::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      for (int i = 0; i < Cfg::STAGES; ++i) {
        if (!mbar_wait(empty_bar(s), ph ^ 1u, p.status, 0x12)) break;
        if (++s == Cfg::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader CTA)
    // lane 0 alone, like the one-CTA kernel: no warp-wide reconvergence per k-block
    if (rank == 0 && lane == 0) {
      int s = 0;
      u32 ph = 0;
      int it = 0;
      for (int t = pair; t < ntiles && !*abort_flag; t += npairs, ++it) {
        const int acc = it & 1;
        const u32 acc_ph = (it >> 1) & 1;
        const u32 d_tmem = tmem_base + acc * Cfg::BN;
        if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, p.status, 0x13)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(full_bar(s), ph, p.status, 0x14)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const u32 sa = stage0 + s * Cfg::STAGE_BYTES;
          const u32 sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
            const u64 ad = smem_desc_sw128(sa + k * 32, 16, 1024);
            const u64 bd = smem_desc_sw128(sb + k * Cfg::UMMA_K * 128, Cfg::BK * 128, 1024);
            const u32 accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (Cfg::KIND == KIND_BF16)
              mma2_f16_ss(d_tmem, ad, bd, Cfg::IDESC, accum);
            else
              mma2_f8f6f4_ss(d_tmem, ad, bd, Cfg::IDESC, accum);
          }
          tc_commit2(mapa_cluster(empty_bar(s), 0));
          tc_commit2(mapa_cluster(empty_bar(s), 1));
          if (++s == Cfg::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok || *abort_flag) break;
        tc_commit2(mapa_cluster(tfull_bar(acc), 0));
        tc_commit2(mapa_cluster(tfull_bar(acc), 1));
      }
      tc_commit2(mapa_cluster(drain_bar, 0));
      mbar_wait(drain_bar, 0, p.status, 0x15);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    int it = 0;
    for (int t = pair; t < ntiles && !*abort_flag; t += npairs, ++it) {
      int tm, tn;
      tile_coords<Cfg::GROUP_M>(t, ntm, ntn, tm, tn);
      const int acc = it & 1;
      const u32 acc_ph = (it >> 1) & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(tfull_bar(acc), acc_ph, p.status, 0x16);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = tm * 2 * Cfg::BM + rank * Cfg::BM + q * 32 + lane;
      const u32 t_row = tmem_base + ((u32)(q * 32) << 16) + acc * Cfg::BN;
      bf16_store_tile<Config<Cfg::KIND, Cfg::BN, 1, false, true, false>>(p, t_row, row, tn * Cfg::BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(tempty_bar(acc));
        else
          mbar_arrive_cluster(tempty_bar(acc), 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into both TMEMs are complete
  tc_fence_after();
  if (warp == 1) tmem_dealloc<2>(tmem_base, Cfg::TMEM_COLS);
}

}  // namespace gemm
}  // namespace thork
