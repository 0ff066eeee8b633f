// PISA block statistics on Blackwell: TMA-staged q/k/v tiles, column sums on
// CUDA cores, the centred first-order covariance H_blk = Kc^T V on tcgen05
// with both H_blk (for its Frobenius norm) and the running per-(batch, head)
// sum accumulated in tensor memory.
//
// Semantics are those of stats.cu (HYD: pisa_kernels.cu:167-244; GENERIC:
// pisa_kernel.py:49-84): column sums run over the rows in order in FP32, the
// centred K is split into hi + lo 16-bit halves so the MMA keeps ~16 mantissa
// bits (GENERIC rounds it to 16 bits, as the reference's Triton kernel does).
//
// Work item = G consecutive 64-token blocks of one (batch, head); persistent
// CTAs walk items round-robin.  Per item the CTA writes its H partial sum to
// global memory; stats_reduce_kernel sums partials in a fixed order.
//
// Warps (640 threads, one CTA per SM):
//   warp 0     TMA producer: q, k, v tiles of each block into a 3-stage ring
//   warp 1     TMEM owner + MMA issuer (elected thread)
//   warps 2-7  q/k/v column sums (a thread owns two adjacent columns of one
//              tensor and adds its rows in order); K means to a double-
//              buffered shared array
//   warps 8-15 centring of K into the hi/lo tiles in 16-byte chunks
//   warps 16-19  read-back of H_blk from TMEM: the running H of the item (a
//              thread owns one row of it, kept in TMEM) and the Frobenius norm
// The three groups hand blocks on through mbarriers, so the sums of block
// j+1, the centring of block j and the read-back of block j-1 overlap.
// TMEM (384 columns used): H_blk double buffer, running H.
#include <cudaTypedefs.h>

#include <type_traits>

#include "kernels.h"
#include "umma.cuh"

namespace b2 {
namespace {

using namespace umma;

// warps: 0 producer, 1 MMA, 2-7 sums, 8-15 centring, 16-19 read-back
constexpr int kSumWarps = 6, kCentreWarps = 8, kReadWarps = 4;
constexpr int kSumWarp0 = 2, kCentreWarp0 = kSumWarp0 + kSumWarps, kReadWarp0 = kCentreWarp0 + kCentreWarps;
constexpr int kThreads = 32 * (kReadWarp0 + kReadWarps);
#ifndef B2_SUM_UNROLL
#define B2_SUM_UNROLL 8
#endif
constexpr int kSumUnroll = B2_SUM_UNROLL;  // 8-row groups of the column sums unrolled together
constexpr int kStages = 4;   // q/k/v ring depth
constexpr int kKcBufs = 1;   // centred-K (hi | lo) buffers: 4 x 48 KB ring + one 32 KB Kc fit in 227 KB
constexpr uint32_t kTile = 64 * 128 * 2;  // one 64-row x 128-col 16-bit tile (two 8 KB halves)
constexpr uint32_t kStageBytes = 3 * kTile;

struct __align__(8) Misc {
  uint64_t full[kStages];
  uint64_t empty[kStages];  // count 2: compute warps + MMA completion
  uint64_t kc_full[2];      // centred K tile written
  uint64_t mma_done[2];     // H_blk[b] ready (and Kc[b] consumed)
  uint64_t hblk_free[2];    // H_blk[b] read back (one arrival per read-back warp)
  uint64_t km_full[2];      // kmean[b] written (one arrival per sum warp)
  uint64_t km_free[2];      // kmean[b] consumed by the centring (one arrival per centring warp)
  uint64_t fin;             // all MMAs of this CTA complete
  uint32_t tmem;
  int abort_flag;
  float norm_part[8];
  __align__(16) float kmean[2][128];
};

struct Layout {
  static constexpr uint32_t stages = 0;
  static constexpr uint32_t kc = stages + kStages * kStageBytes;  // [kKcBufs][hi | lo]
  static constexpr uint32_t misc = kc + kKcBufs * 2 * kTile;
  static constexpr uint32_t total = misc + sizeof(Misc);
};
static_assert(Layout::total <= 232448, "shared memory budget");

struct StatsArgs {
  int kind;  // 0 linear 4D map, 1 tiled 5D map
  int heads, tokens, blocks, group, items;
  int frames, tiles_per_row, tiles_per_frame;
  int mode;  // B2_STATS_HYD or B2_STATS_GENERIC
  void* q_centroids;
  float* k_centroids;
  void* v_stats;
  float* h_norm;
  float* partial;
  int* status;
};

// plain: one 64-row x 256-byte box (row-major, unswizzled; q and k, read by
// the CUDA cores); otherwise two 64-column halves in the 128-byte swizzled
// layout the MMA reads (v).
__device__ __forceinline__ void load_tile(const CUtensorMap* map, const StatsArgs& a, char* dst, uint64_t* bar,
                                          int bh, int blk, bool plain) {
  const int b = bh / a.heads;
  const int h = bh - b * a.heads;
  for (int dh = 0; dh < (plain ? 1 : 2); ++dh) {
    if (a.kind == 0) {
      tma_load_4d(dst + dh * 8192, map, bar, dh * 64, blk * 64, h, b);
    } else {
      const int f = blk / a.tiles_per_frame;
      const int tile = blk - f * a.tiles_per_frame;
      const int tr = tile / a.tiles_per_row;
      const int tc = tile - tr * a.tiles_per_row;
      tma_load_5d(dst + dh * 8192, map, bar, dh * 64, h, tc * 8, tr * 8, b * a.frames + f);
    }
  }
}

template <bool BF16, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
stats_umma_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                  const __grid_constant__ CUtensorMap v_map, const __grid_constant__ StatsArgs a) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ __align__(1024) char smem[];
  Misc& m = *reinterpret_cast<Misc*>(smem + Layout::misc);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool with_norm = a.h_norm != nullptr;
  const bool with_lo = MODE == B2_STATS_HYD;
  if (threadIdx.x == 0) {
    m.abort_flag = (smem_u32(smem) & 1023u) ? 1 : 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&m.full[s], 1);
      mbar_init(&m.empty[s], kSumWarps + kCentreWarps + 1);  // every warp that read the stage + the MMAs
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&m.kc_full[b], kCentreWarps);
      mbar_init(&m.mma_done[b], 1);
      mbar_init(&m.hblk_free[b], kReadWarps);
      mbar_init(&m.km_full[b], kSumWarps);
      mbar_init(&m.km_free[b], kCentreWarps);
    }
    mbar_init(&m.fin, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc<512>(&m.tmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = m.tmem;
  volatile int* abort_flag = &m.abort_flag;
  const int groups = (a.blocks + a.group - 1) / a.group;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !*abort_flag) {
      tma_prefetch_desc(&q_map);
      tma_prefetch_desc(&k_map);
      tma_prefetch_desc(&v_map);
      int j = 0;  // running block counter of this CTA
      for (int item = blockIdx.x; item < a.items; item += gridDim.x) {
        const int bh = item / groups;
        const int g = item - bh * groups;
        const int first = g * a.group;
        const int last = min(a.blocks, first + a.group);
        for (int blk = first; blk < last; ++blk, ++j) {
          const int s = j % kStages;
          if (!mbar_wait(&m.empty[s], ((j / kStages) & 1) ^ 1, abort_flag, a.status, 21)) return;
          char* st = smem + Layout::stages + s * kStageBytes;
          mbar_expect_tx(&m.full[s], kStageBytes);
          load_tile(&q_map, a, st, &m.full[s], bh, blk, true);
          load_tile(&k_map, a, st + kTile, &m.full[s], bh, blk, true);
          load_tile(&v_map, a, st + 2 * kTile, &m.full[s], bh, blk, false);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      // H[i][j] = sum_r Kc[r][i] V[r][j]: A = Kc^T and B = V, both MN-major
      const uint32_t idesc = idesc_f16(128, 128, BF16, true, true);
      int j = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < a.items; item += gridDim.x, ++it) {
        const int bh = item / groups;
        const int g = item - bh * groups;
        const int first = g * a.group;
        const int last = min(a.blocks, first + a.group);
        for (int blk = first; blk < last; ++blk, ++j) {
          const int s = j % kStages;
          const int b = j & 1;
          if (!mbar_wait(&m.full[s], (j / kStages) & 1, abort_flag, a.status, 23) ||
              !mbar_wait(&m.kc_full[j % kKcBufs], (j / kKcBufs) & 1, abort_flag, a.status, 24)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&m.hblk_free[b], ((j >> 1) & 1) ^ 1, abort_flag, a.status, 25)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + Layout::stages + s * kStageBytes + 2 * kTile);
          const uint32_t hi_addr = smem_u32(smem + Layout::kc + (j % kKcBufs) * 2 * kTile);
          const uint32_t lo_addr = hi_addr + kTile;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dv = smem_desc_sw128(v_addr + kk * 2048, 8192, 1024);
            const uint64_t dh = smem_desc_sw128(hi_addr + kk * 2048, 8192, 1024);
            const uint64_t dl = smem_desc_sw128(lo_addr + kk * 2048, 8192, 1024);
            mma_ss(tmem + 128 * b, dh, dv, idesc, kk > 0 ? 1u : 0u);
            if (with_lo) mma_ss(tmem + 128 * b, dl, dv, idesc, 1u);
          }
          mma_commit(&m.mma_done[b]);
          mma_commit(&m.empty[s]);
        }
      }
      // every MMA issued has completed before TMEM is released (time-bounded)
      mma_commit(&m.fin);
      int no_abort = 0;
      mbar_wait(&m.fin, 0, &no_abort, a.status, 30);
    }
  } else if (warp < kCentreWarp0) {
    // ------------------------------------------------------------ column sums (warps 2-7)
    const int tid = threadIdx.x - 32 * kSumWarp0;  // 0..191: column pair of (q, k, v)
    const int tensor = tid >> 6;
    const int col = (tid & 63) * 2;
    int j = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < a.items; item += gridDim.x) {
      const int bh = item / groups;
      const int g = item - bh * groups;
      const int first = g * a.group;
      const int last = min(a.blocks, first + a.group);
      for (int blk = first; ok && blk < last; ++blk, ++j) {
        const int s = j % kStages;
        const int b = j & 1;
        const int len = min(64, a.tokens - blk * 64);
        if (!mbar_wait(&m.full[s], (j / kStages) & 1, abort_flag, a.status, 27)) {
          ok = false;
          break;
        }
        const char* tile = smem + Layout::stages + s * kStageBytes + tensor * kTile;
        // rows in order; q and k tiles are row-major 256-byte rows, v is in the
        // MMA's layout: (row 8*rr + u, col) at rr*1024 + u*128 + ((chunk ^ u) << 4)
        float s0 = 0.f, s1 = 0.f;
        const bool swz = tensor == 2;
        const char* base = swz ? tile + (col >> 6) * 8192 + ((col & 7) << 1) : tile + col * 2;
        const int chunk = (col & 63) >> 3;
        const int full_rows = len & ~7;
#pragma unroll kSumUnroll
        for (int rr = 0; rr < full_rows; rr += 8) {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int off = swz ? (rr + u) * 128 + ((chunk ^ u) << 4) : (rr + u) * 256;
            const uint32_t w = *reinterpret_cast<const uint32_t*>(base + off);
            float f0, f1;
            Cvt<T>::unpack2(w, f0, f1);
            s0 += f0;
            s1 += f1;
          }
        }
        for (int r = full_rows; r < len; ++r) {
          const int off = swz ? r * 128 + ((chunk ^ (r & 7)) << 4) : r * 256;
          const uint32_t w = *reinterpret_cast<const uint32_t*>(base + off);
          float f0, f1;
          Cvt<T>::unpack2(w, f0, f1);
          s0 += f0;
          s1 += f1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&m.empty[s]);  // this warp is done with the stage
        // kmean[b] was last read by the centring of block j - 2
        if (tensor == 1 && j >= 2 && !mbar_wait(&m.km_free[b], ((j - 2) >> 1) & 1, abort_flag, a.status, 29)) {
          ok = false;
          break;
        }
        const int64_t o = (int64_t(bh) * a.blocks + blk) * 128 + col;
        if (MODE == B2_STATS_HYD) {
          const float inv = 1.0f / static_cast<float>(len);
          const float m0 = s0 * inv, m1 = s1 * inv;
          if (tensor == 0) {
            *reinterpret_cast<uint32_t*>(static_cast<T*>(a.q_centroids) + o) = Cvt<T>::pack2(m0, m1);
          } else if (tensor == 1) {
            *reinterpret_cast<float2*>(a.k_centroids + o) = make_float2(m0, m1);
            *reinterpret_cast<float2*>(&m.kmean[b][col]) = make_float2(m0, m1);
          } else {
            *reinterpret_cast<uint32_t*>(static_cast<T*>(a.v_stats) + o) = Cvt<T>::pack2(m0, m1);
          }
        } else {
          const float flen = static_cast<float>(len);
          if (tensor == 0) {
            *reinterpret_cast<float2*>(static_cast<float*>(a.q_centroids) + o) = make_float2(s0 / flen, s1 / flen);
          } else if (tensor == 1) {
            const float m0 = s0 / flen, m1 = s1 / flen;
            *reinterpret_cast<float2*>(a.k_centroids + o) = make_float2(m0, m1);
            *reinterpret_cast<float2*>(&m.kmean[b][col]) = make_float2(m0, m1);
          } else {
            *reinterpret_cast<float2*>(static_cast<float*>(a.v_stats) + o) = make_float2(s0, s1);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&m.km_full[b]);
      }
    }
  } else if (warp < kReadWarp0) {
    // ------------------------------------------------------------ centring (warps 8-15)
    const int tid = threadIdx.x - 32 * kCentreWarp0;  // 0..255
    int j = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < a.items; item += gridDim.x) {
      const int bh = item / groups;
      const int g = item - bh * groups;
      const int first = g * a.group;
      const int last = min(a.blocks, first + a.group);
      (void)bh;
      for (int blk = first; ok && blk < last; ++blk, ++j) {
        const int s = j % kStages;
        const int b = j & 1;
        const int len = min(64, a.tokens - blk * 64);
        // the stage's K tile has landed, kmean[b] holds this block's K means,
        // and the Kc buffer was last read by the MMAs of block j - kKcBufs
        const int pj = j - kKcBufs;
        if (!mbar_wait(&m.full[s], (j / kStages) & 1, abort_flag, a.status, 27) ||
            !mbar_wait(&m.km_full[b], (j >> 1) & 1, abort_flag, a.status, 31) ||
            (pj >= 0 && !mbar_wait(&m.mma_done[pj & 1], (pj >> 1) & 1, abort_flag, a.status, 28))) {
          ok = false;
          break;
        }
        const char* st = smem + Layout::stages + s * kStageBytes;
        const float* kmean = m.kmean[b];
        // ---- centred K -> hi / lo tiles, 16-byte chunks (rows past len are 0)
        char* hi = smem + Layout::kc + (j % kKcBufs) * 2 * kTile;
        char* lo = hi + kTile;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int task = tid + 256 * i;
          const int r = task >> 4;
          const int chunk16 = task & 15;
          const int half = chunk16 >> 3;
          const int cc = chunk16 & 7;
          const uint32_t off = half * 8192 + r * 128 + ((cc ^ (r & 7)) << 4);
          const int c0 = half * 64 + cc * 8;
          const uint4 raw = *reinterpret_cast<const uint4*>(st + kTile + r * 256 + chunk16 * 16);
          const float4 km0 = *reinterpret_cast<const float4*>(kmean + c0);
          const float4 km1 = *reinterpret_cast<const float4*>(kmean + c0 + 4);
          const float km[8] = {km0.x, km0.y, km0.z, km0.w, km1.x, km1.y, km1.z, km1.w};
          const uint32_t kw[4] = {raw.x, raw.y, raw.z, raw.w};
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float x0 = 0.f, x1 = 0.f;
            if (r < len) {
              Cvt<T>::unpack2(kw[e], x0, x1);
              x0 -= km[2 * e];
              x1 -= km[2 * e + 1];
            }
            hw[e] = Cvt<T>::pack2(x0, x1);
            float h0, h1;
            Cvt<T>::unpack2(hw[e], h0, h1);
            lw[e] = Cvt<T>::pack2(x0 - h0, x1 - h1);
          }
          *reinterpret_cast<uint4*>(hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          if (with_lo) *reinterpret_cast<uint4*>(lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&m.kc_full[j % kKcBufs]);
          mbar_arrive(&m.km_free[b]);
          mbar_arrive(&m.empty[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ H read-back (warps 16-19)
    // one block behind the centring: add H_blk to the running H of the item
    // (TMEM columns 256-383, row trow, in block order) and reduce its norm
    const int rw = warp - kReadWarp0;  // 0..3
    const int sub = warp & 3;          // TMEM sub-partition
    const int trow = sub * 32 + lane;  // H row this thread reads back
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    const uint32_t run = tmem + lane_base + 256;
    int j = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < a.items; item += gridDim.x) {
      const int bh = item / groups;
      const int g = item - bh * groups;
      const int first = g * a.group;
      const int last = min(a.blocks, first + a.group);
      for (int blk = first; ok && blk < last; ++blk, ++j) {
        const int b = j & 1;
        if (!mbar_wait(&m.mma_done[b], (j >> 1) & 1, abort_flag, a.status, 26)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s0 = 0.f, s1 = 0.f;
#pragma unroll 1
        for (int h4 = 0; h4 < 4; ++h4) {
          uint32_t r[32], acc[32];
          tmem_ld32(tmem + lane_base + 128 * b + 32 * h4, r);
          if (blk != first) tmem_ld32(run + 32 * h4, acc);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float x0 = __uint_as_float(r[e]), x1 = __uint_as_float(r[e + 1]);
            s0 = fmaf(x0, x0, s0);
            s1 = fmaf(x1, x1, s1);
            if (blk != first) {
              r[e] = __float_as_uint(__uint_as_float(acc[e]) + x0);
              r[e + 1] = __float_as_uint(__uint_as_float(acc[e + 1]) + x1);
            }
          }
          tmem_st32(run + 32 * h4, r);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&m.hblk_free[b]);
        if (with_norm) {
          float sq = s0 + s1;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
          // parity-buffered partial norms: the next block's writes cannot
          // overtake this block's final sum
          if (lane == 0) m.norm_part[(j & 1) * 4 + rw] = sq;
          named_barrier_sync(2, 128);
          if (rw == 0 && lane == 0) {
            const float* np = m.norm_part + (j & 1) * 4;
            a.h_norm[int64_t(bh) * a.blocks + blk] = sqrtf(np[0] + np[1] + np[2] + np[3]);
          }
        }
      }
      if (!ok) break;
      // running H of this item -> partial[bh][g]
      float* dst = a.partial + (int64_t(bh) * groups + g) * 128 * 128 + int64_t(trow) * 128;
#pragma unroll 1
      for (int h4 = 0; h4 < 4; ++h4) {
        uint32_t acc[32];
        tmem_ld32(run + 32 * h4, acc);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(dst + 32 * h4 + e) =
              make_float4(__uint_as_float(acc[e]), __uint_as_float(acc[e + 1]), __uint_as_float(acc[e + 2]),
                          __uint_as_float(acc[e + 3]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

}  // namespace
}  // namespace b2

namespace b2 {
namespace {
PFN_cuTensorMapEncodeTiled_v12000 stats_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// Row-block tensor map (64 columns x 64 rows, or one 8x8 spatial tile).
bool stats_map(CUtensorMap* map, const b2_view& v, int* kind, bool plain) {
  auto fn = stats_encode_fn();
  if (fn == nullptr) return false;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt = v.dtype == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t e = 2;
  if (v.order == B2_ORDER_LINEAR) {
    const cuuint64_t dims[4] = {cuuint64_t(v.head_dim), cuuint64_t(v.tokens), cuuint64_t(v.heads), cuuint64_t(v.batch)};
    const uint64_t st = uint64_t(v.stride_t) * e;
    const uint64_t sh = v.heads > 1 ? uint64_t(v.stride_h) * e : st * v.tokens;
    const uint64_t sb = v.batch > 1 ? uint64_t(v.stride_b) * e : sh * v.heads;
    const cuuint64_t strides[3] = {st, sh, sb};
    const cuuint32_t box[4] = {plain ? 128u : 64u, 64, 1, 1};
    *kind = 0;
    return fn(map, dt, 4, v.base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              plain ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  const int64_t frame = int64_t(v.grid_h) * v.grid_w;
  const int64_t frames = v.tokens / frame;
  if (v.batch > 1 && v.stride_b != frames * frame * v.stride_t) return false;
  const cuuint64_t dims[5] = {cuuint64_t(v.head_dim), cuuint64_t(v.heads), cuuint64_t(v.grid_w), cuuint64_t(v.grid_h),
                              cuuint64_t(frames * v.batch)};
  const uint64_t st = uint64_t(v.stride_t) * e;
  const uint64_t sh = v.heads > 1 ? uint64_t(v.stride_h) * e : 16;
  const cuuint64_t strides[4] = {sh, st, st * v.grid_w, st * v.grid_w * v.grid_h};
  const cuuint32_t box[5] = {plain ? 128u : 64u, 1, 8, 8, 1};
  *kind = 1;
  return fn(map, dt, 5, v.base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            plain ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_stats_umma(const b2_view& q, const b2_view& k, const b2_view& v, int mode, int group,
                              void* q_centroids, float* k_centroids, void* v_stats, float* h_norm, float* partial,
                              int* status, cudaStream_t stream, bool* launched) {
  *launched = false;
  // D < 128 (multiples of 8): columns past D load as zeros (TMA fill), so
  // centroids and H carry zeros there
  if (q.head_dim > 128 || q.head_dim % 8 || q.dtype == B2_F32 || (mode != B2_STATS_HYD && mode != B2_STATS_GENERIC))
    return cudaSuccess;
  CUtensorMap qm, km, vm;
  int qk = 0, kk = 0, vk = 0;
  if (!stats_map(&qm, q, &qk, true) || !stats_map(&km, k, &kk, true) || !stats_map(&vm, v, &vk, false) || qk != kk ||
      kk != vk)
    return cudaSuccess;
  StatsArgs a{};
  a.kind = qk;
  a.heads = q.heads;
  a.tokens = q.tokens;
  a.blocks = (q.tokens + 63) / 64;
  a.group = group;
  const int bh = q.batch * q.heads;
  a.items = bh * ((a.blocks + group - 1) / group);
  if (qk == 1) {
    const int64_t frame = int64_t(q.grid_h) * q.grid_w;
    a.frames = static_cast<int>(q.tokens / frame);
    a.tiles_per_row = q.grid_w / 8;
    a.tiles_per_frame = static_cast<int>(frame / 64);
  } else {
    a.frames = a.tiles_per_row = a.tiles_per_frame = 1;
  }
  a.mode = mode;
  a.q_centroids = q_centroids;
  a.k_centroids = k_centroids;
  a.v_stats = v_stats;
  a.h_norm = h_norm;
  a.partial = partial;
  a.status = status;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = a.items < sms ? a.items : sms;
  const size_t smem = Layout::total;
  cudaError_t err;
#define B2_SU_LAUNCH(BF, MODE)                                                                                  \
  do {                                                                                                         \
    err = ensure_smem(reinterpret_cast<const void*>(stats_umma_kernel<BF, MODE>), int(smem)); \
    if (err != cudaSuccess) return err;                                                                        \
    stats_umma_kernel<BF, MODE><<<grid, kThreads, smem, stream>>>(qm, km, vm, a);                             \
  } while (0)
  if (q.dtype == B2_BF16) {
    if (mode == B2_STATS_HYD) B2_SU_LAUNCH(true, B2_STATS_HYD);
    else B2_SU_LAUNCH(true, B2_STATS_GENERIC);
  } else {
    if (mode == B2_STATS_HYD) B2_SU_LAUNCH(false, B2_STATS_HYD);
    else B2_SU_LAUNCH(false, B2_STATS_GENERIC);
  }
#undef B2_SU_LAUNCH
  *launched = true;
  return cudaGetLastError();
}

}  // namespace b2
