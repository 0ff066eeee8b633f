// Blackwell-native attention kernel: TMA-staged Q/K/V tiles, tcgen05.mma
// with TMEM accumulators for Q.K^T and P.V, warp-specialised pipeline.
//
// One CTA owns a pair of 64-row query blocks (M = 128 rows, the native
// tcgen05 tile height) of one (batch, head).  The key tiles it visits are
//   * PISA (mode LIST): the centroid tail tiles, then the union of the two
//     query blocks' selected exact blocks; a tile only contributes to the rows
//     of the query block(s) that selected it (other rows are masked).
//     rdna35_pisa_ck/__init__.py:272-316 (exact Flex attention over the
//     routed blocks + centroid tail with log-length bias + first-order
//     correction) merged in one online softmax;
//   * full attention (mode ALL): every 64-key tile (triton_kernel.py:113-160);
//   * fixed block (mode DIAG): each query block's own key block
//     (triton_kernel.py:53-100, optional causal mask).
//
// Warp roles (192 threads):
//   warp 0    TMA producer: Q pair once, then K/V (or centroid) tiles into a
//             2-stage ring, finally H (first-order operand) for the correction
//   warp 1    TMEM owner + single-thread MMA issuer:
//             S(j) = Q K(j)^T  -> TMEM S[j%2] (128 x 64 FP32)
//             O   += P(j) V(j) -> TMEM O      (128 x 128 FP32)
//             C    = Q H       -> TMEM (reuses the S columns after the loop)
//   warps 2-5 softmax: thread r owns query row r (TMEM lane r); reads S with
//             tcgen05.ld, masks/scales in the log2 domain, online max with
//             lazy O rescaling (only when the max grows by > 2^8), writes P as
//             BF16 into a 128-byte-swizzled shared tile, and finally reads O
//             and C to produce (O + tail_mass * corr_scale * C) / l.
// TMEM: 256 columns (O 0-127, S0 128-191, S1 192-255) so two CTAs share an SM.
#include <cudaTypedefs.h>

#include <type_traits>

#include "kernels.h"
#include "umma.cuh"

namespace b2 {

namespace {

using namespace umma;

constexpr int kThreads = 192;
constexpr int kMaxList = 192;  // union of two selected lists
constexpr int kMaxSelWords = 32;
constexpr uint32_t kQBytes = 128 * 128 * 2;
constexpr uint32_t kStageBytes = 2 * 64 * 128 * 2;  // K + V tile

struct __align__(8) Misc {
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint64_t c_full;
  uint64_t mma_done;
  uint32_t tmem;
  int abort_flag;
  int ntiles;
  int nlist;
  uint32_t sel[2][kMaxSelWords];
  uint16_t list[kMaxList];
};

struct SmemLayout {
  static constexpr uint32_t q = 0;                     // [2 d-halves][128 rows][128 B]
  static constexpr uint32_t kv = q + kQBytes;          // [2 stages][K 2x8KB | V 2x8KB]
  static constexpr uint32_t p = kv + 2 * kStageBytes;  // [128 rows][128 B]
  static constexpr uint32_t misc = p + 128 * 128;
  static constexpr uint32_t total = misc + sizeof(Misc);
};

// Tile descriptor: kind (0 = centroid tail, 1 = key block), block index and
// the two-bit mask of query halves it applies to.
struct Tile {
  int tail;
  int blk;
  uint32_t mask;
};

__device__ __forceinline__ Tile tile_at(const UmmaArgs& a, const Misc& m, int j, int ntail) {
  Tile t;
  if (j < ntail) {
    t.tail = 1;
    t.blk = j;
    t.mask = 3u;
    return t;
  }
  const int jj = j - ntail;
  t.tail = 0;
  if (a.mode == 0) {
    t.blk = jj;
    t.mask = 3u;
  } else {
    const uint32_t e = m.list[jj];
    t.blk = e & 0x3FFF;
    t.mask = e >> 14;
  }
  return t;
}

// TMA load of 64 rows (one key/query block) x 64 columns (half of D=128).
__device__ __forceinline__ void load_block(const CUtensorMap* map, const UmmaArgs& a, void* dst, uint64_t* bar,
                                           int kind, int bh, int blk, int dh) {
  const int b = bh / a.heads;
  const int h = bh - b * a.heads;
  if (kind == 0) {
    tma_load_4d(dst, map, bar, dh * 64, blk * 64, h, b);
  } else {
    const int f = blk / a.tiles_per_frame;
    const int tile = blk - f * a.tiles_per_frame;
    const int tr = tile / a.tiles_per_row;
    const int tc = tile - tr * a.tiles_per_row;
    tma_load_5d(dst, map, bar, dh * 64, h, tc * 8, tr * 8, b * a.frames + f);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 2)
attn_umma_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                 const __grid_constant__ CUtensorMap v_map, const __grid_constant__ CUtensorMap kc_map,
                 const __grid_constant__ CUtensorMap vc_map, const __grid_constant__ CUtensorMap h_map,
                 const UmmaArgs a) {
  extern __shared__ __align__(1024) char smem[];
  Misc& m = *reinterpret_cast<Misc*>(smem + SmemLayout::misc);
  char* q_s = smem + SmemLayout::q;
  char* kv_s = smem + SmemLayout::kv;
  char* p_s = smem + SmemLayout::p;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x;
  const int bh = blockIdx.y;
  const int qa = 2 * pair;
  const int qb = 2 * pair + 1;
  const bool has_b = qb < a.nqb;
  const int ntail = a.nb > 0 ? (a.nb + 63) / 64 : 0;
  const int words = (a.nb + 31) >> 5;

  if (threadIdx.x == 0) {
    if ((smem_u32(smem) & 1023u) != 0) {
      m.abort_flag = 1;
      atomicCAS(a.status, 0, 0x300);
    } else {
      m.abort_flag = 0;
    }
    mbar_init(&m.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&m.kv_full[s], 1);
      mbar_init(&m.kv_empty[s], 1);
      mbar_init(&m.s_full[s], 1);
      mbar_init(&m.s_free[s], 4);
    }
    mbar_init(&m.p_full, 4);
    mbar_init(&m.pv_done, 1);
    mbar_init(&m.c_full, 1);
    mbar_init(&m.mma_done, 1);
    // key tile list
    int nlist = 0;
    if (a.mode == 1) {
      const int32_t* la = a.indices + (int64_t(bh) * a.nqb + qa) * a.nsel;
      const int32_t* lb = a.indices + (int64_t(bh) * a.nqb + (has_b ? qb : qa)) * a.nsel;
      const int nbk = (a.tk + 63) / 64;
      int ia = 0, ib = has_b ? 0 : a.nsel;
      while ((ia < a.nsel || ib < a.nsel) && nlist < kMaxList) {
        const int va = ia < a.nsel ? min(max(la[ia], 0), nbk - 1) : 0x7fffffff;
        const int vb = ib < a.nsel ? min(max(lb[ib], 0), nbk - 1) : 0x7fffffff;
        uint32_t e;
        if (va == vb) {
          e = va | (3u << 14);
          ++ia;
          ++ib;
        } else if (va < vb) {
          e = va | (1u << 14);
          ++ia;
        } else {
          e = vb | (2u << 14);
          ++ib;
        }
        m.list[nlist++] = static_cast<uint16_t>(e);
      }
    } else if (a.mode == 2) {
      m.list[nlist++] = static_cast<uint16_t>(qa | (1u << 14));
      if (has_b) m.list[nlist++] = static_cast<uint16_t>(qb | (2u << 14));
    } else {
      nlist = (a.tk + 63) / 64;
    }
    m.nlist = nlist;
    m.ntiles = ntail + nlist;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (ntail > 0) {
    for (int i = threadIdx.x; i < 2 * words; i += kThreads) {
      const int half = i / words;
      const int w = i - half * words;
      const int qblk = half && has_b ? qb : qa;
      m.sel[half][w] = a.sel_bits[(int64_t(bh) * a.nqb + qblk) * words + w];
    }
  }
  if (warp == 1) tmem_alloc<256>(&m.tmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = m.tmem;
  const int n = m.ntiles;
  volatile int* abort_flag = &m.abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !*abort_flag) {
      tma_prefetch_desc(&q_map);
      tma_prefetch_desc(&k_map);
      tma_prefetch_desc(&v_map);
      mbar_expect_tx(&m.q_full, kQBytes);
      for (int half = 0; half < 2; ++half)
        for (int dh = 0; dh < 2; ++dh)
          load_block(&q_map, a, q_s + dh * 16384 + half * 8192, &m.q_full, a.q_kind, bh, half ? qb : qa, dh);
      const int total = n + (a.has_corr ? 1 : 0);
      for (int j = 0; j < total; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&m.kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, a.status, 1)) break;
        char* stage = kv_s + s * kStageBytes;
        mbar_expect_tx(&m.kv_full[s], kStageBytes);
        if (j < n) {
          const Tile t = tile_at(a, m, j, ntail);
          for (int dh = 0; dh < 2; ++dh) {
            if (t.tail) {
              tma_load_3d(stage + dh * 8192, &kc_map, &m.kv_full[s], dh * 64, t.blk * 64, bh);
              tma_load_3d(stage + 16384 + dh * 8192, &vc_map, &m.kv_full[s], dh * 64, t.blk * 64, bh);
            } else {
              load_block(&k_map, a, stage + dh * 8192, &m.kv_full[s], a.kv_kind, bh, t.blk, dh);
              load_block(&v_map, a, stage + 16384 + dh * 8192, &m.kv_full[s], a.kv_kind, bh, t.blk, dh);
            }
          }
        } else {
          for (int dh = 0; dh < 2; ++dh) tma_load_3d(stage + dh * 16384, &h_map, &m.kv_full[s], dh * 64, 0, bh);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc_s = idesc_f16(128, 64, BF16, false, false);
      const uint32_t idesc_o = idesc_f16(128, 128, BF16, false, true);
      const uint32_t q_addr = smem_u32(q_s);
      const uint32_t p_addr = smem_u32(p_s);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(&m.p_full, i & 1, abort_flag, a.status, 2)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(kv_s + (i & 1) * kStageBytes + 16384);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t da = smem_desc_sw128(p_addr + kk * 32, 16, 1024);
          const uint64_t db = smem_desc_sw128(v_addr + kk * 2048, 8192, 1024);
          mma_ss(tmem, da, db, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&m.pv_done);
        mma_commit(&m.kv_empty[i & 1]);
        return true;
      };
      bool ok = mbar_wait(&m.q_full, 0, abort_flag, a.status, 3);
      for (int j = 0; ok && j < n; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&m.kv_full[s], (j >> 1) & 1, abort_flag, a.status, 4)) break;
        if (!mbar_wait(&m.s_free[s], ((j >> 1) & 1) ^ 1, abort_flag, a.status, 5)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(kv_s + s * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t da = smem_desc_sw128(q_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t db = smem_desc_sw128(k_addr + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
          mma_ss(tmem + 128 + 64 * s, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&m.s_full[s]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && n > 0) ok = issue_pv(n - 1);
      if (ok && a.has_corr) {
        const int s = n & 1;
        if (mbar_wait(&m.kv_full[s], (n >> 1) & 1, abort_flag, a.status, 6)) {
          tc_fence_after();
          const uint32_t h_addr = smem_u32(kv_s + s * kStageBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = smem_desc_sw128(q_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(h_addr + kk * 2048, 16384, 1024);
            mma_ss(tmem + 128, da, db, idesc_o, kk > 0 ? 1u : 0u);
          }
          mma_commit(&m.c_full);
        }
      }
      // every MMA this thread issued has completed before TMEM is released
      // (bounded by time only, even after an abort)
      mma_commit(&m.mma_done);
      int no_abort = 0;
      mbar_wait(&m.mma_done, 0, &no_abort, a.status, 7);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int sub = warp & 3;         // TMEM sub-partition of this warp
    const int row = sub * 32 + lane;  // query row within the pair
    const int half = row >> 6;        // 0: block qa, 1: block qb
    const int qblk = half ? qb : qa;
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    const int tq_row = qblk * 64 + (row & 63);
    float mrun = -INFINITY, lrun = 0.f, tmass = 0.f;
    char* prow = p_s + (row >> 3) * 1024 + (row & 7) * 128;
    for (int j = 0; j < n; ++j) {
      const int s = j & 1;
      const Tile t = tile_at(a, m, j, ntail);
      const bool active = ((t.mask >> half) & 1u) != 0;
      uint32_t v[64];
      if (!mbar_wait(&m.s_full[s], (j >> 1) & 1, abort_flag, a.status, 8)) break;
      tc_fence_after();
      tmem_ld32(tmem + lane_base + 128 + 64 * s, v);
      tmem_ld32(tmem + lane_base + 128 + 64 * s + 32, v + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&m.s_free[s]);
      float alpha = 1.f;
      bool rescale = false;
      if (active) {
        float mx = -INFINITY;
        if (t.tail) {
          const uint32_t w0 = m.sel[half][(t.blk * 64) >> 5];
          const uint32_t w1 = (t.blk * 64 + 32) < a.nb ? m.sel[half][((t.blk * 64) >> 5) + 1] : 0u;
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int jj = t.blk * 64 + c;
            const uint32_t bit = c < 32 ? (w0 >> c) & 1u : (w1 >> (c - 32)) & 1u;
            const bool masked = jj >= a.nb || bit;
            const float bias = jj == a.nb - 1 ? a.log2_last : 6.0f;  // log2(64) = 6
            const float xv = masked ? -INFINITY : fmaf(__uint_as_float(v[c]), a.scale_log2, bias);
            v[c] = __float_as_uint(xv);
            mx = fmaxf(mx, xv);
          }
        } else {
          const int klen = min(64, a.tk - t.blk * 64);
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            bool masked = c >= klen;
            if (a.causal) masked = masked || (t.blk * 64 + c > tq_row);
            const float xv = masked ? -INFINITY : __uint_as_float(v[c]) * a.scale_log2;
            v[c] = __float_as_uint(xv);
            mx = fmaxf(mx, xv);
          }
        }
        const float mnew = fmaxf(mrun, mx);
        if (mrun == -INFINITY) {
          mrun = mnew;
        } else if (mnew > mrun + 8.0f) {
          alpha = ex2(mrun - mnew);
          mrun = mnew;
          rescale = true;
        }
        float sum = 0.f;
        if (mrun == -INFINITY) {
#pragma unroll
          for (int c = 0; c < 64; ++c) v[c] = 0u;
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const float pv = ex2(__uint_as_float(v[c]) - mrun);
            v[c] = __float_as_uint(pv);
            sum += pv;
          }
        }
        lrun = lrun * alpha + sum;
        tmass = tmass * alpha + (t.tail ? sum : 0.f);
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) v[c] = 0u;
      }
      if (j >= 1 && !mbar_wait(&m.pv_done, (j - 1) & 1, abort_flag, a.status, 9)) break;
      if (__any_sync(0xffffffffu, rescale)) {
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(tmem + lane_base + c0, o);
        }
        tmem_wait_st();
      }
      // P row -> 128-byte swizzled K-major tile (chunk c of row r at c ^ (r % 8))
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 w;
        w.x = Cvt<typename std::conditional<BF16, __nv_bfloat16, __half>::type>::pack2(__uint_as_float(v[8 * c]),
                                                                                      __uint_as_float(v[8 * c + 1]));
        w.y = Cvt<typename std::conditional<BF16, __nv_bfloat16, __half>::type>::pack2(__uint_as_float(v[8 * c + 2]),
                                                                                      __uint_as_float(v[8 * c + 3]));
        w.z = Cvt<typename std::conditional<BF16, __nv_bfloat16, __half>::type>::pack2(__uint_as_float(v[8 * c + 4]),
                                                                                      __uint_as_float(v[8 * c + 5]));
        w.w = Cvt<typename std::conditional<BF16, __nv_bfloat16, __half>::type>::pack2(__uint_as_float(v[8 * c + 6]),
                                                                                      __uint_as_float(v[8 * c + 7]));
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = w;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&m.p_full);
    }
    // ---- epilogue
    bool ok = n == 0 || mbar_wait(&m.pv_done, (n - 1) & 1, abort_flag, a.status, 10);
    if (ok && a.has_corr) ok = mbar_wait(&m.c_full, 0, abort_flag, a.status, 11);
    tc_fence_after();
    const bool store = ok && (half == 0 || has_b) && tq_row < a.tq;
    const float inv = lrun > 0.f ? 1.f / lrun : 0.f;
    const float cw = tmass * a.corr_scale;
    char* orow = store ? a.o.row(bh, tq_row) : nullptr;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 32) {
      uint32_t o[32], cr[32];
      tmem_ld32(tmem + lane_base + c0, o);
      if (a.has_corr) tmem_ld32(tmem + lane_base + 128 + c0, cr);
      tmem_wait_ld();
      if (store) {
        uint32_t packed[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float f0 = __uint_as_float(o[c]);
          float f1 = __uint_as_float(o[c + 1]);
          if (a.has_corr) {
            f0 = fmaf(__uint_as_float(cr[c]), cw, f0);
            f1 = fmaf(__uint_as_float(cr[c + 1]), cw, f1);
          }
          packed[c / 2] = Cvt<typename std::conditional<BF16, __nv_bfloat16, __half>::type>::pack2(f0 * inv, f1 * inv);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c0 * 2);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          dst[q4] = make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
      }
    }
    if (store && a.lse != nullptr) {
      a.lse[int64_t(bh) * a.tq + tq_row] = lrun > 0.f ? (mrun + __log2f(lrun)) * 0.6931471805599453f : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<256>(tmem);
  }
}

__device__ int g_status;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

CUtensorMapDataType tma_dtype(int dtype) {
  return dtype == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

bool encode(CUtensorMap* map, int dtype, int rank, void* base, const cuuint64_t* dims, const cuuint64_t* strides,
            const cuuint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(map, tma_dtype(dtype), rank, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-block tensor map of a b2_view: kind 0 = linear 4D (D,T,H,B), kind 1 =
// 8x8-tiled 5D (D,H,x,y,frame*batch).  Box: 64 columns x 64 rows.
bool rows_map(CUtensorMap* map, const b2_view& v, int* kind) {
  const uint64_t es = 2;
  if (v.order == B2_ORDER_LINEAR) {
    const cuuint64_t dims[4] = {cuuint64_t(v.head_dim), cuuint64_t(v.tokens), cuuint64_t(v.heads),
                                cuuint64_t(v.batch)};
    uint64_t st = uint64_t(v.stride_t) * es;
    uint64_t sh = v.heads > 1 ? uint64_t(v.stride_h) * es : st * v.tokens;
    uint64_t sb = v.batch > 1 ? uint64_t(v.stride_b) * es : sh * v.heads;
    if (st == 0 || sh == 0 || sb == 0) return false;
    const cuuint64_t strides[3] = {st, sh, sb};
    const cuuint32_t box[4] = {64, 64, 1, 1};
    *kind = 0;
    return encode(map, v.dtype, 4, v.base, dims, strides, box);
  }
  const int64_t frame = int64_t(v.grid_h) * v.grid_w;
  const int64_t frames = v.tokens / frame;
  if (v.batch > 1 && v.stride_b != frames * frame * v.stride_t) return false;
  const cuuint64_t dims[5] = {cuuint64_t(v.head_dim), cuuint64_t(v.heads), cuuint64_t(v.grid_w),
                              cuuint64_t(v.grid_h), cuuint64_t(frames * v.batch)};
  const uint64_t st = uint64_t(v.stride_t) * es;
  const uint64_t sh = v.heads > 1 ? uint64_t(v.stride_h) * es : 16;
  const cuuint64_t strides[4] = {sh, st, st * v.grid_w, st * v.grid_w * v.grid_h};
  const cuuint32_t box[5] = {64, 1, 8, 8, 1};
  *kind = 1;
  return encode(map, v.dtype, 5, v.base, dims, strides, box);
}

bool rows3_map(CUtensorMap* map, int dtype, const void* base, int rows, int batch, int box_rows) {
  const cuuint64_t dims[3] = {128, cuuint64_t(rows), cuuint64_t(batch)};
  const cuuint64_t strides[2] = {256, cuuint64_t(rows) * 256};
  const cuuint32_t box[3] = {64, cuuint32_t(box_rows), 1};
  return encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box);
}

}  // namespace

int* device_status_ptr() {
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_status) != cudaSuccess) return nullptr;
  return static_cast<int*>(ptr);
}

bool umma_supported(const b2_view& q, const b2_view& k, const b2_view& v, const b2_view& o) {
  if (q.head_dim != 128 || q.dtype == B2_F32) return false;
  for (const b2_view* x : {&q, &k, &v}) {
    if (x->order == B2_ORDER_TILED8) {
      const int64_t frame = int64_t(x->grid_h) * x->grid_w;
      if (x->batch > 1 && x->stride_b != (x->tokens / frame) * frame * x->stride_t) return false;
    }
  }
  (void)o;
  return encode_fn() != nullptr;
}

cudaError_t launch_attn_umma(const b2_view& qv, const b2_view& kv, const b2_view& vv, const b2_view& ov,
                             const AttnParams& p, int* status, cudaStream_t stream, bool* launched) {
  *launched = false;
  UmmaArgs a{};
  CUtensorMap q_map, k_map, v_map, kc_map, vc_map, h_map;
  int qk = 0, kk = 0, vk = 0;
  if (!rows_map(&q_map, qv, &qk) || !rows_map(&k_map, kv, &kk) || !rows_map(&v_map, vv, &vk) || kk != vk)
    return cudaSuccess;
  const int bh = qv.batch * qv.heads;
  a.q_kind = qk;
  a.kv_kind = kk;
  if (qk != kk) return cudaSuccess;
  a.heads = qv.heads;
  a.tq = qv.tokens;
  a.tk = kv.tokens;
  a.nqb = (qv.tokens + 63) / 64;
  if (kk == 1) {
    const int64_t frame = int64_t(kv.grid_h) * kv.grid_w;
    a.frames = static_cast<int>(kv.tokens / frame);
    a.tiles_per_row = kv.grid_w / 8;
    a.tiles_per_frame = static_cast<int>(frame / 64);
  } else {
    a.frames = 1;
    a.tiles_per_row = 1;
    a.tiles_per_frame = 1;
  }
  if (qk == 1 && kk == 1 && (qv.grid_h != kv.grid_h || qv.grid_w != kv.grid_w)) return cudaSuccess;
  a.mode = p.mode;
  a.indices = p.indices;
  a.nsel = p.nsel;
  a.sel_bits = p.sel_bits;
  a.nb = p.nb;
  if (p.mode == 1 && 2 * p.nsel > kMaxList) return cudaSuccess;
  if (p.nb > 32 * kMaxSelWords) return cudaSuccess;
  a.has_corr = p.h != nullptr ? 1 : 0;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.corr_scale = p.corr_scale;
  a.causal = p.causal;
  a.o = p.o;
  a.lse = p.lse;
  a.status = status;
  if (p.nb > 0) {
    const int last_len = kv.tokens - 64 * (p.nb - 1);
    a.log2_last = log2f(static_cast<float>(last_len));
    if (!rows3_map(&kc_map, qv.dtype, p.kc, p.nb, bh, 64) || !rows3_map(&vc_map, qv.dtype, p.vc, p.nb, bh, 64))
      return cudaSuccess;
  } else {
    kc_map = k_map;
    vc_map = v_map;
  }
  if (p.h != nullptr) {
    if (!rows3_map(&h_map, qv.dtype, p.h, 128, bh, 128)) return cudaSuccess;
  } else {
    h_map = k_map;
  }
  const size_t smem = SmemLayout::total;
  dim3 grid((a.nqb + 1) / 2, bh);
  cudaError_t err;
  if (qv.dtype == B2_BF16) {
    err = cudaFuncSetAttribute(attn_umma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    attn_umma_kernel<true><<<grid, kThreads, smem, stream>>>(q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  } else {
    err = cudaFuncSetAttribute(attn_umma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    attn_umma_kernel<false><<<grid, kThreads, smem, stream>>>(q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  }
  *launched = true;
  return cudaGetLastError();
}

}  // namespace b2
