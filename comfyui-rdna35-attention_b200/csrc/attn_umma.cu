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
// Two layouts, chosen by NW (softmax warpgroups per CTA):
//   NW = 1 (default): 224 threads, 256 TMEM columns, 2-stage K/V rings,
//     two CTAs per SM -- one CTA's set-up (barriers, TMEM, union list, Q
//     load, pipeline fill) and epilogue overlap the other CTA's main loop.
//   NW = 2: 384 threads, 512 TMEM columns, 6-stage rings, one CTA per SM;
//     the two warpgroups split the key tiles (split K inside the CTA) and
//     merge their partial softmaxes at the end.
// Warp roles:
//   warp 0    TMA producer: Q pair once, then K (or centroid) tiles into the
//             K ring, finally H (first-order operand) for the correction
//   warp 2+4NW  TMA producer of the V tiles (own ring)
//   warp 1 (and 11 when NW = 2)  single-thread MMA issuer per softmax
//             warpgroup (warp 1 also owns the TMEM columns):
//             S(j) = Q K(j)^T  -> TMEM S buffer of warpgroup j%NW (128 x 64
//                                 FP32, two buffers per warpgroup)
//             O   += P(j) V(j) -> TMEM O of warpgroup j%NW (128 x 128 FP32),
//                                 P read from TMEM (tcgen05.mma A operand)
//             C    = Q H       -> TMEM (reuses warpgroup 0's S columns)
//             S(j) reuses the buffer of P(j-2NW), so it is issued only after
//             that P.V has completed; otherwise S and P.V go out as their
//             operands arrive.
//   warps 2..1+4NW  softmax warpgroup(s): thread r owns query row r (TMEM
//             lane r); reads its 64 logits with one tcgen05.ld pair,
//             computes exp2 of the scaled logits with packed f32x2
//             arithmetic, keeps a lazy running max (O is rescaled in TMEM
//             only when the max grows by more than 2^8), and writes P as
//             16-bit pairs back over the S columns with tcgen05.st.  At the
//             end (O + tail_mass * corr_scale * C) / l is stored (with NW = 2
//             after merging the two partial softmaxes, each warpgroup writing
//             half of the columns).
#include <cudaTypedefs.h>

#include <type_traits>

#include "kernels.h"
#include "umma.cuh"

namespace b2 {

namespace {

using namespace umma;

// NW = softmax warpgroups per CTA.
//   NW = 2: 384 threads (K producer, 2 MMA issuers, 2 softmax warpgroups, V
//           producer), 512 TMEM columns, 6-stage K/V rings, one CTA per SM.
//   NW = 1: 224 threads (K producer, MMA issuer, 1 softmax warpgroup, V
//           producer), 256 TMEM columns, 2-stage K and 3-stage V rings
//           (113 KB of shared memory), two CTAs per SM: one CTA's set-up and
//           epilogue overlap the other's main loop.
template <int NW>
struct Cfg {
  static constexpr int kThreads = NW == 2 ? 384 : 224;
  static constexpr int kStagesK = NW == 2 ? 6 : 2;  // K ring (also carries the two H halves)
  static constexpr int kStagesV = NW == 2 ? 6 : 3;  // V ring: P.V(j) needs V(j) one tile later than S(j) needs K(j)
  static constexpr int kVWarp = 2 + 4 * NW;  // V producer warp
  static constexpr uint32_t kTmemCols = 256 * NW;
  static constexpr int kCtasPerSm = NW == 2 ? 1 : 2;
};
constexpr int kMaxStages = 6;
constexpr int kMaxList = 192;  // union of two selected lists
constexpr int kMaxSelWords = 32;
constexpr uint32_t kQBytes = 128 * 128 * 2;
constexpr uint32_t kSlotBytes = 64 * 128 * 2;  // one K or V tile (two 8 KB d-halves)

struct __align__(8) Misc {
  uint64_t q_full;
  uint64_t k_full[kMaxStages];
  uint64_t k_empty[kMaxStages];
  uint64_t v_full[kMaxStages];
  uint64_t v_empty[kMaxStages];
  uint64_t s_full[2][2];
  uint64_t p_full[2][2];  // [warpgroup][S buffer]: a warpgroup may run one tile ahead of the P.V issue
  uint64_t pv_done[2][2];  // [warpgroup][S buffer]
  uint64_t pv_all;         // every P.V complete (before C reuses warpgroup 0's S columns)
  uint64_t c_full;
  uint64_t mma_done[2];
  uint32_t tmem;
  int abort_flag;
  int ntiles;
  int nlist;
  uint32_t sel[2][kMaxSelWords];
  uint16_t list[kMaxList];
};

template <int NW>
struct SmemLayout {
  static constexpr uint32_t q = 0;                 // [2 d-halves][128 rows][128 B]
  static constexpr uint32_t k = q + kQBytes;       // [stages][2 d-halves x 8 KB]
  static constexpr uint32_t v = k + Cfg<NW>::kStagesK * kSlotBytes;
  static constexpr uint32_t misc = v + Cfg<NW>::kStagesV * kSlotBytes;
  static constexpr uint32_t total = misc + sizeof(Misc);
};
static_assert(SmemLayout<2>::total <= 232448, "shared memory budget");
static_assert(2 * (SmemLayout<1>::total + 1024) <= 233472, "two CTAs per SM");

struct Tile {
  int tail;  // 1: centroid tail tile, 0: key block
  int blk;
  uint32_t mask;  // bit h: applies to query half h
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

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (lo, hi) = (x0, x1) * (s, s) + (t, t) with one packed f32x2 FMA
__device__ __forceinline__ void fma2(float& lo, float& hi, float x0, float x1, float s, float t) {
  uint64_t x, sv, tv, d;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(x) : "f"(x0), "f"(x1));
  asm("mov.b64 %0, {%1, %1};\n" : "=l"(sv) : "f"(s));
  asm("mov.b64 %0, {%1, %1};\n" : "=l"(tv) : "f"(t));
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(x), "l"(sv), "l"(tv));
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(lo), "=f"(hi) : "l"(d));
}

// (a0, a1) += (b0, b1) with one packed f32x2 add
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  uint64_t x, y, d;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(y) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(a0), "=f"(a1) : "l"(d));
}

// S(j) = Q K(j)^T into the S buffer of warpgroup j%2; frees K slot on completion.
// The buffer last held P(j-4): the caller issues S(j) only once that P.V has
// completed (it reads P from these TMEM columns).
template <bool BF16, int NW>
__device__ __forceinline__ bool issue_s(Misc& m, char* k_s, uint32_t q_addr, uint32_t tmem, const UmmaArgs& a,
                                        volatile int* abort_flag, int j, long long* trace) {
  constexpr int kStages = Cfg<NW>::kStagesK;
  const int s = j % kStages;
  const int w = j % NW;
  const int i = j / NW;
  const int sb = i & 1;
  if (!mbar_wait(&m.k_full[s], (j / kStages) & 1, abort_flag, a.status, 4)) return false;
  tc_fence_after();
  if (trace && j < 256) trace[6 * j + 1] = clock64();
  const uint32_t idesc_s = idesc_f16(128, 64, BF16, false, false);
  const uint32_t k_addr = smem_u32(k_s + s * kSlotBytes);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t da = smem_desc_sw128(q_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
    const uint64_t db = smem_desc_sw128(k_addr + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
    mma_ss(tmem + w * 256 + 128 + 64 * sb, da, db, idesc_s, kk > 0 ? 1u : 0u);
  }
  mma_commit(&m.s_full[w][sb]);
  mma_commit(&m.k_empty[s]);
  if (trace && j < 256) trace[6 * 256 + 1 + 256 + 1024 + j] = clock64();
  return true;
}

// O(w) += P(jj) V(jj) for key tile jj (warpgroup w = jj % 2); P is read from
// TMEM, where the softmax wrote it over the tile's S columns.
template <bool BF16, int NW>
__device__ __forceinline__ bool issue_pv(Misc& m, char* smem, uint32_t tmem, const UmmaArgs& a,
                                         volatile int* abort_flag, int jj, long long* trace) {
  constexpr int kStages = Cfg<NW>::kStagesV;
  const int w = jj % NW;
  const int i = jj / NW;
  const uint32_t p_tmem = tmem + w * 256 + 128 + 64 * (i & 1);
  if (!mbar_wait(&m.p_full[w][i & 1], (i >> 1) & 1, abort_flag, a.status, 2)) return false;
  if (!mbar_wait(&m.v_full[jj % kStages], (jj / kStages) & 1, abort_flag, a.status, 12)) return false;
  tc_fence_after();
  const uint32_t idesc_o = idesc_f16(128, 128, BF16, false, true);
  const uint32_t v_addr = smem_u32(smem + SmemLayout<NW>::v + (jj % kStages) * kSlotBytes);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t db = smem_desc_sw128(v_addr + kk * 2048, 8192, 1024);
    mma_ts(tmem + w * 256, p_tmem + kk * 8, db, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
  }
  mma_commit(&m.pv_done[w][i & 1]);
  mma_commit(&m.v_empty[jj % kStages]);
  if (trace && jj < 256) trace[6 * 256 + 1 + jj] = clock64();
  return true;
}

// WITHHOLD (the timeout diagnostics of b2_debug_withhold_q only): the Q tile
// is never loaded, so the pipeline's bounded waits run out.  MASKED (mode
// DIAG with a mask): every row adds its FP32 mask terms a.bias to the scaled
// scores, and a row whose keys are all masked stores NaN.  MIRROR (head-
// sharded calls): every output row is also stored into a.n_mirror peer
// copies of the output buffer.
template <bool BF16, int NW, bool WITHHOLD, bool MASKED, bool MIRROR>
__global__ void __launch_bounds__(Cfg<NW>::kThreads, Cfg<NW>::kCtasPerSm)
attn_umma_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                 const __grid_constant__ CUtensorMap v_map, const __grid_constant__ CUtensorMap kc_map,
                 const __grid_constant__ CUtensorMap vc_map, const __grid_constant__ CUtensorMap h_map,
                 const __grid_constant__ UmmaArgs a) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ __align__(1024) char smem[];
  constexpr int kThreads = Cfg<NW>::kThreads;
  constexpr int kStagesK = Cfg<NW>::kStagesK;
  constexpr int kStagesV = Cfg<NW>::kStagesV;
  Misc& m = *reinterpret_cast<Misc*>(smem + SmemLayout<NW>::misc);
  char* q_s = smem + SmemLayout<NW>::q;
  char* k_s = smem + SmemLayout<NW>::k;
  char* v_s = smem + SmemLayout<NW>::v;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x;
  const int bh = blockIdx.y;
  int qa = 2 * pair;
  int qb = 2 * pair + 1;
  bool has_b = qb < a.nqb;  // the pairing kernel's output is read after grid_dep_wait
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
    for (int s = 0; s < kStagesK; ++s) {
      mbar_init(&m.k_full[s], 1);
      mbar_init(&m.k_empty[s], 1);
    }
    for (int s = 0; s < kStagesV; ++s) {
      mbar_init(&m.v_full[s], 1);
      mbar_init(&m.v_empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&m.s_full[w][b], 1);
      }
      mbar_init(&m.p_full[w][0], 4);
      mbar_init(&m.p_full[w][1], 4);
      mbar_init(&m.pv_done[w][0], 1);
      mbar_init(&m.pv_done[w][1], 1);
    }
    mbar_init(&m.c_full, 1);
    mbar_init(&m.mma_done[0], 1);
    mbar_init(&m.mma_done[1], 1);
    mbar_init(&m.pv_all, 1);
    if (a.mode != 1) {
      int nlist = 0;
      if (a.mode == 2) {
        m.list[nlist++] = static_cast<uint16_t>(qa | (1u << 14));
        if (has_b) m.list[nlist++] = static_cast<uint16_t>(qb | (2u << 14));
      } else {
        nlist = (a.tk + 63) / 64;
      }
      m.nlist = nlist;
      m.ntiles = ntail + nlist;
    }
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  // launched with programmatic stream serialization: everything below reads
  // the routing results (or the inputs) and writes the output
  grid_dep_wait();
  if (a.pairs != nullptr) {
    qa = a.pairs[(int64_t(bh) * gridDim.x + pair) * 2];
    qb = a.pairs[(int64_t(bh) * gridDim.x + pair) * 2 + 1];
    if (qb < 0) qb = a.nqb;  // single block: half B inactive
    has_b = qb < a.nqb;
  }
  if (a.mode == 1 && warp == 0) {
    // union of the two query blocks' selected key blocks, sorted, each entry
    // tagged with the half(s) that selected it: the lanes OR the (clamped)
    // indices into two bitsets in parallel, then lane l emits the set bits of
    // word l at the offset given by a warp prefix sum of the popcounts
    const int nbk = (a.tk + 63) / 64;
    const int wk = (nbk + 31) >> 5;
    // scratch bitsets in the V ring, which no TMA writes before the set-up
    // barrier below
    uint32_t* ua = reinterpret_cast<uint32_t*>(v_s);
    uint32_t* ub = ua + kMaxSelWords;
    if (lane < wk) {
      ua[lane] = 0u;
      ub[lane] = 0u;
    }
    __syncwarp();
    const int32_t* la = a.indices + (int64_t(bh) * a.nqb + qa) * a.nsel;
    const int32_t* lb = a.indices + (int64_t(bh) * a.nqb + (has_b ? qb : qa)) * a.nsel;
    for (int e = lane; e < a.nsel; e += 32) {
      const int va = min(max(la[e], 0), nbk - 1);
      atomicOr(&ua[va >> 5], 1u << (va & 31));
      if (has_b) {
        const int vb = min(max(lb[e], 0), nbk - 1);
        atomicOr(&ub[vb >> 5], 1u << (vb & 31));
      }
    }
    __syncwarp();
    const uint32_t wa = lane < wk ? ua[lane] : 0u;
    const uint32_t wb = lane < wk ? ub[lane] : 0u;
    uint32_t u = wa | wb;
    const int cnt = __popc(u);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int pos = incl - cnt;
    while (u != 0u) {
      const int bit = __ffs(u) - 1;
      u &= u - 1u;
      const uint32_t tag = ((wa >> bit) & 1u) | (((wb >> bit) & 1u) << 1);
      if (pos < kMaxList) m.list[pos] = static_cast<uint16_t>((lane * 32 + bit) | (tag << 14));
      ++pos;
    }
    const int nlist = min(__shfl_sync(0xffffffffu, incl, 31), kMaxList);
    if (lane == 0) {
      m.nlist = nlist;
      m.ntiles = ntail + nlist;
    }
    // the scratch words are generic-proxy writes to memory that TMA (async
    // proxy) fills after the set-up barrier
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
  if (warp == 1) tmem_alloc<Cfg<NW>::kTmemCols>(&m.tmem);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = m.tmem;
  const int n = m.ntiles;
  volatile int* abort_flag = &m.abort_flag;
  long long* trace = (a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0) ? a.trace : nullptr;
  if (trace && threadIdx.x == 0) trace[6 * 256] = clock64();

  if (warp == 0) {
    // ------------------------------------------------------------ Q / K / H producer
    if (lane == 0 && !*abort_flag) {
      tma_prefetch_desc(&q_map);
      tma_prefetch_desc(&k_map);
      if constexpr (!WITHHOLD) {
        mbar_expect_tx(&m.q_full, kQBytes);
        for (int half = 0; half < 2; ++half)
          for (int dh = 0; dh < 2; ++dh)
            load_block(&q_map, a, q_s + dh * 16384 + half * 8192, &m.q_full, a.q_kind, bh, half ? qb : qa, dh);
      }
      // key tiles 0..n-1, then the two 64-column halves of H as "tiles" n, n+1
      const int total = n + (a.has_corr ? 2 : 0);
      int issued = 0;
      for (int j = 0; j < total; ++j, issued = j) {
        const int s = j % kStagesK;
        if (!mbar_wait(&m.k_empty[s], ((j / kStagesK) & 1) ^ 1, abort_flag, a.status, 1)) break;
        char* slot = k_s + s * kSlotBytes;
        if (trace && j < 256) trace[6 * j] = clock64();
        if (j < n) {
          mbar_expect_tx(&m.k_full[s], kSlotBytes);
          const Tile t = tile_at(a, m, j, ntail);
          for (int dh = 0; dh < 2; ++dh) {
            if (t.tail) tma_load_3d(slot + dh * 8192, &kc_map, &m.k_full[s], dh * 64, t.blk * 64, bh);
            else load_block(&k_map, a, slot + dh * 8192, &m.k_full[s], a.kv_kind, bh, t.blk, dh);
          }
        } else {
          // H[:, 64*(j-n) : 64*(j-n)+64]: 128 rows x 128 B
          mbar_expect_tx(&m.k_full[s], kSlotBytes);
          tma_load_3d(slot, &h_map, &m.k_full[s], (j - n) * 64, 0, bh);
        }
      }
      if (*abort_flag) drain_loads(m.k_full, kStagesK, issued, WITHHOLD ? nullptr : &m.q_full, a.status);
    }
  } else if (warp == Cfg<NW>::kVWarp) {
    // ------------------------------------------------------------ V producer
    if (lane == 0 && !*abort_flag) {
      tma_prefetch_desc(&v_map);
      int issued = 0;
      for (int j = 0; j < n; ++j, issued = j) {
        const int s = j % kStagesV;
        if (!mbar_wait(&m.v_empty[s], ((j / kStagesV) & 1) ^ 1, abort_flag, a.status, 13)) break;
        char* slot = v_s + s * kSlotBytes;
        mbar_expect_tx(&m.v_full[s], kSlotBytes);
        const Tile t = tile_at(a, m, j, ntail);
        for (int dh = 0; dh < 2; ++dh) {
          if (t.tail) tma_load_3d(slot + dh * 8192, &vc_map, &m.v_full[s], dh * 64, t.blk * 64, bh);
          else load_block(&v_map, a, slot + dh * 8192, &m.v_full[s], a.kv_kind, bh, t.blk, dh);
        }
      }
      if (*abort_flag) drain_loads(m.v_full, kStagesV, issued, nullptr, a.status);
    }
  } else if (warp == 1 || (NW == 2 && warp == 11)) {
    // ------------------------------------------------------------ MMA issuers
    // One issuing thread per softmax warpgroup (tcgen05.commit tracks the
    // issuing thread's MMAs), so the two warpgroups' S -> P -> P.V chains
    // never wait behind each other.  Warpgroup w owns key tiles j = w, w+2, ...
    // (local index i = j / 2) and S buffers i % 2.
    if (elect_one()) {
      const int w = warp == 1 ? 0 : 1;
      const uint32_t q_addr = smem_u32(q_s);
      const int cnt = (n - w + NW - 1) / NW;
      // S(i) may go out once P.V(i-2) (same S buffer) has completed and its K
      // tile is in; P.V(i) once P(i) and V(i) are.  S is preferred.
      bool ok = mbar_wait(&m.q_full, 0, abort_flag, a.status, 3);
      int ns = 0, npv = 0;
      const long long start = clock64();
      while (ok && npv < cnt) {
        bool did = false;
        if (ns < cnt) {
          const int j = NW * ns + w;
          const bool buf_free = ns < 2 || (ns - 2 < npv && mbar_test_wait(&m.pv_done[w][ns & 1], ((ns - 2) >> 1) & 1));
          if (buf_free && mbar_test_wait(&m.k_full[j % kStagesK], (j / kStagesK) & 1)) {
            ok = issue_s<BF16, NW>(m, k_s, q_addr, tmem, a, abort_flag, j, trace);
            ++ns;
            did = true;
          }
        }
        if (!did && ok && npv < ns) {
          const int j = NW * npv + w;
          if (mbar_test_wait(&m.p_full[w][npv & 1], (npv >> 1) & 1) &&
              mbar_test_wait(&m.v_full[j % kStagesV], (j / kStagesV) & 1)) {
            ok = issue_pv<BF16, NW>(m, smem, tmem, a, abort_flag, j, trace);
            ++npv;
            did = true;
          }
        }
        if (!did) {
          if (*abort_flag) {
            ok = false;
          } else if (clock64() - start > (1ll << 33)) {
            // far beyond any legitimate CTA duration
            *abort_flag = 1;
            atomicCAS(a.status, kStatusOk, (kStatusTimeout << 8) | 23);
            ok = false;
          }
        }
      }
      if (w == 0 && ok && a.has_corr) {
        // C overwrites warpgroup 0's S columns: its P.V must have read its P
        mma_commit(&m.pv_all);
        ok = mbar_wait(&m.pv_all, 0, abort_flag, a.status, 24);
      }
      if (w == 0 && ok && a.has_corr) {
        // C = Q H as two N=64 products, one per 64-column half of H
        const uint32_t idesc_c = idesc_f16(128, 64, BF16, false, true);
        for (int hh = 0; ok && hh < 2; ++hh) {
          const int j = n + hh;
          const int s = j % kStagesK;
          ok = mbar_wait(&m.k_full[s], (j / kStagesK) & 1, abort_flag, a.status, 6);
          if (!ok) break;
          tc_fence_after();
          const uint32_t h_addr = smem_u32(k_s + s * kSlotBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = smem_desc_sw128(q_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(h_addr + kk * 2048, 16384, 1024);
            mma_ss(tmem + 128 + 64 * hh, da, db, idesc_c, kk > 0 ? 1u : 0u);
          }
        }
        if (ok) mma_commit(&m.c_full);
      }
      // every MMA this thread issued completes before TMEM is released
      // (bounded by time only, even after an abort)
      mma_commit(&m.mma_done[w]);
      int no_abort = 0;
      mbar_wait(&m.mma_done[w], 0, &no_abort, a.status, 7);
    }
  } else if (warp >= 2 && warp < 2 + 4 * NW) {
    // ------------------------------------------------------------ softmax
    const int wg = (warp - 2) >> 2;   // 0 or 1
    const int sub = warp & 3;         // TMEM sub-partition of this warp
    const int row = sub * 32 + lane;  // query row within the pair
    const int half = row >> 6;        // 0: block qa, 1: block qb
    const int qblk = half ? qb : qa;
    const uint32_t lane_base = static_cast<uint32_t>(sub * 32) << 16;
    const uint32_t o_base = tmem + lane_base + wg * 256;
    const int tq_row = qblk * 64 + (row & 63);
    float mrun = -INFINITY, lrun = 0.f, tmass = 0.f;
    const int nb_ = a.nb, causal_ = a.causal, tk_ = a.tk;
    const float log2_last_ = a.log2_last, scale_log2_ = a.scale_log2;
    int i = 0;
    bool ok = true;
    for (int j = wg; j < n; j += NW, ++i) {
      const int sb = i & 1;
      const Tile t = tile_at(a, m, j, ntail);
      const bool active = ((t.mask >> half) & 1u) != 0;
      if (!mbar_wait(&m.s_full[wg][sb], (i >> 1) & 1, abort_flag, a.status, 8)) {
        ok = false;
        break;
      }
      if (trace && lane == 0 && sub == 0 && j < 256) trace[6 * j + 3] = clock64();
      tc_fence_after();
      const uint32_t s_addr = o_base + 128 + 64 * sb;
      const int klen = t.tail ? 64 : min(64, tk_ - t.blk * 64);
      const bool plain = !MASKED && !t.tail && klen == 64 && !causal_;
      // masked columns of this tile as two 32-bit words (bit c = column c),
      // and the column that carries the last (ragged) block's log2 length
      uint32_t bad0 = 0u, bad1 = 0u;
      int lastc = -1;
      float bias = 0.f;
      if (!plain) {
        uint64_t bad;
        if (t.tail) {
          const int c0 = t.blk * 64;
          const uint32_t w0 = m.sel[half][c0 >> 5];
          const uint32_t w1 = (c0 + 32) < nb_ ? m.sel[half][(c0 >> 5) + 1] : 0u;
          const int valid = min(64, nb_ - c0);
          bad = (static_cast<uint64_t>(w1) << 32) | w0;
          if (valid < 64) bad |= ~0ull << valid;
          lastc = nb_ - 1 - c0;
          bias = 6.0f;  // log2(64)
        } else {
          bad = klen < 64 ? (~0ull << klen) : 0ull;
          if (causal_) {
            const int lim = tq_row - t.blk * 64;  // columns > lim are masked
            if (lim < 63) bad |= lim < 0 ? ~0ull : (~0ull << (lim + 1));
          }
        }
        bad0 = static_cast<uint32_t>(bad);
        bad1 = static_cast<uint32_t>(bad >> 32);
      }
      const float last_bias = log2_last_;
      float alpha = 1.f;
      bool rescale = false;
      // the row's 64 logits are read from TMEM once; P goes back over them
      uint32_t v[64];
      if (active) {
        tmem_ld32(s_addr, v);
        tmem_ld32(s_addr + 32, v + 32);
        tmem_wait_ld();
      }
      if (trace && lane == 0 && sub == 0 && j < 256) trace[6 * j + 2] = clock64();
      // logits in the log2 domain: x = s * scale_log2 (+ log2 len for the
      // tail), masked -> -inf.  Plain tiles keep raw s and fold the scale
      // into the exp2 argument.
      float mul = scale_log2_;
      if (active) {
        float mx;
        if (plain) {
          float m0 = fmaxf(__uint_as_float(v[0]), __uint_as_float(v[1]));
          float m1 = fmaxf(__uint_as_float(v[2]), __uint_as_float(v[3]));
#pragma unroll
          for (int c = 4; c < 64; c += 4) {
            m0 = max3(m0, __uint_as_float(v[c]), __uint_as_float(v[c + 1]));
            m1 = max3(m1, __uint_as_float(v[c + 2]), __uint_as_float(v[c + 3]));
          }
          mx = fmaxf(m0, m1) * scale_log2_;
        } else {
          mx = -INFINITY;
          if constexpr (MASKED) {
            // x = (s * scale + mask term) * log2(e); rows past the last token read no terms
            const float* brow = a.bias + int64_t(bh) * a.bias_bh_stride + int64_t(tq_row) * 64;
            const bool in_range = tq_row < a.tq;
#pragma unroll
            for (int c = 0; c < 64; c += 4) {
              const float4 b4 = in_range ? *reinterpret_cast<const float4*>(brow + c) : make_float4(0.f, 0.f, 0.f, 0.f);
              const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t bw = c < 32 ? bad0 : bad1;
                const float x = fmaf(__uint_as_float(v[c + e]), scale_log2_, bb[e] * 1.4426950408889634f);
                const float xm = ((bw >> ((c + e) & 31)) & 1u) ? -INFINITY : x;
                v[c + e] = __float_as_uint(xm);
                mx = fmaxf(mx, xm);
              }
            }
          } else {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              const uint32_t bw = c < 32 ? bad0 : bad1;
              const float x = fmaf(__uint_as_float(v[c]), scale_log2_, c == lastc ? last_bias : bias);
              const float xm = ((bw >> (c & 31)) & 1u) ? -INFINITY : x;
              v[c] = __float_as_uint(xm);
              mx = fmaxf(mx, xm);
            }
          }
          mul = 1.f;
        }
        const float mnew = fmaxf(mrun, mx);
        if (mrun == -INFINITY) {
          mrun = mnew;
        } else if (mnew > mrun + 8.0f) {
          alpha = ex2(mrun - mnew);
          mrun = mnew;
          rescale = true;
        }
      }
      if (trace && lane == 0 && sub == 0 && j < 256) trace[6 * j + 4] = clock64();
      if (__any_sync(0xffffffffu, rescale)) {
        // O may be rescaled once this warpgroup's previous P.V is done (the
        // one before it completed ahead of S(j))
        if (i >= 1 && !mbar_wait(&m.pv_done[wg][(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag, a.status, 9)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_base + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(o_base + c0, o);
        }
        tmem_wait_st();
      }
      // P = exp2(x - m) -> 16-bit pairs, written back over the first 32 S
      // columns of the buffer (the A operand of P.V)
      if (active && mrun != -INFINITY) {
        const float neg = -mrun;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          float x0, x1;
          fma2(x0, x1, __uint_as_float(v[c]), __uint_as_float(v[c + 1]), mul, neg);
          const float p0 = ex2(x0);
          const float p1 = ex2(x1);
          add2(s0, s1, p0, p1);
          v[c / 2] = Cvt<T>::pack2(p0, p1);
        }
        const float sum = s0 + s1;
        lrun = lrun * alpha + sum;
        tmass = tmass * alpha + (t.tail ? sum : 0.f);
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = 0u;
      }
      tmem_st32(s_addr, v);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&m.p_full[wg][sb]);
      if (trace && lane == 0 && j < 256) trace[6 * 256 + 257 + 4 * j + sub] = clock64();
      if (trace && lane == 0 && sub == 0 && j < 256) trace[6 * j + 5] = clock64();
    }
    // ---- merge the two partial softmaxes, add the correction, store
    if (ok && i >= 1) ok = mbar_wait(&m.pv_done[wg][(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag, a.status, 10);
    float mm = mrun, a0 = 1.f, a1 = 0.f, lt = lrun, tt = tmass;
    if constexpr (NW == 2) {
      // partial statistics [m | l | tail mass] x 128 rows per warpgroup go
      // into the V ring (every P.V has completed once both warpgroups get here)
      named_barrier_sync(1, 256);
      float* stat_own = reinterpret_cast<float*>(v_s + wg * 2048);
      const float* stat0 = reinterpret_cast<const float*>(v_s);
      const float* stat1 = reinterpret_cast<const float*>(v_s + 2048);
      stat_own[row] = mrun;
      stat_own[128 + row] = lrun;
      stat_own[256 + row] = tmass;
      named_barrier_sync(1, 256);
      const float m0 = stat0[row], m1 = stat1[row];
      mm = fmaxf(m0, m1);
      a0 = m0 == -INFINITY ? 0.f : ex2(m0 - mm);
      a1 = m1 == -INFINITY ? 0.f : ex2(m1 - mm);
      lt = stat0[128 + row] * a0 + stat1[128 + row] * a1;
      tt = stat0[256 + row] * a0 + stat1[256 + row] * a1;
    }
    if (ok && a.has_corr) ok = mbar_wait(&m.c_full, 0, abort_flag, a.status, 11);
    tc_fence_after();
    const bool store = ok && !*abort_flag && (half == 0 || has_b) && tq_row < a.tq;
    const float inv = lt > 0.f ? 1.f / lt : (MASKED ? __int_as_float(0x7fc00000) : 0.f);
    const float cw = tt * a.corr_scale;
    char* orow = store ? a.o.row(bh, tq_row) : nullptr;
    const uint32_t row_base = tmem + lane_base;
#pragma unroll 1
    for (int c0 = wg * (128 / NW); c0 < (wg + 1) * (128 / NW); c0 += 32) {
      // each warpgroup stores 128 / NW of the output columns
      uint32_t o0[32], o1[32], cr[32];
      tmem_ld32(row_base + c0, o0);
      if constexpr (NW == 2) tmem_ld32(row_base + 256 + c0, o1);
      if (a.has_corr) tmem_ld32(row_base + 128 + c0, cr);
      tmem_wait_ld();
      if (store) {
        uint32_t packed[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float f0 = __uint_as_float(o0[c]) * a0;
          float f1 = __uint_as_float(o0[c + 1]) * a0;
          if constexpr (NW == 2) {
            f0 = fmaf(__uint_as_float(o1[c]), a1, f0);
            f1 = fmaf(__uint_as_float(o1[c + 1]), a1, f1);
          }
          if (a.has_corr) {
            f0 = fmaf(__uint_as_float(cr[c]), cw, f0);
            f1 = fmaf(__uint_as_float(cr[c + 1]), cw, f1);
          }
          packed[c / 2] = Cvt<T>::pack2(f0 * inv, f1 * inv);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c0 * 2);
        if (a.o.dim == 128) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
        } else {  // head dim < 128: the columns past D were zero-filled inputs, not outputs
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            if (c0 + 8 * q4 < a.o.dim)
              dst[q4] = make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
        }
        if constexpr (MIRROR && NW == 1) {
          // stage the row for the peer copies: 128 rows x 256 B in the (now
          // idle) K ring, 16-byte chunks XOR-swizzled by the row
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int chunk = (c0 >> 3) + q4;
            *reinterpret_cast<uint4*>(k_s + row * 256 + ((chunk ^ (row & 15)) << 4)) =
                make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
          }
        } else if constexpr (MIRROR) {
          // the same 16-byte stores into the other GPUs' copies of the output
          // buffer (peer memory over NVLink), at the same offset
          const int64_t off = (orow - a.o.base) + c0 * 2;
          for (int mi = 0; mi < a.n_mirror; ++mi) {
            uint4* md = reinterpret_cast<uint4*>(a.mirror[mi] + off);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
              if (c0 + 8 * q4 < a.o.dim)
                md[q4] = make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
          }
        }
      }
    }
    if constexpr (MIRROR && NW == 1) {
      // peer copies with coalesced rows: a warp writes two whole 256-byte
      // rows per instruction over NVLink
      named_barrier_sync(1, 128);
      const int tid = threadIdx.x - 64;
      if (!*abort_flag) {
        for (int i = tid; i < 128 * 16; i += 128) {
          const int r = i >> 4;
          const int ch = i & 15;
          const int rh = r >> 6;
          const int tq_r = (rh ? qb : qa) * 64 + (r & 63);
          if ((rh == 0 || has_b) && tq_r < a.tq && ch * 8 < a.o.dim) {
            const uint4 val = *reinterpret_cast<const uint4*>(k_s + r * 256 + ((ch ^ (r & 15)) << 4));
            const int64_t off = (a.o.row(bh, tq_r) - a.o.base) + ch * 16;
            if (a.mirror_multicast)
              multimem_st16(a.mirror[0] + off, val);
            else
              for (int mi = 0; mi < a.n_mirror; ++mi) *reinterpret_cast<uint4*>(a.mirror[mi] + off) = val;
          }
        }
      }
    }
    if (store && wg == 0 && a.lse != nullptr) {
      a.lse[int64_t(bh) * a.tq + tq_row] = lt > 0.f ? (mm + __log2f(lt)) * 0.6931471805599453f : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<Cfg<NW>::kTmemCols>(tmem);
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
  // D < 128 (multiples of 8): the TMA boxes stay 64 columns wide and read
  // the columns past D as zeros, which changes no dot product
  if (q.head_dim > 128 || q.head_dim % 8 || q.dtype == B2_F32) return false;
  if (o.head_dim != q.head_dim || v.head_dim != q.head_dim) return false;
  for (const b2_view* x : {&q, &k, &v}) {
    if (x->order == B2_ORDER_TILED8) {
      const int64_t frame = int64_t(x->grid_h) * x->grid_w;
      if (x->batch > 1 && x->stride_b != (x->tokens / frame) * frame * x->stride_t) return false;
    }
  }
  return encode_fn() != nullptr;
}

// Softmax warpgroups per attention CTA: 1 (default; two CTAs per SM, measured
// 27% faster on the Anima PISA call) or 2 (B200ATTN_ATTN_WG=2; one CTA per SM).
int attn_warpgroups() {
  static const int nw = [] {
    const char* env = getenv("B200ATTN_ATTN_WG");
    return env != nullptr && env[0] == '2' ? 2 : 1;
  }();
  return nw;
}

template <bool BF16, int NW, bool WITHHOLD, bool MASKED, bool MIRROR>
cudaError_t launch_variant(dim3 grid, cudaStream_t stream, const CUtensorMap& q_map, const CUtensorMap& k_map,
                           const CUtensorMap& v_map, const CUtensorMap& kc_map, const CUtensorMap& vc_map,
                           const CUtensorMap& h_map, const UmmaArgs& a) {
  const int smem = static_cast<int>(SmemLayout<NW>::total);
  const cudaError_t err =
      ensure_smem(reinterpret_cast<const void*>(attn_umma_kernel<BF16, NW, WITHHOLD, MASKED, MIRROR>), smem);
  if (err != cudaSuccess) return err;
  return launch_pdl(attn_umma_kernel<BF16, NW, WITHHOLD, MASKED, MIRROR>, grid, dim3(Cfg<NW>::kThreads), size_t(smem), stream,
                    q_map, k_map, v_map, kc_map, vc_map, h_map, a);
}

template <bool BF16, int NW>
cudaError_t launch_nw(dim3 grid, cudaStream_t stream, const CUtensorMap& q_map, const CUtensorMap& k_map,
                      const CUtensorMap& v_map, const CUtensorMap& kc_map, const CUtensorMap& vc_map,
                      const CUtensorMap& h_map, const UmmaArgs& a) {
  if (a.debug_withhold_q)
    return launch_variant<BF16, NW, true, false, false>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  if (a.bias != nullptr)
    return launch_variant<BF16, NW, false, true, false>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  if (a.n_mirror > 0)
    return launch_variant<BF16, NW, false, false, true>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  return launch_variant<BF16, NW, false, false, false>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a);
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
  if (p.mode == 1 && (2 * p.nsel > kMaxList || (kv.tokens + 63) / 64 > 32 * kMaxSelWords)) return cudaSuccess;
  if (p.nb > 32 * kMaxSelWords) return cudaSuccess;
  a.has_corr = p.h != nullptr ? 1 : 0;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.corr_scale = p.corr_scale;
  a.causal = p.causal;
  a.o = p.o;
  a.lse = p.lse;
  a.status = status;
  a.trace = p.trace;
  a.debug_withhold_q = p.debug_withhold_q;
  a.bias = p.mode == 2 ? p.bias : nullptr;
  a.bias_bh_stride = p.bias_bh_stride;
  a.n_mirror = p.n_mirror;
  a.mirror_multicast = p.mirror_multicast;
  // multicast stores exist only on the staged (one-warpgroup) epilogue
  if (p.mirror_multicast && attn_warpgroups() != 1) return cudaSuccess;
  for (int mi = 0; mi < kMaxMirrors; ++mi) a.mirror[mi] = mi < p.n_mirror ? p.mirror[mi] : nullptr;
  a.pairs = p.mode == 1 ? p.pairs : nullptr;
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
  dim3 grid((a.nqb + 1) / 2, bh);
  cudaError_t err;
  if (attn_warpgroups() == 1)
    err = qv.dtype == B2_BF16 ? launch_nw<true, 1>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a)
                              : launch_nw<false, 1>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  else
    err = qv.dtype == B2_BF16 ? launch_nw<true, 2>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a)
                              : launch_nw<false, 2>(grid, stream, q_map, k_map, v_map, kc_map, vc_map, h_map, a);
  if (err != cudaSuccess) return err;
  *launched = true;
  return cudaGetLastError();
}

}  // namespace b2
