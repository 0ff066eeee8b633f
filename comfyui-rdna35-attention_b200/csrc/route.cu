// PISA routing: per query block i, score every key block j by its centroid
// dot product (plus the HYD covariance-norm bias) and keep the top-k blocks.
//
// Follows native/rdna35_pisa_ck/rdna35_pisa_ck/__init__.py:258-269 (HYD:
// BF16 centroids, FP32 accumulate, *scale, + log(h_norm + 1e-5), optional
// +inf sink, topk then ascending sort) and generic_pisa.py:172-184 (FP32
// centroids, no bias).  Ties at the cut resolve to the lower block index.
//
// One CTA owns 16 query blocks.  BF16 centroids (HYD): scores on the tensor
// cores (mma.sync, FP32 accumulate) straight from global memory; FP32
// centroids (generic): FP32 FMAs over centroids staged transposed in shared
// memory.  Then each warp selects the top-k of one row by a bitwise search
// for the k-th largest order-preserving integer key (redux.sync counts).
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kRows = 16;       // query blocks per CTA
constexpr int kThreadsR = 512;  // 16 warps: one query-block row each for the top-k
constexpr int kRowsPerWarp = kRows / (kThreadsR / 32);
constexpr int kFmaThreads = 256;  // FP32 path: 16 rows x 16 column lanes
constexpr int kColChunk = 128;  // key centroids staged per pass
constexpr int kDim = 128;
constexpr int kMaxBlocks = 1024;

// Float -> uint32 whose unsigned order is the float order.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// D(16x8, f32) += A(16x16, bf16, row-major) * B(16x8, bf16, col-major)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Top-k of one score row (blocks <= 32 * NM), as this lane's selection word:
// bit b of lane l's word <-> column 32 l + b.  The k-th largest order key T
// comes from a bitwise search from the top bit (the largest T with at least
// k keys >= T; a candidate with exactly k keys >= it ends the search: those
// keys are the top k and every other key is strictly below them); then every
// key > T plus the lowest-index keys == T up to k.  Lane l holds columns
// l + 32 m.  Equivalent to k rounds of "largest remaining, lowest index on
// ties".  NM bounds the unrolled loops (8 / 16 / 32 words of 32 columns).
template <int NM>
__device__ __forceinline__ uint32_t select_row(const float* srow, int blocks, int nm, int k, int lane) {
  uint32_t key[NM];
#pragma unroll
  for (int m = 0; m < NM; ++m) {
    const int j = lane + 32 * m;
    key[m] = (m < nm && j < blocks) ? order_key(srow[j]) : 0u;
  }
  uint32_t thr = 0u;
  bool exact = false;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = thr | (1u << bit);
    int c = 0;
#pragma unroll
    for (int m = 0; m < NM; ++m)
      if (m < nm) c += key[m] >= cand ? 1 : 0;
    const int total = static_cast<int>(__reduce_add_sync(0xffffffffu, static_cast<unsigned>(c)));
    if (total >= k) thr = cand;
    if (total == k) {
      exact = true;
      break;
    }
  }
  int gt = 0;
#pragma unroll
  for (int m = 0; m < NM; ++m)
    if (m < nm) gt += (exact ? key[m] >= thr : key[m] > thr) ? 1 : 0;
  int need = k - static_cast<int>(__reduce_add_sync(0xffffffffu, static_cast<unsigned>(gt)));
  uint32_t word = 0;
#pragma unroll
  for (int m = 0; m < NM; ++m) {
    if (m < nm) {
      const int j = lane + 32 * m;
      uint32_t bits = __ballot_sync(0xffffffffu, exact ? key[m] >= thr : key[m] > thr);
      uint32_t eq = exact ? 0u : __ballot_sync(0xffffffffu, j < blocks && key[m] == thr);
      while (need > 0 && eq != 0u) {  // ties at the cut: lowest index first
        bits |= eq & (~eq + 1u);
        eq &= eq - 1u;
        --need;
      }
      if (lane == m) word = bits;
    }
  }
  return word;
}

// Scores of kRows query blocks against every key block, then per-row top-k.
// Thread (r, cl) accumulates columns cl + 16*i of row r over d in order
// (FP32 FMA), reading q from a broadcast row and k from a transposed chunk.
__global__ void __launch_bounds__(kThreadsR, 2)
route_kernel(const void* __restrict__ qc, int qc_is_f32, const float* __restrict__ kc, int kc_round_bf16,
             const float* __restrict__ h_norm, int blocks, int dim, int k, float scale, int sink,
             int32_t* __restrict__ indices, uint32_t* __restrict__ sel_bits) {
  extern __shared__ __align__(16) float rs[];
  grid_dep_wait();
  const int words = (blocks + 31) >> 5;
  const int chunk = min(kColChunk, (blocks + 15) & ~15);  // columns staged per pass
  const int pitch = chunk + 1;
  const bool mma_path = !qc_is_f32 && kc_round_bf16;
  float* qrow = rs;                        // [16][128]          (FP32 path)
  float* kct = qrow + kRows * kDim;        // [128][pitch]       (FP32 path)
  float* scores = mma_path ? rs : kct + kDim * pitch;  // [16][blocks]
  (void)dim;
  const int bh = blockIdx.y;
  const int row0 = blockIdx.x * kRows;
  const int t = threadIdx.x;
  const int r = t >> 4;
  const int cl = t & 15;
  if (mma_path) {
    // BF16 centroids (HYD): exact bf16 products on the tensor cores with FP32
    // accumulation (mma.sync m16n8k16; the sum order differs from the
    // sequential one only by FP32 rounding).  Warp w owns 8-column tiles
    // w, w+8, ...; A (16 query rows x 128) stays in registers.
    const int warp = t >> 5;
    const int lane = t & 31;
    const int g = lane >> 2;        // fragment row / column group
    const int q2 = (lane & 3) * 2;  // fragment k pair
    const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(qc) + int64_t(bh) * blocks * kDim;
    uint32_t af[kDim / 16][4];
#pragma unroll
    for (int ks = 0; ks < kDim / 16; ++ks) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int rr = g + ((h & 1) ? 8 : 0);
        const int kk = ks * 16 + q2 + ((h & 2) ? 8 : 0);
        const int qi = row0 + rr;
        af[ks][h] = qi < blocks ? *reinterpret_cast<const uint32_t*>(qb + int64_t(qi) * kDim + kk) : 0u;
      }
    }
    const int ntiles = (blocks + 7) >> 3;
    for (int nt = warp; nt < ntiles; nt += kThreadsR / 32) {
      const int n = nt * 8 + g;  // key block of this lane's B fragment
      const float* kr = kc + (int64_t(bh) * blocks + min(n, blocks - 1)) * kDim;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < kDim / 16; ++ks) {
        const float2 lo = *reinterpret_cast<const float2*>(kr + ks * 16 + q2);
        const float2 hi = *reinterpret_cast<const float2*>(kr + ks * 16 + q2 + 8);
        mma_bf16_16816(d, af[ks], pack_bf16x2(lo.x, lo.y), pack_bf16x2(hi.x, hi.y));
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int rr = g + ((h & 2) ? 8 : 0);
        const int j = nt * 8 + q2 + (h & 1);
        if (j < blocks) {
          float sc = d[h] * scale;
          if (h_norm != nullptr) sc = sc + logf(h_norm[int64_t(bh) * blocks + j] + 1e-5f);
          scores[rr * blocks + j] = sc;
        }
      }
    }
  } else {
    for (int idx = t; idx < kRows * kDim; idx += kThreadsR) {
      const int rr = idx >> 7;
      const int d = idx & (kDim - 1);
      const int qi = row0 + rr;
      float val = 0.f;
      if (qi < blocks) {
        const int64_t off = (int64_t(bh) * blocks + qi) * kDim + d;
        val = qc_is_f32 ? static_cast<const float*>(qc)[off]
                        : __bfloat162float(static_cast<const __nv_bfloat16*>(qc)[off]);
      }
      qrow[idx] = val;
    }
    for (int c0 = 0; c0 < blocks; c0 += chunk) {
      __syncthreads();
      const int ncol = min(chunk, blocks - c0);
      // k rows read as float4 (coalesced), stored transposed
      for (int idx = t; idx < chunk * (kDim / 4); idx += kThreadsR) {
        const int j = idx >> 5;
        const int d4 = (idx & 31) * 4;
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < ncol) {
          val = *reinterpret_cast<const float4*>(kc + (int64_t(bh) * blocks + c0 + j) * kDim + d4);
          if (kc_round_bf16) {
            val.x = __bfloat162float(__float2bfloat16_rn(val.x));
            val.y = __bfloat162float(__float2bfloat16_rn(val.y));
            val.z = __bfloat162float(__float2bfloat16_rn(val.z));
            val.w = __bfloat162float(__float2bfloat16_rn(val.w));
          }
        }
        kct[(d4 + 0) * pitch + j] = val.x;
        kct[(d4 + 1) * pitch + j] = val.y;
        kct[(d4 + 2) * pitch + j] = val.z;
        kct[(d4 + 3) * pitch + j] = val.w;
      }
      __syncthreads();
      const int na = (ncol + 15) >> 4;  // accumulators in use (<= 16)
      if (t < kFmaThreads) {
      float acc[kColChunk / 16];
  #pragma unroll
      for (int i = 0; i < kColChunk / 16; ++i) acc[i] = 0.f;
      const float* qr = qrow + r * kDim;
  #pragma unroll 2
      for (int d = 0; d < kDim; ++d) {
        const float qv = qr[d];
        const float* kr = kct + d * pitch + cl;
  #pragma unroll
        for (int i = 0; i < kColChunk / 16; ++i)
          if (i < na) acc[i] = fmaf(qv, kr[16 * i], acc[i]);
      }
  #pragma unroll
      for (int i = 0; i < kColChunk / 16; ++i) {
        const int j = cl + 16 * i;
        if (i < na && j < ncol) {
          float sc = acc[i] * scale;
          if (h_norm != nullptr) sc = sc + logf(h_norm[int64_t(bh) * blocks + c0 + j] + 1e-5f);
          scores[r * blocks + c0 + j] = sc;
        }
      }
      }
    }
  }
  __syncthreads();
  // ---- per-row top-k: warp w handles rows kRowsPerWarp*w ...
  const int warp = t >> 5;
  const int lane = t & 31;
  for (int rr = kRowsPerWarp * warp; rr < kRowsPerWarp * (warp + 1); ++rr) {
    const int qi = row0 + rr;
    if (qi >= blocks) break;
    float* srow = scores + rr * blocks;
    if (sink != -2 && k > 0) {
      const int sj = sink < 0 ? blocks + sink : sink;
      if (lane == 0) srow[sj] = __int_as_float(0x7f800000);
      __syncwarp();
    }
    const int nm = (blocks + 31) >> 5;
    uint32_t word = 0;
    if (k > 0) {
      if (nm <= 8) word = select_row<8>(srow, blocks, nm, k, lane);
      else if (nm <= 16) word = select_row<16>(srow, blocks, nm, k, lane);
      else word = select_row<32>(srow, blocks, nm, k, lane);
    }
    const int64_t rowid = int64_t(bh) * blocks + qi;
    if (lane < words) sel_bits[rowid * words + lane] = word;
    const int cnt = lane < words ? __popc(word) : 0;
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int pos = incl - cnt;
    uint32_t wbits = word;
    while (wbits) {
      const int b = __ffs(wbits) - 1;
      wbits &= wbits - 1;
      indices[rowid * k + pos++] = lane * 32 + b;
    }
  }
}

// Pair query blocks so that the two blocks of an attention CTA share as many
// selected key blocks as possible (the CTA visits the union of both lists).
// One warp per (batch, head): blocks are taken in ascending order; each
// unpaired block is matched with the unpaired block of largest selection
// overlap (ties: lowest index).  pairs[bh][p] = (a, b), b = -1 for a single.
// Only overlaps with later blocks are ever read, so they are kept as the
// strict upper triangle: row a holds j = a+1 .. blocks-1.
__host__ __device__ __forceinline__ int tri_row(int a, int blocks) { return a * (blocks - 1) - (a * (a - 1)) / 2; }
// Row pitch of the selection bitsets in shared memory: odd, so that lanes
// reading the rows of 32 consecutive blocks hit 32 different banks.
__host__ __device__ __forceinline__ int bits_pitch(int words) { return words | 1; }

constexpr int kPairThreads = 512;

// Largest-overlap unpaired candidate j > a among this lane's columns
// j = lane + 32 m (m < W, a compile-time bound so all loads issue together).
template <int W>
__device__ __forceinline__ uint32_t best_candidate(const uint8_t* row, int a, int blocks, int words, int lane,
                                                   uint32_t mine) {
  uint32_t best = 0u;
#pragma unroll
  for (int m = 0; m < W; ++m) {
    const int j = (m << 5) + lane;
    const bool cand = m < words && j > a && j < blocks && !((mine >> m) & 1u);
    const uint32_t o = cand ? row[j] : 0u;
    if (cand) best = max(best, (o << 16) | (0xffffu - static_cast<uint32_t>(j)));
  }
  return best;
}

// Upper-triangle overlaps popc(sel[a] & sel[j]), j > a: warp w takes rows
// a = w, w + nwarps, ...; row a's words stay in registers.
template <int W>
__device__ __forceinline__ void overlap_rows(const uint32_t* bits, uint8_t* tri, int blocks, int words, int pitch,
                                             int warp, int nwarps, int lane) {
  for (int a = warp; a < blocks - 1; a += nwarps) {
    uint32_t ra[W];
#pragma unroll
    for (int w = 0; w < W; ++w) ra[w] = w < words ? bits[a * pitch + w] : 0u;
    uint8_t* row = tri + tri_row(a, blocks) - (a + 1);
    for (int j = a + 1 + lane; j < blocks; j += 32) {
      const uint32_t* bj = bits + j * pitch;
      int o = 0;
#pragma unroll
      for (int w = 0; w < W; ++w)
        if (w < words) o += __popc(ra[w] & bj[w]);
      row[j] = static_cast<uint8_t>(min(o, 255));
    }
  }
}

__global__ void __launch_bounds__(kPairThreads) pair_kernel(const uint32_t* __restrict__ sel_bits, int blocks,
                                                              int32_t* __restrict__ pairs) {
  extern __shared__ uint32_t ps[];
  grid_dep_wait();
  const int words = (blocks + 31) >> 5;
  const int pitch = bits_pitch(words);
  uint32_t* bits = ps;                                              // [blocks][pitch]
  uint8_t* tri = reinterpret_cast<uint8_t*>(bits + blocks * pitch);  // upper-triangle overlaps (<= 255)
  const int bh = blockIdx.x;
  const int t = threadIdx.x;
  for (int i = t; i < blocks * words; i += blockDim.x) {
    const int r = i / words;
    bits[r * pitch + (i - r * words)] = sel_bits[int64_t(bh) * blocks * words + i];
  }
  __syncthreads();
  if (words <= 8) overlap_rows<8>(bits, tri, blocks, words, pitch, t >> 5, blockDim.x >> 5, t & 31);
  else if (words <= 16) overlap_rows<16>(bits, tri, blocks, words, pitch, t >> 5, blockDim.x >> 5, t & 31);
  else overlap_rows<32>(bits, tri, blocks, words, pitch, t >> 5, blockDim.x >> 5, t & 31);
  __syncthreads();
  if (t >= 32) return;
  // greedy matching by one warp; lane l owns candidates j = l + 32*m and keeps
  // their "already paired" flags in the register mask `mine`
  const int lane = t;
  uint32_t mine = 0;
  int np = 0;
  for (int a = 0; a < blocks; ++a) {
    const uint32_t a_used = __shfl_sync(0xffffffffu, (mine >> (a >> 5)) & 1u, a & 31);
    if (a_used) continue;
    // candidate key = overlap << 16 | (0xffff - j): one warp max reduction
    // picks the largest overlap, ties to the lowest index; 0 = no candidate
    const uint8_t* row = tri + tri_row(a, blocks) - (a + 1);  // row[j] valid for j > a
    const uint32_t best = words <= 8 ? best_candidate<8>(row, a, blocks, words, lane, mine)
                                     : best_candidate<32>(row, a, blocks, words, lane, mine);
    const uint32_t wbest = __reduce_max_sync(0xffffffffu, best);
    const int b = wbest == 0u ? -1 : static_cast<int>(0xffffu - (wbest & 0xffffu));
    if ((a & 31) == lane) mine |= 1u << (a >> 5);
    if (b >= 0 && (b & 31) == lane) mine |= 1u << (b >> 5);
    if (lane == 0) {
      int32_t* dst = pairs + (int64_t(bh) * ((blocks + 1) / 2) + np) * 2;
      dst[0] = a;
      dst[1] = b;
    }
    ++np;
  }
}

}  // namespace

size_t pair_smem_bytes(int blocks) {
  const size_t pitch = bits_pitch((blocks + 31) / 32);
  return sizeof(uint32_t) * size_t(blocks) * pitch + size_t(blocks) * (blocks - 1) / 2;
}

bool pair_supported(int blocks) { return blocks >= 1 && blocks <= 1024 && pair_smem_bytes(blocks) <= 227 * 1024; }

cudaError_t launch_pair(const uint32_t* sel_bits, int batch_heads, int blocks, int32_t* pairs, cudaStream_t stream) {
  if (!pair_supported(blocks)) return cudaErrorInvalidValue;
  const size_t smem = pair_smem_bytes(blocks);
  cudaError_t err = ensure_smem(reinterpret_cast<const void*>(pair_kernel), int(smem));
  if (err != cudaSuccess) return err;
  return launch_pdl(pair_kernel, dim3(batch_heads), dim3(kPairThreads), smem, stream, sel_bits, blocks, pairs);
}

cudaError_t launch_route(const void* qc, int qc_dtype, const float* kc, int kc_round, const float* h_norm,
                         int batch_heads, int blocks, int dim, int k, float scale, int sink, int32_t* indices,
                         uint32_t* sel_bits, cudaStream_t stream) {
  if (blocks > kMaxBlocks) return cudaErrorInvalidValue;
  if (dim != kDim) return cudaErrorInvalidValue;
  const int chunk = blocks < kColChunk ? ((blocks + 15) & ~15) : kColChunk;
  const bool mma_path = qc_dtype != B2_F32 && kc_round == B2_BF16;
  const size_t smem = sizeof(float) * ((mma_path ? 0 : kRows * kDim + kDim * (chunk + 1)) + kRows * blocks);
  cudaError_t err = ensure_smem(reinterpret_cast<const void*>(route_kernel), static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  dim3 grid((blocks + kRows - 1) / kRows, batch_heads);
  return launch_pdl(route_kernel, grid, dim3(kThreadsR), smem, stream, qc, static_cast<int>(qc_dtype == B2_F32), kc,
                    static_cast<int>(kc_round == B2_BF16), h_norm, blocks, dim, k, scale, sink, indices, sel_bits);
}

}  // namespace b2
