// PISA routing: per query block i, score every key block j by its centroid
// dot product (plus the HYD covariance-norm bias) and keep the top-k blocks.
//
// Follows native/rdna35_pisa_ck/rdna35_pisa_ck/__init__.py:258-269 (HYD:
// BF16 centroids, FP32 accumulate, *scale, + log(h_norm + 1e-5), optional
// +inf sink, topk then ascending sort) and generic_pisa.py:172-184 (FP32
// centroids, no bias).  Ties at the cut resolve to the lower block index.
//
// One CTA owns 16 query blocks: scores are built in shared memory 128 key
// centroids at a time (staged transposed so the 16 column lanes of a row read
// consecutive words), then each warp runs k rounds of warp-wide argmax for two
// rows.
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kRows = 16;       // query blocks per CTA
constexpr int kThreadsR = 256;  // 16 rows x 16 column lanes
constexpr int kColChunk = 256;  // key centroids staged per pass
constexpr int kDim = 128;
constexpr int kMaxBlocks = 1024;

// Scores of kRows query blocks against every key block, then per-row top-k.
// Thread (r, cl) accumulates columns cl + 16*i of row r over d in order
// (FP32 FMA), reading q from a broadcast row and k from a transposed chunk.
__global__ void __launch_bounds__(kThreadsR)
route_kernel(const void* __restrict__ qc, int qc_is_f32, const float* __restrict__ kc, int kc_round_bf16,
             const float* __restrict__ h_norm, int blocks, int dim, int k, float scale, int sink,
             int32_t* __restrict__ indices, uint32_t* __restrict__ sel_bits) {
  extern __shared__ __align__(16) float rs[];
  const int words = (blocks + 31) >> 5;
  const int chunk = min(kColChunk, (blocks + 15) & ~15);  // columns staged per pass
  const int pitch = chunk + 1;
  float* qrow = rs;                        // [16][128]
  float* kct = qrow + kRows * kDim;        // [128][pitch]
  float* scores = kct + kDim * pitch;      // [16][blocks]
  (void)dim;
  const int bh = blockIdx.y;
  const int row0 = blockIdx.x * kRows;
  const int t = threadIdx.x;
  const int r = t >> 4;
  const int cl = t & 15;
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
  __syncthreads();
  // ---- per-row top-k: warp w handles rows 2w and 2w+1
  const int warp = t >> 5;
  const int lane = t & 31;
  for (int rr = 2 * warp; rr < 2 * warp + 2; ++rr) {
    const int qi = row0 + rr;
    if (qi >= blocks) break;
    float* srow = scores + rr * blocks;
    if (sink != -2 && k > 0) {
      const int sj = sink < 0 ? blocks + sink : sink;
      if (lane == 0) srow[sj] = __int_as_float(0x7f800000);
      __syncwarp();
    }
    uint32_t taken = 0;  // bit m <-> column lane + 32*m
    for (int round = 0; round < k; ++round) {
      float best = -__int_as_float(0x7f800000);
      int best_j = 0x7fffffff;
      for (int m = 0, j = lane; j < blocks; ++m, j += 32) {
        if (taken & (1u << m)) continue;
        const float val = srow[j];
        if (val > best || (val == best && j < best_j)) {
          best = val;
          best_j = j;
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oj = __shfl_xor_sync(0xffffffffu, best_j, off);
        if (ov > best || (ov == best && oj < best_j)) {
          best = ov;
          best_j = oj;
        }
      }
      if (best_j != 0x7fffffff && (best_j & 31) == lane) taken |= 1u << (best_j >> 5);
    }
    uint32_t word = 0;
    for (int w = 0; w < words; ++w) {
      const uint32_t bits = __ballot_sync(0xffffffffu, (taken >> w) & 1u);
      if (lane == w) word = bits;
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
__global__ void __launch_bounds__(256) pair_kernel(const uint32_t* __restrict__ sel_bits, int blocks,
                                                     int32_t* __restrict__ pairs) {
  extern __shared__ uint32_t ps[];
  const int words = (blocks + 31) >> 5;
  uint32_t* bits = ps;                                             // [blocks][words]
  uint8_t* ov = reinterpret_cast<uint8_t*>(bits + blocks * words);  // [blocks][blocks] overlaps (<= 255)
  const int bh = blockIdx.x;
  const int t = threadIdx.x;
  for (int i = t; i < blocks * words; i += blockDim.x) bits[i] = sel_bits[int64_t(bh) * blocks * words + i];
  __syncthreads();
  for (int idx = t; idx < blocks * blocks; idx += blockDim.x) {
    const int a = idx / blocks;
    const int j = idx - a * blocks;
    int o = 0;
    for (int w = 0; w < words; ++w) o += __popc(bits[a * words + w] & bits[j * words + w]);
    ov[idx] = static_cast<uint8_t>(min(o, 255));
  }
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
    int best = -1, best_j = 0x7fffffff;
    const uint8_t* row = ov + a * blocks;
    for (int m = (a + 1) >> 5; (m << 5) < blocks; ++m) {
      const int j = (m << 5) + lane;
      if (j <= a || j >= blocks || ((mine >> m) & 1u)) continue;
      const int o = row[j];
      if (o > best) {
        best = o;
        best_j = j;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const int ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oj = __shfl_xor_sync(0xffffffffu, best_j, off);
      if (ob > best || (ob == best && oj < best_j)) {
        best = ob;
        best_j = oj;
      }
    }
    const int b = best_j == 0x7fffffff ? -1 : best_j;
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

cudaError_t launch_pair(const uint32_t* sel_bits, int batch_heads, int blocks, int32_t* pairs, cudaStream_t stream) {
  const int words = (blocks + 31) / 32;
  const size_t smem = sizeof(uint32_t) * size_t(blocks) * words + size_t(blocks) * blocks;
  if (smem > 227 * 1024 || blocks > 1024) return cudaErrorInvalidValue;
  cudaError_t err = ensure_smem(reinterpret_cast<const void*>(pair_kernel), int(smem));
  if (err != cudaSuccess) return err;
  pair_kernel<<<batch_heads, 256, smem, stream>>>(sel_bits, blocks, pairs);
  return cudaGetLastError();
}

cudaError_t launch_route(const void* qc, int qc_dtype, const float* kc, int kc_round, const float* h_norm,
                         int batch_heads, int blocks, int dim, int k, float scale, int sink, int32_t* indices,
                         uint32_t* sel_bits, cudaStream_t stream) {
  if (blocks > kMaxBlocks) return cudaErrorInvalidValue;
  if (dim != kDim) return cudaErrorInvalidValue;
  const int chunk = blocks < kColChunk ? ((blocks + 15) & ~15) : kColChunk;
  const size_t smem = sizeof(float) * (kRows * kDim + kDim * (chunk + 1) + kRows * blocks);
  cudaError_t err = ensure_smem(reinterpret_cast<const void*>(route_kernel), static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  dim3 grid((blocks + kRows - 1) / kRows, batch_heads);
  route_kernel<<<grid, kThreadsR, smem, stream>>>(qc, qc_dtype == B2_F32, kc, kc_round == B2_BF16, h_norm,
                                                         blocks, dim, k, scale, sink, indices, sel_bits);
  return cudaGetLastError();
}

}  // namespace b2
