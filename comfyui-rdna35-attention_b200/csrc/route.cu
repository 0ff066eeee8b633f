// PISA routing: per query block i, score every key block j by its centroid
// dot product (plus the HYD covariance-norm bias) and keep the top-k blocks.
//
// Follows native/rdna35_pisa_ck/rdna35_pisa_ck/__init__.py:258-269 (HYD:
// BF16 centroids, FP32 accumulate, *scale, + log(h_norm + 1e-5), optional
// +inf sink, topk then ascending sort) and generic_pisa.py:172-184 (FP32
// centroids, no bias).  Ties at the cut resolve to the lower block index.
//
// One warp owns one query block.  Scores for the CTA's 8 rows are built in
// shared memory in 64-column chunks (key centroids staged transposed so lanes
// read consecutive columns), then each warp runs k rounds of warp-wide argmax.
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kRouteWarps = 8;
constexpr int kChunk = 64;
constexpr int kMaxBlocks = 1024;

__global__ void __launch_bounds__(kRouteWarps * 32)
route_kernel(const void* __restrict__ qc, int qc_is_f32, const float* __restrict__ kc, int kc_round_bf16,
             const float* __restrict__ h_norm, int blocks, int dim, int k, float scale, int sink,
             int32_t* __restrict__ indices, uint32_t* __restrict__ sel_bits) {
  extern __shared__ __align__(16) float rs[];
  const int words = (blocks + 31) >> 5;
  float* qrow = rs;                                  // [8][dim]
  float* kct = qrow + kRouteWarps * dim;             // [dim][kChunk+1]
  float* scores = kct + dim * (kChunk + 1);          // [8][blocks]
  const int bh = blockIdx.y;
  const int row0 = blockIdx.x * kRouteWarps;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nthreads = kRouteWarps * 32;

  for (int idx = threadIdx.x; idx < kRouteWarps * dim; idx += nthreads) {
    const int r = idx / dim;
    const int d = idx - r * dim;
    const int qi = row0 + r;
    float val = 0.f;
    if (qi < blocks) {
      const int64_t off = (int64_t(bh) * blocks + qi) * dim + d;
      val = qc_is_f32 ? static_cast<const float*>(qc)[off]
                      : __bfloat162float(static_cast<const __nv_bfloat16*>(qc)[off]);
    }
    qrow[idx] = val;
  }
  for (int c0 = 0; c0 < blocks; c0 += kChunk) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kChunk * dim; idx += nthreads) {
      const int j = idx / dim;
      const int d = idx - j * dim;
      float val = 0.f;
      if (c0 + j < blocks) {
        val = kc[(int64_t(bh) * blocks + c0 + j) * dim + d];
        if (kc_round_bf16) val = __bfloat162float(__float2bfloat16_rn(val));
      }
      kct[d * (kChunk + 1) + j] = val;
    }
    __syncthreads();
    for (int jj = lane; jj < kChunk; jj += 32) {
      const int j = c0 + jj;
      if (j >= blocks) break;
      float acc = 0.f;
      const float* qr = qrow + warp * dim;
      for (int d = 0; d < dim; ++d) acc = fmaf(qr[d], kct[d * (kChunk + 1) + jj], acc);
      float sc = acc * scale;
      if (h_norm != nullptr) sc = sc + logf(h_norm[int64_t(bh) * blocks + j] + 1e-5f);
      scores[warp * blocks + j] = sc;
    }
  }
  __syncwarp();
  const int qi = row0 + warp;
  if (qi >= blocks) return;
  float* srow = scores + warp * blocks;
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
  // transpose "taken" (per lane, column lane+32m) into words (column 32w+l)
  uint32_t word = 0;
  for (int w = 0; w < words; ++w) {
    const uint32_t bits = __ballot_sync(0xffffffffu, (taken >> w) & 1u);
    if (lane == w) word = bits;
  }
  const int64_t rowid = int64_t(bh) * blocks + qi;
  if (lane < words) sel_bits[rowid * words + lane] = word;
  // ascending index list: exclusive prefix of popcounts across words
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

}  // namespace

cudaError_t launch_route(const void* qc, int qc_dtype, const float* kc, int kc_round, const float* h_norm,
                         int batch_heads, int blocks, int dim, int k, float scale, int sink, int32_t* indices,
                         uint32_t* sel_bits, cudaStream_t stream) {
  if (blocks > kMaxBlocks) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float) * (kRouteWarps * dim + dim * (kChunk + 1) + kRouteWarps * blocks);
  cudaError_t err = cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  dim3 grid((blocks + kRouteWarps - 1) / kRouteWarps, batch_heads);
  route_kernel<<<grid, kRouteWarps * 32, smem, stream>>>(qc, qc_dtype == B2_F32, kc, kc_round == B2_BF16, h_norm,
                                                         blocks, dim, k, scale, sink, indices, sel_bits);
  return cudaGetLastError();
}

}  // namespace b2
