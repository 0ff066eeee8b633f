// Fixed 64-token block-diagonal attention for FP32 inputs (the CPU reference
// semantics of rdna35_block_attention/reference.py:159-200: FP32 scores,
// optional causal mask, softmax, FP32 P.V).  Tensor cores would round the
// operands, so this path runs on FP32 FMA units; the work is tiny (64x64xD
// per block) and bound by reading Q/K/V once.
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kFThreads = 256;

__global__ void __launch_bounds__(kFThreads)
fixed_f32_kernel(Rows q, Rows k, Rows v, Rows o, float scale, int causal) {
  extern __shared__ float fs[];
  const int D = q.dim;
  const int DP = D + 1;
  float* qs = fs;
  float* ks = qs + kBlock * DP;
  float* vs = ks + kBlock * DP;
  float* ps = vs + kBlock * DP;  // [64][65]
  const int blk = blockIdx.x;
  const int bh = blockIdx.y;
  const int start = blk * kBlock;
  const int len = min(kBlock, q.tokens - start);
  for (int idx = threadIdx.x; idx < kBlock * D; idx += kFThreads) {
    const int r = idx / D;
    const int d = idx - r * D;
    float qv = 0.f, kv = 0.f, vv = 0.f;
    if (r < len) {
      qv = reinterpret_cast<const float*>(q.row(bh, start + r))[d];
      kv = reinterpret_cast<const float*>(k.row(bh, start + r))[d];
      vv = reinterpret_cast<const float*>(v.row(bh, start + r))[d];
    }
    qs[r * DP + d] = qv;
    ks[r * DP + d] = kv;
    vs[r * DP + d] = vv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kBlock * kBlock; idx += kFThreads) {
    const int r = idx >> 6;
    const int c = idx & 63;
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(qs[r * DP + d], ks[c * DP + d], acc);
    float sc = acc * scale;
    if (c >= len || (causal && c > r)) sc = -INFINITY;
    ps[r * 65 + c] = sc;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int r = warp; r < kBlock; r += kFThreads / 32) {
    float a = ps[r * 65 + lane];
    float b = ps[r * 65 + lane + 32];
    float mx = fmaxf(a, b);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float muse = mx == -INFINITY ? 0.f : mx;
    a = expf(a - muse);
    b = expf(b - muse);
    float sum = a + b;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    ps[r * 65 + lane] = a * inv;
    ps[r * 65 + lane + 32] = b * inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kBlock * D; idx += kFThreads) {
    const int r = idx / D;
    const int d = idx - r * D;
    if (r >= len) continue;
    float acc = 0.f;
    for (int c = 0; c < len; ++c) acc = fmaf(ps[r * 65 + c], vs[c * DP + d], acc);
    reinterpret_cast<float*>(o.row(bh, start + r))[d] = acc;
  }
}

}  // namespace

cudaError_t launch_fixed_f32(const Rows& q, const Rows& k, const Rows& v, const Rows& o, int batch_heads,
                             float scale, int causal, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (3 * kBlock * (q.dim + 1) + kBlock * 65);
  cudaError_t err = ensure_smem(reinterpret_cast<const void*>(fixed_f32_kernel), static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  dim3 grid((q.tokens + kBlock - 1) / kBlock, batch_heads);
  fixed_f32_kernel<<<grid, kFThreads, smem, stream>>>(q, k, v, o, scale, causal);
  return cudaGetLastError();
}

}  // namespace b2
