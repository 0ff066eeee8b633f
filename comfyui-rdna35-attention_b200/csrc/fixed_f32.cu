// Fixed 64-token block-diagonal attention for FP32 inputs (the CPU reference
// semantics of rdna35_block_attention/reference.py:159-200: FP32 scores,
// optional causal mask, softmax, FP32 P.V).  Tensor cores would round the
// operands, so this path runs on FP32 FMA units; the work is tiny (64x64xD
// per block) and bound by reading Q/K/V once plus launch latency.
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kFThreads = 256;
constexpr int kFRows = 32;  // query rows per CTA: half of a 64-token block

// One CTA = 32 query rows of one block against the block's 64 keys.  Thread
// (ty, tx) = (t / 16, t % 16) owns rows ty and ty + 16; its score columns are
// tx + 16 i (i < 4) and its output columns tx + 16 i (i < D / 16), so the
// shared-memory reads of K^T, P and V are conflict-free or broadcasts.
// Dot products and P.V sums run over d and key index in ascending order.
__global__ void __launch_bounds__(kFThreads)
fixed_f32_kernel(Rows q, Rows k, Rows v, Rows o, float scale, int causal, const float* __restrict__ bias,
                 int64_t bias_bh_stride) {
  extern __shared__ float fs[];
  const int D = q.dim;
  const int QP = D + 1;
  float* qs = fs;                 // [32][D + 1]
  float* kt = qs + kFRows * QP;   // [D][65]: K transposed
  float* vs = kt + D * 65;        // [64][D]
  float* ps = vs + kBlock * D;    // [32][65]
  const int start = blockIdx.x * kBlock;
  const int bh = blockIdx.y;
  const int r_base = blockIdx.z * kFRows;  // first query row of this CTA within the block
  const int len = min(kBlock, q.tokens - start);
  const int nr = min(kFRows, len - r_base);
  if (nr <= 0) return;  // the whole CTA leaves before any barrier
  const int d4n = D >> 2;
  // K and V rows: idx -> (key c = idx % 64, 4-float group idx / 64), so the
  // transposed K stores of a warp go to consecutive columns
  for (int idx = threadIdx.x; idx < kBlock * d4n; idx += kFThreads) {
    const int c = idx & 63;
    const int d4 = (idx >> 6) << 2;
    float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 vv4 = kv4;
    if (c < len) {
      kv4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(k.row(bh, start + c)) + d4);
      vv4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(v.row(bh, start + c)) + d4);
    }
    kt[(d4 + 0) * 65 + c] = kv4.x;
    kt[(d4 + 1) * 65 + c] = kv4.y;
    kt[(d4 + 2) * 65 + c] = kv4.z;
    kt[(d4 + 3) * 65 + c] = kv4.w;
    *reinterpret_cast<float4*>(vs + c * D + d4) = vv4;
  }
  for (int idx = threadIdx.x; idx < kFRows * d4n; idx += kFThreads) {
    const int r = idx / d4n;
    const int d4 = (idx - r * d4n) << 2;
    float4 qv4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nr) qv4 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(q.row(bh, start + r_base + r)) + d4);
    qs[r * QP + d4 + 0] = qv4.x;
    qs[r * QP + d4 + 1] = qv4.y;
    qs[r * QP + d4 + 2] = qv4.z;
    qs[r * QP + d4 + 3] = qv4.w;
  }
  __syncthreads();
  const int ty = threadIdx.x >> 4;
  const int tx = threadIdx.x & 15;
  const int r0 = ty;
  const int r1 = ty + 16;
  {
    float s0[4] = {0.f, 0.f, 0.f, 0.f};
    float s1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < D; ++d) {
      const float a0 = qs[r0 * QP + d];
      const float a1 = qs[r1 * QP + d];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float b = kt[d * 65 + tx + 16 * i];
        s0[i] = fmaf(a0, b, s0[i]);
        s1[i] = fmaf(a1, b, s1[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = tx + 16 * i;
      const bool bad0 = c >= len || (causal && c > r_base + r0);
      const bool bad1 = c >= len || (causal && c > r_base + r1);
      float x0 = bad0 ? -INFINITY : s0[i] * scale;
      float x1 = bad1 ? -INFINITY : s1[i] * scale;
      if (bias != nullptr) {  // mask terms of the row's own block, added after the causal mask
        const float* brow = bias + int64_t(bh) * bias_bh_stride + int64_t(start + r_base) * kBlock;
        if (r0 < nr) x0 += brow[r0 * kBlock + c];
        if (r1 < nr) x1 += brow[r1 * kBlock + c];
      }
      ps[r0 * 65 + c] = x0;
      ps[r1 * 65 + c] = x1;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int r = warp; r < kFRows; r += kFThreads / 32) {
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
    // a row with every key masked: NaN, as softmax over all -inf gives
    const float inv = sum > 0.f ? 1.f / sum : (bias != nullptr ? __int_as_float(0x7fc00000) : 0.f);
    ps[r * 65 + lane] = a * inv;
    ps[r * 65 + lane + 32] = b * inv;
  }
  __syncthreads();
  float o0[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float o1[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int c = 0; c < len; ++c) {
    const float p0 = ps[r0 * 65 + c];
    const float p1 = ps[r1 * 65 + c];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = tx + 16 * i;
      if (d < D) {
        const float b = vs[c * D + d];
        o0[i] = fmaf(p0, b, o0[i]);
        o1[i] = fmaf(p1, b, o1[i]);
      }
    }
  }
  float* out0 = r0 < nr ? reinterpret_cast<float*>(o.row(bh, start + r_base + r0)) : nullptr;
  float* out1 = r1 < nr ? reinterpret_cast<float*>(o.row(bh, start + r_base + r1)) : nullptr;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = tx + 16 * i;
    if (d < D) {
      if (out0) out0[d] = o0[i];
      if (out1) out1[d] = o1[i];
    }
  }
}

}  // namespace

cudaError_t launch_fixed_f32(const Rows& q, const Rows& k, const Rows& v, const Rows& o, int batch_heads,
                             float scale, int causal, const float* bias, int64_t bias_bh_stride,
                             cudaStream_t stream) {
  if (q.dim > 128 || (q.dim & 3) != 0) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float) * (kFRows * (q.dim + 1) + q.dim * 65 + kBlock * q.dim + kFRows * 65);
  cudaError_t err = ensure_smem(reinterpret_cast<const void*>(fixed_f32_kernel), static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  dim3 grid((q.tokens + kBlock - 1) / kBlock, batch_heads, kBlock / kFRows);
  fixed_f32_kernel<<<grid, kFThreads, smem, stream>>>(q, k, v, o, scale, causal, bias, bias_bh_stride);
  return cudaGetLastError();
}

}  // namespace b2
