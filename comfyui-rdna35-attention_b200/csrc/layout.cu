// Bandwidth-bound layout kernels: tiled pack / unpack of [B,H,T,D] rows, the
// standalone LSE-weighted merge epilogue, the MiniMax-H3 interleaved-QKV pack
// and the centroid preparation used by the fused attention kernel.  All move
// 16-byte vectors; a warp covers whole 128- or 256-byte rows so every global
// access is a fully used sector.
#include "common.cuh"

namespace b2 {
namespace {

// dst[bh][t][:] = src.row(bh, t)  (pisa_kernels.cu:247-272)
__global__ void pack_rows_kernel(Rows src, char* __restrict__ dst, int64_t nvec, int vec_per_row) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const int64_t row = i / vec_per_row;
    const int vec = static_cast<int>(i - row * vec_per_row);
    const int bh = static_cast<int>(row / src.tokens);
    const int t = static_cast<int>(row - int64_t(bh) * src.tokens);
    const uint4 val = *reinterpret_cast<const uint4*>(src.row(bh, t) + vec * 16);
    *reinterpret_cast<uint4*>(dst + i * 16) = val;
  }
}

// dst.row(bh, t) = src[bh][t][:]  (pisa_kernels.cu:275-293)
__global__ void unpack_rows_kernel(const char* __restrict__ src, Rows dst, int64_t nvec, int vec_per_row) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const int64_t row = i / vec_per_row;
    const int vec = static_cast<int>(i - row * vec_per_row);
    const int bh = static_cast<int>(row / dst.tokens);
    const int t = static_cast<int>(row - int64_t(bh) * dst.tokens);
    *reinterpret_cast<uint4*>(dst.row(bh, t) + vec * 16) = *reinterpret_cast<const uint4*>(src + i * 16);
  }
}

// LSE-weighted merge (pisa_kernels.cu:296-340), 8 output elements per thread.
template <typename T>
__global__ void merge_kernel(const T* __restrict__ exact, const float* __restrict__ exact_lse,
                             const T* __restrict__ approx, const float* __restrict__ approx_lse,
                             const float* __restrict__ corr, Rows dst, int64_t nvec, int vec_per_row) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const int64_t row = i / vec_per_row;
    const int vec = static_cast<int>(i - row * vec_per_row);
    const int bh = static_cast<int>(row / dst.tokens);
    const int t = static_cast<int>(row - int64_t(bh) * dst.tokens);
    const float le = exact_lse[row];
    const float la = approx_lse[row];
    const float mx = fmaxf(le, la);
    const float total = mx + logf(expf(le - mx) + expf(la - mx));
    const float we = expf(le - total);
    const float wa = expf(la - total);
    const int64_t e0 = i * 8;
    const uint4 ev = *reinterpret_cast<const uint4*>(exact + e0);
    const uint4 av = *reinterpret_cast<const uint4*>(approx + e0);
    const float4 c0 = *reinterpret_cast<const float4*>(corr + e0);
    const float4 c1 = *reinterpret_cast<const float4*>(corr + e0 + 4);
    const T* ep = reinterpret_cast<const T*>(&ev);
    const T* ap = reinterpret_cast<const T*>(&av);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    uint4 outv;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float m0 = Cvt<T>::to_f(ep[e]) * we + Cvt<T>::to_f(ap[e]) * wa + cv[e] * wa;
      const float m1 = Cvt<T>::to_f(ep[e + 1]) * we + Cvt<T>::to_f(ap[e + 1]) * wa + cv[e + 1] * wa;
      ow[e / 2] = Cvt<T>::pack2(m0, m1);
    }
    *reinterpret_cast<uint4*>(dst.row(bh, t) + vec * 16) = outv;
  }
}

// kc16 = round(kc); vc16 = HYD ? vstat : round(vsum / len)
template <typename T>
__global__ void centroid_prep_kernel(const float* __restrict__ kc, const void* __restrict__ vstat, int vstat_is_sum,
                                     int blocks, int tokens, int dim, int64_t n, T* __restrict__ kc16,
                                     T* __restrict__ vc16) {
  grid_dep_wait();
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    kc16[i] = Cvt<T>::from_f(kc[i]);
    if (vstat_is_sum) {
      const int blk = static_cast<int>((i / dim) % blocks);
      const float len = static_cast<float>(min(kBlock, tokens - blk * kBlock));
      vc16[i] = Cvt<T>::from_f(static_cast<const float*>(vstat)[i] / len);
    } else {
      vc16[i] = static_cast<const T*>(vstat)[i];
    }
  }
}

// Diagonal-block bias of an attention mask (reference.py:114-156 slicing +
// the bool masked_fill / float add of reference.py:182-186): for every mask
// row (bh, t) of the [BHm, T, T] mask, the 64 entries of t's own key block,
// as FP32 additive terms: bool True -> 0, False -> -inf, float values as
// they are; columns past a ragged last block -> -inf.  One thread per
// (row, 4 columns).
template <typename M>
__device__ __forceinline__ float mask_term(const M* p) {
  return Cvt<M>::to_f(*p);
}
template <>
__device__ __forceinline__ float mask_term<bool>(const bool* p) {
  return *reinterpret_cast<const unsigned char*>(p) ? 0.f : -INFINITY;
}
template <>
__device__ __forceinline__ float mask_term<float>(const float* p) {
  return *p;
}

template <typename M>
__global__ void block_bias_kernel(const M* __restrict__ mask, int64_t s_bh, int64_t s_row, int64_t s_col, int tokens,
                                  int64_t n, float* __restrict__ bias) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t row = i >> 4;  // (bh, t)
    const int c0 = static_cast<int>(i & 15) * 4;
    const int bh = static_cast<int>(row / tokens);
    const int t = static_cast<int>(row - int64_t(bh) * tokens);
    const int start = (t / kBlock) * kBlock;
    const int len = min(kBlock, tokens - start);
    const M* src = mask + int64_t(bh) * s_bh + int64_t(t) * s_row;
    float vals[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + e;
      vals[e] = c < len ? mask_term<M>(src + int64_t(start + c) * s_col) : -INFINITY;
    }
    *reinterpret_cast<float4*>(bias + row * kBlock + c0) = make_float4(vals[0], vals[1], vals[2], vals[3]);
  }
}

inline int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  const int64_t cap = 148 * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace

cudaError_t launch_pack_rows(const Rows& src, int batch_heads, void* dst, cudaStream_t stream) {
  const int vpr = src.dim * src.esize / 16;
  const int64_t nvec = int64_t(batch_heads) * src.tokens * vpr;
  pack_rows_kernel<<<grid_for(nvec, 256), 256, 0, stream>>>(src, static_cast<char*>(dst), nvec, vpr);
  return cudaGetLastError();
}

cudaError_t launch_unpack_rows(const void* src, const Rows& dst, int batch_heads, cudaStream_t stream) {
  const int vpr = dst.dim * dst.esize / 16;
  const int64_t nvec = int64_t(batch_heads) * dst.tokens * vpr;
  unpack_rows_kernel<<<grid_for(nvec, 256), 256, 0, stream>>>(static_cast<const char*>(src), dst, nvec, vpr);
  return cudaGetLastError();
}

cudaError_t launch_merge(const void* exact, const float* exact_lse, const void* approx, const float* approx_lse,
                         const float* corr, const Rows& dst, int dtype, int batch_heads, cudaStream_t stream) {
  const int vpr = dst.dim / 8;
  const int64_t nvec = int64_t(batch_heads) * dst.tokens * vpr;
  if (dtype == B2_BF16)
    merge_kernel<__nv_bfloat16><<<grid_for(nvec, 256), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(exact), exact_lse, static_cast<const __nv_bfloat16*>(approx), approx_lse,
        corr, dst, nvec, vpr);
  else
    merge_kernel<__half><<<grid_for(nvec, 256), 256, 0, stream>>>(static_cast<const __half*>(exact), exact_lse,
                                                                  static_cast<const __half*>(approx), approx_lse,
                                                                  corr, dst, nvec, vpr);
  return cudaGetLastError();
}

cudaError_t launch_block_bias(const void* mask, int mask_dtype, int64_t s_bh, int64_t s_row, int64_t s_col,
                              int mask_rows_bh, int tokens, float* bias, cudaStream_t stream) {
  const int64_t n = int64_t(mask_rows_bh) * tokens * 16;
  const int g = grid_for(n, 256);
  switch (mask_dtype) {
    case B2_MASK_BOOL:
      block_bias_kernel<bool><<<g, 256, 0, stream>>>(static_cast<const bool*>(mask), s_bh, s_row, s_col, tokens, n,
                                                     bias);
      break;
    case B2_MASK_F32:
      block_bias_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(mask), s_bh, s_row, s_col, tokens,
                                                      n, bias);
      break;
    case B2_MASK_F16:
      block_bias_kernel<__half><<<g, 256, 0, stream>>>(static_cast<const __half*>(mask), s_bh, s_row, s_col, tokens,
                                                       n, bias);
      break;
    default:
      block_bias_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(mask), s_bh, s_row,
                                                              s_col, tokens, n, bias);
  }
  return cudaGetLastError();
}

cudaError_t launch_centroid_prep(const float* kc, const void* vstat, int vstat_is_sum, int batch_heads, int blocks,
                                 int tokens, int dim, int dtype, void* kc16, void* vc16, cudaStream_t stream) {
  const int64_t n = int64_t(batch_heads) * blocks * dim;
  if (dtype == B2_BF16)
    return launch_pdl(centroid_prep_kernel<__nv_bfloat16>, dim3(grid_for(n, 256)), dim3(256), 0, stream, kc, vstat,
                      vstat_is_sum, blocks, tokens, dim, n, static_cast<__nv_bfloat16*>(kc16),
                      static_cast<__nv_bfloat16*>(vc16));
  return launch_pdl(centroid_prep_kernel<__half>, dim3(grid_for(n, 256)), dim3(256), 0, stream, kc, vstat,
                    vstat_is_sum, blocks, tokens, dim, n, static_cast<__half*>(kc16), static_cast<__half*>(vc16));
}

}  // namespace b2
