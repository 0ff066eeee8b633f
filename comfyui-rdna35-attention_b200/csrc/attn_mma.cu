// Flash-attention forward over a per-CTA list of 64-key tiles, with the PISA
// centroid tail and first-order correction fused into the same online
// softmax.  Tensor-core path: warp-level mma.sync m16n8k16 (16-bit inputs,
// FP32 accumulate), cp.async double-buffered K/V tiles, P kept in registers.
//
// One CTA = 64 query rows (4 warps x 16 rows) of one (batch, head).  Tile
// sources, in processing order:
//   1. tail tiles (PISA only): 64 key-block centroids per tile; logit =
//      q.kc*scale + log(len_j), blocks selected as exact are masked
//      (rdna35_pisa_ck/__init__.py:139-164, score_mod at :147-152);
//   2. key tiles: the selected exact blocks (mode LIST, __init__.py:286-298),
//      every key tile (mode ALL, triton_kernel.py:113-160) or the query
//      block's own block (mode DIAG, triton_kernel.py:53-100).
// The tail mass (sum of tail probabilities, rescaled with the running max)
// weights the correction q.H*scale/T added at the end, which equals the
// LSE-weighted merge of pisa_kernels.cu:317-339 in exact arithmetic.
#include "kernels.h"

namespace b2 {


namespace {

constexpr int kM = 64;
constexpr int kN = 64;
constexpr int kThreads = 128;

template <typename T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <int D>
struct TileDesc {
  static constexpr int P = D + 8;  // padded pitch (elements)
};

// Stage one 64-row tile of K and V (or of the centroids) into shared memory.
template <int D>
__device__ __forceinline__ void load_kv_tile(const AttnParams& p, int bh, int qblk, int tile, int ntail,
                                             char* ks, char* vs) {
  constexpr int P = TileDesc<D>::P;
  constexpr int VEC = D / 8;  // 16-byte vectors per row
  const bool tail = tile < ntail;
  int start = 0, len = 0;
  if (tail) {
    start = tile * kN;
    len = min(kN, p.nb - start);
  } else {
    const int t = tile - ntail;
    int blk = t;
    if (p.mode == 1) blk = p.indices[(int64_t(bh) * ((p.tq + kM - 1) / kM) + qblk) * p.nsel + t];
    else if (p.mode == 2) blk = qblk;
    blk = min(max(blk, 0), (p.tk + kN - 1) / kN - 1);
    start = blk * kN;
    len = min(kN, p.tk - start);
  }
  for (int idx = threadIdx.x; idx < 2 * kN * VEC; idx += kThreads) {
    const int which = idx / (kN * VEC);
    const int rem = idx - which * kN * VEC;
    const int r = rem / VEC;
    const int vec = rem - r * VEC;
    const bool valid = r < len;
    const char* src;
    if (tail) {
      const char* base = static_cast<const char*>(which == 0 ? p.kc : p.vc);
      src = base + ((int64_t(bh) * p.nb + start + (valid ? r : 0)) * D) * 2 + vec * 16;
    } else {
      const Rows& rows = which == 0 ? p.k : p.v;
      src = valid ? rows.row(bh, start + r) + vec * 16 : rows.base;
    }
    char* dst = (which == 0 ? ks : vs) + (r * P + vec * 8) * 2;
    cp_async16(smem_u32(dst), src, valid ? 16 : 0);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
attn_kernel(const AttnParams p) {
  constexpr int P = TileDesc<D>::P;
  constexpr int KSTEPS = D / 16;  // QK^T k-steps
  constexpr int NT = D / 8;       // output n-tiles
  extern __shared__ __align__(16) char smem[];
  T* qs = reinterpret_cast<T*>(smem);
  T* kv = qs + kM * P;  // [stage][K|V][64][P]
  const int qblk = blockIdx.x;
  const int bh = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = qblk * kM;
  const int qlen = min(kM, p.tq - q0);

  const int ntail = p.nb > 0 ? (p.nb + kN - 1) / kN : 0;
  int nmain;
  if (p.mode == 0) nmain = (p.tk + kN - 1) / kN;
  else if (p.mode == 1) nmain = p.nsel;
  else nmain = 1;
  const int ntiles = ntail + nmain;

  // ---- Q tile
  {
    constexpr int VEC = D / 8;
    for (int idx = threadIdx.x; idx < kM * VEC; idx += kThreads) {
      const int r = idx / VEC;
      const int vec = idx - r * VEC;
      const bool valid = r < qlen;
      const char* src = valid ? p.q.row(bh, q0 + r) + vec * 16 : p.q.base;
      cp_async16(smem_u32(&qs[r * P + vec * 8]), src, valid ? 16 : 0);
    }
  }
  if (ntiles > 0) load_kv_tile<D>(p, bh, qblk, 0, ntail, reinterpret_cast<char*>(kv),
                                  reinterpret_cast<char*>(kv + kN * P));
  cp_async_commit();

  const uint32_t* selw = nullptr;
  if (ntail > 0) selw = p.sel_bits + (int64_t(bh) * ((p.tq + kM - 1) / kM) + qblk) * ((p.nb + 31) >> 5);

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  float tmass[2] = {0.f, 0.f};
  uint32_t qf[KSTEPS][4];
  const int mat = lane >> 3;
  const int g = lane >> 2;
  const int cq = 2 * (lane & 3);

  for (int t = 0; t < ntiles; ++t) {
    const int stage = t & 1;
    if (t + 1 < ntiles) {
      T* kn = kv + ((stage ^ 1) * 2) * kN * P;
      load_kv_tile<D>(p, bh, qblk, t + 1, ntail, reinterpret_cast<char*>(kn), reinterpret_cast<char*>(kn + kN * P));
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int r = warp * 16 + (lane & 7) + ((mat & 1) << 3);
        const int c = ks * 16 + ((mat >> 1) << 3);
        ldsm_x4(smem_u32(&qs[r * P + c]), qf[ks]);
      }
    }
    const T* ks_tile = kv + (stage * 2) * kN * P;
    const T* vs_tile = ks_tile + kN * P;
    const bool tail = t < ntail;

    // ---- S = Q K^T (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        const int key = np * 16 + (lane & 7) + ((mat >> 1) << 3);
        const int c = ks * 16 + ((mat & 1) << 3);
        ldsm_x4(smem_u32(&ks_tile[key * P + c]), b);
        mma16816<T>(s[2 * np], qf[ks], b[0], b[1]);
        mma16816<T>(s[2 * np + 1], qf[ks], b[2], b[3]);
      }
    }
    // ---- scale, bias, masks (log2 domain)
    int kstart, klen;
    if (tail) {
      kstart = t * kN;
      klen = min(kN, p.nb - kstart);
    } else {
      const int tt = t - ntail;
      int blk = tt;
      if (p.mode == 1) blk = p.indices[(int64_t(bh) * ((p.tq + kM - 1) / kM) + qblk) * p.nsel + tt];
      else if (p.mode == 2) blk = qblk;
      blk = min(max(blk, 0), (p.tk + kN - 1) / kN - 1);
      kstart = blk * kN;
      klen = min(kN, p.tk - kstart);
    }
    const float LOG2E = 1.4426950408889634f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = n * 8 + cq + (e & 1);
        const int row = warp * 16 + g + ((e >> 1) << 3);
        float val = s[n][e] * p.scale;
        bool masked = col >= klen;
        if (tail) {
          const int j = kstart + col;
          if (!masked) {
            masked = (selw[j >> 5] >> (j & 31)) & 1u;
            const int lj = min(kN, p.tk - j * kN);
            val = val + logf(static_cast<float>(lj));
          }
        } else if (p.causal) {
          masked = masked || (kstart + col > q0 + row);
        }
        float x = masked ? -INFINITY : val;
        if (p.bias != nullptr && !tail && q0 + row < p.tq && col < klen)  // fixed-block mask terms
          x += p.bias[int64_t(bh) * p.bias_bh_stride + int64_t(q0 + row) * kN + col];
        s[n][e] = x * LOG2E;
      }
    }
    // ---- online softmax
    float alpha[2], psum[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(mrow[hr], mx);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      alpha[hr] = exp2f(mrow[hr] - muse);
      mrow[hr] = mnew;
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float p0 = exp2f(s[n][2 * hr] - muse);
        const float p1 = exp2f(s[n][2 * hr + 1] - muse);
        s[n][2 * hr] = p0;
        s[n][2 * hr + 1] = p1;
        sum += p0 + p1;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      psum[hr] = sum;
      lrow[hr] = lrow[hr] * alpha[hr] + sum;
      tmass[hr] = tmass[hr] * alpha[hr] + (tail ? sum : 0.f);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = Cvt<T>::pack2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = Cvt<T>::pack2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = Cvt<T>::pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = Cvt<T>::pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b[4];
        const int key = kk * 16 + (lane & 7) + ((mat & 1) << 3);
        const int c = np * 16 + ((mat >> 1) << 3);
        ldsm_x4_t(smem_u32(&vs_tile[key * P + c]), b);
        mma16816<T>(o[2 * np], a, b[0], b[1]);
        mma16816<T>(o[2 * np + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();
  }

  // ---- first-order correction: O += tail_mass * corr_scale * (Q H)
  if (p.h != nullptr) {
    static_assert(D <= 2 * kN, "H must fit in one K|V stage");
    {
      constexpr int VEC = D / 8;
      const char* hb = static_cast<const char*>(p.h) + int64_t(bh) * D * D * 2;
      for (int idx = threadIdx.x; idx < D * VEC; idx += kThreads) {
        const int r = idx / VEC;
        const int vec = idx - r * VEC;
        cp_async16(smem_u32(&kv[r * P + vec * 8]), hb + (r * D + vec * 8) * 2, 16);
      }
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();
    }
    if (ntiles == 0) {
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        const int r = warp * 16 + (lane & 7) + ((mat & 1) << 3);
        const int c = ks * 16 + ((mat >> 1) << 3);
        ldsm_x4(smem_u32(&qs[r * P + c]), qf[ks]);
      }
    }
    const float w0 = tmass[0] * p.corr_scale;
    const float w1 = tmass[1] * p.corr_scale;
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        uint32_t b[4];
        const int r = ks * 16 + (lane & 7) + ((mat & 1) << 3);
        const int c = np * 16 + ((mat >> 1) << 3);
        ldsm_x4_t(smem_u32(&kv[r * P + c]), b);
        mma16816<T>(c0, qf[ks], b[0], b[1]);
        mma16816<T>(c1, qf[ks], b[2], b[3]);
      }
      o[2 * np][0] += c0[0] * w0;
      o[2 * np][1] += c0[1] * w0;
      o[2 * np][2] += c0[2] * w1;
      o[2 * np][3] += c0[3] * w1;
      o[2 * np + 1][0] += c1[0] * w0;
      o[2 * np + 1][1] += c1[1] * w0;
      o[2 * np + 1][2] += c1[2] * w1;
      o[2 * np + 1][3] += c1[3] * w1;
    }
  }

  // ---- normalise, stage through shared memory, coalesced row stores
  float inv[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr)  // every key masked: NaN, as the reference's softmax gives
    inv[hr] = lrow[hr] > 0.f ? 1.f / lrow[hr] : (p.bias != nullptr ? __int_as_float(0x7fc00000) : 0.f);
  __syncthreads();  // every warp is done reading qs fragments / H
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int col = n * 8 + cq;
    const int r0 = warp * 16 + g;
    *reinterpret_cast<uint32_t*>(&qs[r0 * P + col]) = Cvt<T>::pack2(o[n][0] * inv[0], o[n][1] * inv[0]);
    *reinterpret_cast<uint32_t*>(&qs[(r0 + 8) * P + col]) = Cvt<T>::pack2(o[n][2] * inv[1], o[n][3] * inv[1]);
  }
  if (p.lse != nullptr && (lane & 3) == 0) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = warp * 16 + g + hr * 8;
      if (r < qlen) {
        const float LN2 = 0.6931471805599453f;
        const float muse = mrow[hr] == -INFINITY ? 0.f : mrow[hr];
        p.lse[int64_t(bh) * p.tq + q0 + r] = lrow[hr] > 0.f ? (muse + log2f(lrow[hr])) * LN2 : -INFINITY;
      }
    }
  }
  __syncthreads();
  {
    constexpr int VEC = D / 8;
    for (int idx = threadIdx.x; idx < kM * VEC; idx += kThreads) {
      const int r = idx / VEC;
      const int vec = idx - r * VEC;
      if (r < qlen) {
        *reinterpret_cast<uint4*>(p.o.row(bh, q0 + r) + vec * 16) = *reinterpret_cast<const uint4*>(&qs[r * P + vec * 8]);
      }
    }
  }
}

}  // namespace

cudaError_t launch_attn_mma(const AttnParams& p, int dtype, int batch_heads, cudaStream_t stream) {
  const int D = p.q.dim;
  const size_t smem = size_t(kM + 4 * kN) * (D + 8) * 2;
  dim3 grid((p.tq + kM - 1) / kM, batch_heads);
  cudaError_t err;
#define B2_ATTN_LAUNCH(T, DD)                                                                              \
  do {                                                                                                     \
    auto kern = attn_kernel<T, DD>;                                                                        \
    err = ensure_smem(reinterpret_cast<const void*>(kern), static_cast<int>(smem)); \
    if (err != cudaSuccess) return err;                                                                    \
    kern<<<grid, kThreads, smem, stream>>>(p);                                                             \
  } while (0)
  if (dtype == B2_BF16) {
    if (D == 128) B2_ATTN_LAUNCH(__nv_bfloat16, 128);
    else if (D == 64) B2_ATTN_LAUNCH(__nv_bfloat16, 64);
    else if (D == 32) B2_ATTN_LAUNCH(__nv_bfloat16, 32);
    else return cudaErrorInvalidValue;
  } else {
    if (D == 128) B2_ATTN_LAUNCH(__half, 128);
    else if (D == 64) B2_ATTN_LAUNCH(__half, 64);
    else if (D == 32) B2_ATTN_LAUNCH(__half, 32);
    else return cudaErrorInvalidValue;
  }
#undef B2_ATTN_LAUNCH
  return cudaGetLastError();
}

}  // namespace b2
