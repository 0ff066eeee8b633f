// PISA per-block statistics: q/k/v centroids, per-block first-order K-V
// covariance H_blk = sum_r (k_r - kbar)^T v_r, its Frobenius norm, and the
// per-(batch*head) sum of H_blk.
//
// Semantics follow native/rdna35_pisa_ck/csrc/pisa_kernels.cu:167-244 (HYD:
// sequential FP32 column sums times 1/len, BF16 q/v centroids, FP32 K
// centring) and rdna35_block_attention/pisa_kernel.py:49-84 (GENERIC: sums
// divided by len, FP32 centroids, centred K rounded to the input type).
//
// Design: one CTA owns G consecutive 64-token blocks of one (batch, head).
// Tiles are staged with 16-byte cp.async into padded shared memory (double
// buffered).  H_blk is a 128x128x64 contraction done on tensor cores with the
// FP32-centred K split into hi+lo 16-bit halves (two MMAs), so products keep
// ~16 mantissa bits; the reference's float atomicAdd into h_sum is replaced
// by per-CTA partial sums reduced in a fixed order by stats_reduce_kernel.
#include <cstdio>
#include <mutex>

#include "kernels.h"

namespace b2 {
namespace {

constexpr int kD = 128;
constexpr int kPad = kD + 8;            // 272-byte rows: conflict-free ldmatrix
constexpr int kTileElems = kBlock * kPad;
constexpr int kStatsThreads = 256;

template <typename T>
struct StatsSmem {
  T tiles[2][3][kTileElems];  // [stage][q,k,v]
  T kc_hi[kTileElems];
  T kc_lo[kTileElems];
  float kmean[kD];
  float norm_part[8];
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

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

template <typename T>
__device__ __forceinline__ void issue_block_load(StatsSmem<T>& s, int stage, const Rows& q, const Rows& k,
                                                 const Rows& v, int bh, int start, int len) {
  // 3 tensors x 64 rows x 16 vectors of 16 bytes = 3072 copies / 256 threads
  for (int idx = threadIdx.x; idx < 3 * kBlock * 16; idx += kStatsThreads) {
    const int tensor = idx / (kBlock * 16);
    const int rem = idx - tensor * kBlock * 16;
    const int r = rem >> 4;
    const int vec = rem & 15;
    const Rows& src = tensor == 0 ? q : (tensor == 1 ? k : v);
    const bool valid = r < len;
    const char* g = valid ? src.row(bh, start + r) + vec * 16 : src.base;
    cp_async16(smem_u32(&s.tiles[stage][tensor][r * kPad + vec * 8]), g, valid ? 16 : 0);
  }
  cp_async_commit();
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kStatsThreads, 1)
stats_kernel(Rows q, Rows k, Rows v, int blocks, int group, void* q_centroids, float* k_centroids,
             void* v_stats, float* h_norm, float* h_partial) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  StatsSmem<T>& s = *reinterpret_cast<StatsSmem<T>*>(smem_raw);
  const int g = blockIdx.x;
  const int bh = blockIdx.y;
  const int groups = gridDim.x;
  const int first = g * group;
  const int last = min(blocks, first + group);
  const int tokens = q.tokens;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  float hsum[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) hsum[n][e] = 0.f;

  if (first < last) {
    issue_block_load(s, 0, q, k, v, bh, first * kBlock, min(kBlock, tokens - first * kBlock));
  }
  for (int blk = first; blk < last; ++blk) {
    const int stage = (blk - first) & 1;
    const int start = blk * kBlock;
    const int len = min(kBlock, tokens - start);
    cp_async_wait<0>();
    __syncthreads();
    if (blk + 1 < last) {
      const int ns = (blk + 1) * kBlock;
      issue_block_load(s, stage ^ 1, q, k, v, bh, ns, min(kBlock, tokens - ns));
    }
    // ---- column sums (sequential over rows, as pisa_kernels.cu:191-200)
    const int64_t out_base = (int64_t(bh) * blocks + blk) * kD;
    for (int task = threadIdx.x; task < 3 * kD; task += kStatsThreads) {
      const int tensor = task / kD;
      const int col = task - tensor * kD;
      const T* tile = s.tiles[stage][tensor];
      float acc = 0.f;
      if (MODE == B2_STATS_SCALED) {
        // each element times 1/len before the sum (pisa_kernels.cu:149-156)
        const float inv = 1.0f / static_cast<float>(len);
        for (int r = 0; r < len; ++r) acc += Cvt<T>::to_f(tile[r * kPad + col]) * inv;
      } else {
        for (int r = 0; r < len; ++r) acc += Cvt<T>::to_f(tile[r * kPad + col]);
      }
      if (MODE != B2_STATS_GENERIC) {
        const float inv = 1.0f / static_cast<float>(len);
        const float mean = MODE == B2_STATS_SCALED ? acc : acc * inv;
        (void)inv;
        if (tensor == 0) {
          static_cast<T*>(q_centroids)[out_base + col] = Cvt<T>::from_f(mean);
        } else if (tensor == 1) {
          k_centroids[out_base + col] = mean;
          s.kmean[col] = mean;
        } else {
          static_cast<T*>(v_stats)[out_base + col] = Cvt<T>::from_f(mean);
        }
      } else {
        const float flen = static_cast<float>(len);
        if (tensor == 0) {
          static_cast<float*>(q_centroids)[out_base + col] = acc / flen;
        } else if (tensor == 1) {
          const float mean = acc / flen;
          k_centroids[out_base + col] = mean;
          s.kmean[col] = mean;
        } else {
          static_cast<float*>(v_stats)[out_base + col] = acc;
        }
      }
    }
    __syncthreads();
    // ---- centre K: FP32 difference split into hi + lo halves
    {
      const T* kt = s.tiles[stage][1];
      for (int idx = threadIdx.x; idx < kBlock * kD; idx += kStatsThreads) {
        const int r = idx >> 7;
        const int c = idx & (kD - 1);
        float centred = 0.f;
        if (r < len) centred = Cvt<T>::to_f(kt[r * kPad + c]) - s.kmean[c];
        const T hi = Cvt<T>::from_f(centred);
        s.kc_hi[r * kPad + c] = hi;
        s.kc_lo[r * kPad + c] = Cvt<T>::from_f(MODE != B2_STATS_GENERIC ? centred - Cvt<T>::to_f(hi) : 0.f);
      }
    }
    __syncthreads();
    // ---- H_blk[i][j] = sum_r Kc[r][i] * V[r][j]; warp owns rows i in [16w,16w+16)
    float acc[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    const T* vt = s.tiles[stage][2];
    const int mat = lane >> 3;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t ahi[4], alo[4];
      {
        const int r = ks * 16 + (lane & 7) + ((mat >> 1) << 3);
        const int i = warp * 16 + ((mat & 1) << 3);
        ldsm_x4_trans(smem_u32(&s.kc_hi[r * kPad + i]), ahi[0], ahi[1], ahi[2], ahi[3]);
        if (MODE != B2_STATS_GENERIC) ldsm_x4_trans(smem_u32(&s.kc_lo[r * kPad + i]), alo[0], alo[1], alo[2], alo[3]);
      }
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b[4];
        const int r = ks * 16 + (lane & 7) + ((mat & 1) << 3);
        const int j = 8 * (2 * np + (mat >> 1));
        ldsm_x4_trans(smem_u32(&vt[r * kPad + j]), b[0], b[1], b[2], b[3]);
        mma16816<T>(acc[2 * np], ahi, b[0], b[1]);
        mma16816<T>(acc[2 * np + 1], ahi, b[2], b[3]);
        if (MODE != B2_STATS_GENERIC) {
          mma16816<T>(acc[2 * np], alo, b[0], b[1]);
          mma16816<T>(acc[2 * np + 1], alo, b[2], b[3]);
        }
      }
    }
    // ---- Frobenius norm of H_blk and running sum
    float sq = 0.f;
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sq += acc[n][e] * acc[n][e];
        hsum[n][e] += acc[n][e];
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if (lane == 0) s.norm_part[warp] = sq;
    __syncthreads();
    if (threadIdx.x == 0 && h_norm != nullptr) {
      float total = 0.f;
      for (int w = 0; w < kStatsThreads / 32; ++w) total += s.norm_part[w];
      h_norm[int64_t(bh) * blocks + blk] = sqrtf(total);
    }
  }
  // ---- partial H of this CTA: [bh][g][i][j]
  float* dst = h_partial + (int64_t(bh) * groups + g) * kD * kD;
  const int row0 = warp * 16 + (lane >> 2);
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * (lane & 3);
    *reinterpret_cast<float2*>(&dst[row0 * kD + col]) = make_float2(hsum[n][0], hsum[n][1]);
    *reinterpret_cast<float2*>(&dst[(row0 + 8) * kD + col]) = make_float2(hsum[n][2], hsum[n][3]);
  }
}

// h_sum[bh] = sum over groups in ascending order (deterministic), plus an
// optional 16-bit copy used as the correction GEMM operand.
template <typename T>
__global__ void stats_reduce_kernel(const float* __restrict__ partial, int groups, float* __restrict__ h_sum,
                                    T* __restrict__ h_half) {
  grid_dep_wait();
  const int bh = blockIdx.y;
  const int idx4 = blockIdx.x * blockDim.x + threadIdx.x;  // float4 index within D*D
  if (idx4 >= kD * kD / 4) return;
  const float4* src = reinterpret_cast<const float4*>(partial + int64_t(bh) * groups * kD * kD) + idx4;
  float4 acc = src[0];
  for (int gi = 1; gi < groups; ++gi) {
    const float4 p = src[int64_t(gi) * (kD * kD / 4)];
    acc.x += p.x;
    acc.y += p.y;
    acc.z += p.z;
    acc.w += p.w;
  }
  reinterpret_cast<float4*>(h_sum + int64_t(bh) * kD * kD)[idx4] = acc;
  if (h_half != nullptr) {
    uint2 packed;
    packed.x = Cvt<T>::pack2(acc.x, acc.y);
    packed.y = Cvt<T>::pack2(acc.z, acc.w);
    reinterpret_cast<uint2*>(h_half + int64_t(bh) * kD * kD)[idx4] = packed;
  }
}

}  // namespace

int stats_group_size(int batch_heads, int blocks) {
  // aim at ~2 work items per SM across 148 SMs, 1..16 blocks per item
  const long total = static_cast<long>(batch_heads) * blocks;
  long g = (total + 148 * 2 - 1) / (148 * 2);
  if (g < 1) g = 1;
  if (g > 16) g = 16;
  return static_cast<int>(g);
}

// Blocks per work item on the workspace paths: a function of the block count
// only, so each head's H, reduced over fixed groups in a fixed order, has the
// same bits however many heads share the call (head-sharded or staged calls
// reproduce the single-call output).
int stats_group_for_blocks(int blocks) { return blocks < 16 ? (blocks < 1 ? 1 : blocks) : 16; }

cudaError_t launch_stats(const Rows& q, const Rows& k, const Rows& v, int dtype, int mode, int batch_heads,
                         int blocks, void* q_centroids, float* k_centroids, void* v_stats, float* h_sum,
                         float* h_norm, void* h_half, float* partial, cudaStream_t stream) {
  const int group = stats_group_for_blocks(blocks);
  const int groups = (blocks + group - 1) / group;
  dim3 grid(groups, batch_heads);
  const size_t smem = dtype == B2_BF16 ? sizeof(StatsSmem<__nv_bfloat16>) : sizeof(StatsSmem<__half>);
  cudaError_t err;
#define B2_STATS_LAUNCH(T, M)                                                                              \
  do {                                                                                                     \
    auto kern = stats_kernel<T, M>;                                                                        \
    err = ensure_smem(reinterpret_cast<const void*>(kern), static_cast<int>(smem)); \
    if (err != cudaSuccess) return err;                                                                    \
    kern<<<grid, kStatsThreads, smem, stream>>>(q, k, v, blocks, group, q_centroids, k_centroids, v_stats, \
                                                h_norm, partial);                                          \
  } while (0)
  if (dtype == B2_BF16) {
    if (mode == B2_STATS_HYD) B2_STATS_LAUNCH(__nv_bfloat16, B2_STATS_HYD);
    else if (mode == B2_STATS_SCALED) B2_STATS_LAUNCH(__nv_bfloat16, B2_STATS_SCALED);
    else B2_STATS_LAUNCH(__nv_bfloat16, B2_STATS_GENERIC);
  } else {
    if (mode == B2_STATS_HYD) B2_STATS_LAUNCH(__half, B2_STATS_HYD);
    else if (mode == B2_STATS_SCALED) B2_STATS_LAUNCH(__half, B2_STATS_SCALED);
    else B2_STATS_LAUNCH(__half, B2_STATS_GENERIC);
  }
#undef B2_STATS_LAUNCH
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  dim3 rgrid((kD * kD / 4 + 255) / 256, batch_heads);
  if (dtype == B2_BF16)
    stats_reduce_kernel<__nv_bfloat16><<<rgrid, 256, 0, stream>>>(partial, groups, h_sum,
                                                                  static_cast<__nv_bfloat16*>(h_half));
  else
    stats_reduce_kernel<__half><<<rgrid, 256, 0, stream>>>(partial, groups, h_sum, static_cast<__half*>(h_half));
  return cudaGetLastError();
}

cudaError_t launch_stats_reduce(const float* partial, int groups, int batch_heads, float* h_sum, void* h_half,
                                int dtype, cudaStream_t stream) {
  dim3 rgrid((kD * kD / 4 + 255) / 256, batch_heads);
  if (dtype == B2_BF16)
    return launch_pdl(stats_reduce_kernel<__nv_bfloat16>, rgrid, dim3(256), 0, stream, partial, groups, h_sum,
                      static_cast<__nv_bfloat16*>(h_half));
  return launch_pdl(stats_reduce_kernel<__half>, rgrid, dim3(256), 0, stream, partial, groups, h_sum,
                    static_cast<__half*>(h_half));
}

int64_t stats_partial_bytes(int batch_heads, int blocks) {
  const int group = stats_group_for_blocks(blocks);
  const int groups = (blocks + group - 1) / group;
  return int64_t(batch_heads) * groups * kD * kD * 4;
}

}  // namespace b2

// ---------------------------------------------------------------------------
// Allocation-free variant of the block-statistics entry point.
//
// Some callers cannot allocate device memory at the moment they need the
// statistics: code running inside a custom allocator's own callbacks, hosts
// whose memory pool is fixed at start-up (embedded engines, plugin sandboxes
// that only hand out input/output buffers), or paths that must not add
// allocations while the framework's caching allocator is being reset.  For
// them the per-CTA partial H sums live in a fixed file-scope device array
// instead of a caller-provided workspace.  The array holds kNoAllocScratchBytes
// (8 MiB) on every GPU that loads the library, until the process exits.
namespace b2 {
namespace {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;
static __device__ __align__(256) unsigned char g_stats_scratch[kNoAllocScratchBytes];

// Device address of g_stats_scratch in the current device's context.  It is
// looked up on every call: the host-side symbol is only a stand-in and must
// never reach a kernel, and an address cached across a cudaDeviceReset would
// point into a context that no longer exists.
cudaError_t scratch_address(void** out) {
  void* ptr = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&ptr, g_stats_scratch);
  if (err != cudaSuccess) return err;
  *out = ptr;
  return cudaSuccess;
}

}  // namespace
}  // namespace b2

extern "C" const char* b2_noalloc_last_error(void) { return b2_last_error(); }

extern "C" int b2_pisa_block_stats_noalloc(const b2_view* q, const b2_view* k, const b2_view* v, int32_t mode,
                                           void* q_centroids, float* k_centroids, void* v_stats, float* h_sum,
                                           float* h_norm, void* h_bf16, void* stream) {
  using namespace b2;
  // same argument checks as b2_pisa_block_stats (order, grid, alignment ...)
  int rc = check_stats_call(q, k, v, mode, q_centroids, k_centroids, v_stats, h_sum);
  if (rc) return rc;
  const int bh = q->batch * q->heads;
  const int blocks = (q->tokens + kBlock - 1) / kBlock;
  // The workspace entry's grouping (by block count alone), grown only as far
  // as the fixed array requires; a grown group sums H in another order.
  const int64_t per_group = int64_t(kD) * kD * 4;
  int group = stats_group_for_blocks(blocks);
  while (group < blocks && int64_t(bh) * ((blocks + group - 1) / group) * per_group > kNoAllocScratchBytes) ++group;
  const int groups = (blocks + group - 1) / group;
  if (int64_t(bh) * groups * per_group > kNoAllocScratchBytes)
    return report_error(B2_ERR_UNSUPPORTED,
                        "b2_pisa_block_stats_noalloc: batch*heads exceeds 128, the 8 MiB scratch limit "
                        "(use b2_pisa_block_stats with a caller workspace)");
  void* scratch = nullptr;
  cudaError_t err = scratch_address(&scratch);
  if (err != cudaSuccess) return report_cuda_error(err, "scratch address lookup");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(scratch);
  bool launched = false;
  if (tcgen05_kernels_enabled()) {
    int* status = device_status_ptr();
    if (status != nullptr) {
      err = launch_stats_umma(*q, *k, *v, mode, group, q_centroids, k_centroids, v_stats, h_norm, partial, status,
                              st, &launched);
      if (err != cudaSuccess) return report_cuda_error(err, "PISA statistics launch");
    }
  }
  if (!launched) {
    const Rows qr = make_rows(*q), kr = make_rows(*k), vr = make_rows(*v);
    dim3 grid(groups, bh);
    const size_t smem = q->dtype == B2_BF16 ? sizeof(StatsSmem<__nv_bfloat16>) : sizeof(StatsSmem<__half>);
#define B2_NOALLOC_LAUNCH(T, M)                                                                              \
  do {                                                                                                       \
    auto kern = stats_kernel<T, M>;                                                                          \
    err = ensure_smem(reinterpret_cast<const void*>(kern), static_cast<int>(smem));                          \
    if (err == cudaSuccess)                                                                                  \
      kern<<<grid, kStatsThreads, smem, st>>>(qr, kr, vr, blocks, group, q_centroids, k_centroids, v_stats,  \
                                              h_norm, partial);                                              \
  } while (0)
    if (q->dtype == B2_BF16) {
      if (mode == B2_STATS_HYD) B2_NOALLOC_LAUNCH(__nv_bfloat16, B2_STATS_HYD);
      else if (mode == B2_STATS_SCALED) B2_NOALLOC_LAUNCH(__nv_bfloat16, B2_STATS_SCALED);
      else B2_NOALLOC_LAUNCH(__nv_bfloat16, B2_STATS_GENERIC);
    } else {
      if (mode == B2_STATS_HYD) B2_NOALLOC_LAUNCH(__half, B2_STATS_HYD);
      else if (mode == B2_STATS_SCALED) B2_NOALLOC_LAUNCH(__half, B2_STATS_SCALED);
      else B2_NOALLOC_LAUNCH(__half, B2_STATS_GENERIC);
    }
#undef B2_NOALLOC_LAUNCH
    if (err == cudaSuccess) err = cudaGetLastError();
    if (err != cudaSuccess) return report_cuda_error(err, "PISA statistics launch");
  }
  dim3 rgrid((kD * kD / 4 + 255) / 256, bh);
  if (q->dtype == B2_BF16)
    stats_reduce_kernel<__nv_bfloat16><<<rgrid, 256, 0, st>>>(partial, groups, h_sum,
                                                              static_cast<__nv_bfloat16*>(h_bf16));
  else
    stats_reduce_kernel<__half><<<rgrid, 256, 0, st>>>(partial, groups, h_sum, static_cast<__half*>(h_bf16));
  err = cudaGetLastError();
  if (err != cudaSuccess) return report_cuda_error(err, "PISA statistics reduction launch");
  return report_ok();
}
