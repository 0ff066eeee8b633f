// Shared device helpers for the B200 attention kernels: row addressing of
// b2_view tensors, BF16/FP16 conversions, and thin PTX wrappers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200attn.h"

namespace b2 {

constexpr int kBlock = 64;  // PISA / fixed-block token block
constexpr int kTileDim = 128;  // head-dim width of the tcgen05 tiles and the PISA workspace rows

// Device-side copy of a b2_view (pointer + strides + token order).
struct Rows {
  char* base;
  int64_t sb, sh, st;  // strides in elements
  int heads, tokens, dim, order, gh, gw, esize;

  // token index in storage order for logical (ordered) row t
  __device__ __forceinline__ int map(int t) const {
    if (order == B2_ORDER_LINEAR) return t;
    const int frame_tokens = gh * gw;
    const int f = t / frame_tokens;
    const int o = t - f * frame_tokens;
    const int tile = o >> 6;
    const int intra = o & 63;
    const int tiles_per_row = gw >> 3;
    const int tr = tile / tiles_per_row;
    const int tc = tile - tr * tiles_per_row;
    return f * frame_tokens + (tr * 8 + (intra >> 3)) * gw + tc * 8 + (intra & 7);
  }
  __device__ __forceinline__ char* row(int bh, int t) const {
    const int b = bh / heads;
    const int h = bh - b * heads;
    return base + (int64_t(b) * sb + int64_t(h) * sh + int64_t(map(t)) * st) * esize;
  }
};

inline Rows make_rows(const b2_view& v) {
  Rows r;
  r.base = static_cast<char*>(v.base);
  r.sb = v.stride_b;
  r.sh = v.stride_h;
  r.st = v.stride_t;
  r.heads = v.heads;
  r.tokens = v.tokens;
  r.dim = v.head_dim;
  r.order = v.order;
  r.gh = v.grid_h;
  r.gw = v.grid_w;
  r.esize = v.dtype == B2_F32 ? 4 : 2;
  return r;
}

template <typename T> struct Cvt;
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  // widen a packed pair with integer ops (bf16 is the top half of an f32),
  // keeping the conversion pipe free
  static __device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xFFFF0000u);
  }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    lo = f.x;
    hi = f.y;
  }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device)
// and size: later launches skip the driver call.
cudaError_t ensure_smem(const void* kernel, int bytes);

// ---- Programmatic dependent launch.  Kernels after the first one of a PISA
// call are launched with programmatic stream serialization: their blocks may
// start (barrier set-up, TMEM allocation) while the previous kernel in the
// stream drains, and each calls grid_dep_wait() before it reads or writes any
// global memory that earlier stream work produces or consumes.  For an
// ordinary launch grid_dep_wait() returns at once.  B200ATTN_PDL=0 turns the
// attribute off.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async global->shared copy; src_bytes==0 zero-fills the slot.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

}  // namespace b2
