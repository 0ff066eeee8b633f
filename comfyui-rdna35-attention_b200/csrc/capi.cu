// C ABI entry points: argument validation (the TORCH_CHECK ladders of
// native/rdna35_pisa_ck/csrc/pisa_kernels.cu:563-773 restated as status
// codes), workspace carving and launch orchestration.  No entry point
// allocates device memory or synchronises the stream.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>
#include <vector>
#include <cstring>

#include "kernels.h"


namespace b2 {
bool pdl_enabled() {
  static const bool enabled = [] {
    const char* env = getenv("B200ATTN_PDL");
    return env == nullptr || strcmp(env, "0") != 0;
  }();
  return enabled;
}

cudaError_t ensure_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kernel, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) done[key] = bytes;
  return err;
}
}  // namespace b2

using namespace b2;

namespace {

thread_local char g_error[512] = "";
thread_local const char* g_last_kernel = "none";
long long* g_trace = nullptr;  // diagnostics timeline buffer (b2_set_trace)
int g_withhold_q = 0;           // diagnostics: b2_debug_withhold_q

// B200ATTN_KERNEL=mma forces the warp-level mma.sync attention kernel
// (kept for layouts the TMA maps cannot express); default: tcgen05 kernel.
bool umma_enabled() {
  static const bool enabled = [] {
    const char* env = getenv("B200ATTN_KERNEL");
    return env == nullptr || strcmp(env, "mma") != 0;
  }();
  return enabled;
}

// Block statistics: the TMA/tcgen05 kernel when the views allow it, else the
// warp-MMA kernel; both followed by the fixed-order reduction of partial H.
cudaError_t run_stats(const b2_view* q, const b2_view* k, const b2_view* v, int mode, void* qc, float* kc, void* vs,
                      float* h_sum, float* h_norm, void* h_half, float* partial, cudaStream_t st) {
  const int bh = q->batch * q->heads;
  const int nb = (q->tokens + kBlock - 1) / kBlock;
  if (umma_enabled()) {
    const int group = stats_group_for_blocks(nb);
    int* status = device_status_ptr();
    bool launched = false;
    if (status != nullptr) {
      cudaError_t err = launch_stats_umma(*q, *k, *v, mode, group, qc, kc, vs, h_norm, partial, status, st, &launched);
      if (err != cudaSuccess) return err;
      if (launched) return launch_stats_reduce(partial, (nb + group - 1) / group, bh, h_sum, h_half, q->dtype, st);
    }
  }
  // the warp-MMA statistics kernel reads 128 columns: D < 128 needs the TMA path
  if (q->head_dim != 128) return cudaErrorNotSupported;
  return launch_stats(make_rows(*q), make_rows(*k), make_rows(*v), q->dtype, mode, bh, nb, qc, kc, vs, h_sum, h_norm,
                      h_half, partial, st);
}

void set_mirrors(AttnParams& p, char* const* mirrors, int n, int multicast) {
  p.n_mirror = n;
  p.mirror_multicast = multicast;
  for (int i = 0; i < kMaxMirrors; ++i) p.mirror[i] = i < n ? mirrors[i] : nullptr;
}

cudaError_t run_attention(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* o, const AttnParams& p,
                          cudaStream_t st) {
  // D = 32 / 64 full and fixed-block attention keep the warp-MMA kernel,
  // which computes at D; other D < 128 run zero-filled on the tcgen05 kernel
  const bool mma_native = q->head_dim == 32 || q->head_dim == 64 || q->head_dim == 128;
  const bool prefer_umma = q->head_dim == 128 || p.mode == 1 || !mma_native;
  if (umma_enabled() && prefer_umma && umma_supported(*q, *k, *v, *o)) {
    AttnParams pt = p;
    pt.trace = g_trace;
    pt.debug_withhold_q = g_withhold_q;
    bool launched = false;
    int* status = device_status_ptr();
    if (status != nullptr) {
      const cudaError_t err = launch_attn_umma(*q, *k, *v, *o, pt, status, st, &launched);
      if (err != cudaSuccess || launched) {
        g_last_kernel = "tcgen05";
        return err;
      }
    }
  }
  // only the tcgen05 kernel writes peer copies of the output
  if (!mma_native || (p.mode == 1 && q->head_dim != 128) || p.n_mirror > 0) return cudaErrorNotSupported;
  g_last_kernel = "mma_sync";
  return launch_attn_mma(p, q->dtype, q->batch * q->heads, st);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(B2_ERR_CUDA, "%s failed: %s", what, cudaGetErrorString(err));
}

int ok() {
  g_error[0] = '\0';
  return B2_OK;
}

int esize_of(int dtype) { return dtype == B2_F32 ? 4 : 2; }

// A view is usable by the 16-byte row kernels when every row start is
// 16-byte aligned and the head dimension spans whole 16-byte vectors.
int check_view(const b2_view* v, const char* name) {
  if (v == nullptr) return fail(B2_ERR_INVALID, "%s view is NULL", name);
  if (v->base == nullptr) return fail(B2_ERR_INVALID, "%s has a NULL base pointer", name);
  if (v->batch <= 0 || v->heads <= 0 || v->tokens <= 0 || v->head_dim <= 0)
    return fail(B2_ERR_INVALID, "%s requires positive B, H, T and D", name);
  if (v->dtype != B2_BF16 && v->dtype != B2_F16 && v->dtype != B2_F32)
    return fail(B2_ERR_INVALID, "%s has an unknown dtype %d", name, v->dtype);
  const int es = esize_of(v->dtype);
  if ((int64_t(v->head_dim) * es) % 16 != 0)
    return fail(B2_ERR_INVALID, "%s head_dim*element size must be a multiple of 16 bytes", name);
  if (reinterpret_cast<uintptr_t>(v->base) % 16 != 0) return fail(B2_ERR_INVALID, "%s must be 16-byte aligned", name);
  if ((v->stride_b * es) % 16 || (v->stride_h * es) % 16 || (v->stride_t * es) % 16)
    return fail(B2_ERR_INVALID, "%s strides must be multiples of 16 bytes", name);
  if (v->order == B2_ORDER_TILED8) {
    if (v->grid_h <= 0 || v->grid_w <= 0 || v->grid_h % 8 || v->grid_w % 8)
      return fail(B2_ERR_INVALID, "%s tiled order requires grid sides divisible by 8", name);
    const int64_t frame = int64_t(v->grid_h) * v->grid_w;
    if (v->tokens % frame) return fail(B2_ERR_INVALID, "%s tokens must be a multiple of grid_h*grid_w", name);
  } else if (v->order != B2_ORDER_LINEAR) {
    return fail(B2_ERR_INVALID, "%s has an unknown token order %d", name, v->order);
  }
  return B2_OK;
}

bool same_bht(const b2_view* a, const b2_view* b) {
  return a->batch == b->batch && a->heads == b->heads && a->tokens == b->tokens && a->head_dim == b->head_dim;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct PisaWorkspace {
  void* qc;
  float* kc;
  void* vstat;
  float* hsum;
  void* h16;
  float* hnorm;
  void* kc16;
  void* vc16;
  int32_t* indices;
  uint32_t* sel;
  int32_t* pairs;
  float* partial;
  size_t total;
  size_t offset[B2_WS_FIELDS];  // byte offset of each buffer, in B2_WS_* order
};

PisaWorkspace carve(char* base, int bh, int tokens, int dim, int k) {
  const int nb = (tokens + kBlock - 1) / kBlock;
  const int words = (nb + 31) / 32;
  PisaWorkspace w{};
  size_t off = 0;
  int field = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    w.offset[field++] = off;
    off += align256(bytes);
    return p;
  };
  const size_t cent = size_t(bh) * nb * dim;
  w.qc = take(cent * 4);
  w.kc = reinterpret_cast<float*>(take(cent * 4));
  w.vstat = take(cent * 4);
  w.hsum = reinterpret_cast<float*>(take(size_t(bh) * dim * dim * 4));
  w.h16 = take(size_t(bh) * dim * dim * 2);
  w.hnorm = reinterpret_cast<float*>(take(size_t(bh) * nb * 4));
  w.kc16 = take(cent * 2);
  w.vc16 = take(cent * 2);
  w.indices = reinterpret_cast<int32_t*>(take(size_t(bh) * nb * (k > 0 ? k : 1) * 4));
  w.sel = reinterpret_cast<uint32_t*>(take(size_t(bh) * nb * words * 4));
  w.pairs = reinterpret_cast<int32_t*>(take(size_t(bh) * ((nb + 1) / 2) * 2 * 4));
  w.partial = reinterpret_cast<float*>(take(static_cast<size_t>(stats_partial_bytes(bh, nb))));
  w.total = off;
  return w;
}

AttnParams base_params(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* o, float scale) {
  AttnParams p{};
  p.q = make_rows(*q);
  p.k = make_rows(*k);
  p.v = make_rows(*v);
  p.o = make_rows(*o);
  p.tq = q->tokens;
  p.tk = k->tokens;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  return p;
}

int check_qkv_o(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* o, bool same_tokens) {
  int rc;
  if ((rc = check_view(q, "q")) || (rc = check_view(k, "k")) || (rc = check_view(v, "v")) ||
      (rc = check_view(o, "out")))
    return rc;
  if (!same_bht(k, v)) return fail(B2_ERR_INVALID, "k and v must have matching [B,H,T,D]");
  if (q->batch != k->batch || q->heads != k->heads || q->head_dim != k->head_dim)
    return fail(B2_ERR_INVALID, "q and k must share B, H and D");
  if (same_tokens && q->tokens != k->tokens) return fail(B2_ERR_INVALID, "self-attention requires Tq == Tk");
  if (!same_bht(q, o)) return fail(B2_ERR_INVALID, "out must have q's [B,H,T,D]");
  if (q->dtype != k->dtype || q->dtype != v->dtype || q->dtype != o->dtype)
    return fail(B2_ERR_INVALID, "q, k, v and out must share one dtype");
  return B2_OK;
}

// Copy streams and per-stage events of the pipelined host-memory forward, one
// set per device, created on first use and kept for the process lifetime.
struct HostPipe {
  cudaStream_t h2d = nullptr;
  cudaStream_t d2h = nullptr;
  std::vector<cudaEvent_t> ev;  // [3 * stages]: inputs in, output ready, output out
  cudaEvent_t start = nullptr;
  std::mutex enqueue;  // one call's records and waits are enqueued at a time
};

// The current device's pipe, its streams created on first use.
cudaError_t host_pipe(HostPipe** out) {
  static std::mutex mu;
  static std::map<int, HostPipe> pipes;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(mu);
  HostPipe& p = pipes[dev];
  if (p.h2d == nullptr) {
    if ((err = cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking)) != cudaSuccess) return err;
    if ((err = cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking)) != cudaSuccess) return err;
    if ((err = cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming)) != cudaSuccess) return err;
  }
  *out = &p;
  return cudaSuccess;
}

// At least 3 * stages events; the caller holds pipe.enqueue.
cudaError_t host_pipe_events(HostPipe& p, int stages) {
  while (static_cast<int>(p.ev.size()) < 3 * stages) {
    cudaEvent_t e;
    const cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (err != cudaSuccess) return err;
    p.ev.push_back(e);
  }
  return cudaSuccess;
}

bool is_pinned_host(const void* ptr) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeHost;
}

}  // namespace

namespace b2 {
// Argument checks shared by both block-statistics entry points (the
// workspace one and the allocation-free one): view shape, order, grid,
// alignment, dtype, head dim, mode and output pointers.
int check_stats_call(const b2_view* q, const b2_view* k, const b2_view* v, int mode, const void* q_centroids,
                     const float* k_centroids, const void* v_stats, const float* h_sum) {
  int rc;
  if ((rc = check_view(q, "q")) || (rc = check_view(k, "k")) || (rc = check_view(v, "v"))) return rc;
  if (!same_bht(q, k) || !same_bht(q, v)) return fail(B2_ERR_INVALID, "PISA statistics expect matching q/k/v");
  if (q->dtype != k->dtype || q->dtype != v->dtype) return fail(B2_ERR_INVALID, "q, k and v must share one dtype");
  if (q->dtype == B2_F32) return fail(B2_ERR_UNSUPPORTED, "PISA statistics support bfloat16 and float16");
  if (q->head_dim != 128) return fail(B2_ERR_UNSUPPORTED, "PISA statistics require D=128");
  if (mode != B2_STATS_HYD && mode != B2_STATS_GENERIC && mode != B2_STATS_SCALED)
    return fail(B2_ERR_INVALID, "unknown statistics mode");
  if (!q_centroids || !k_centroids || !v_stats || !h_sum)
    return fail(B2_ERR_INVALID, "PISA statistics outputs and workspace must be non-NULL");
  return B2_OK;
}
int report_error(int code, const char* msg) { return fail(code, "%s", msg); }
int report_cuda_error(cudaError_t err, const char* what) { return cuda_fail(err, what); }
int report_ok() { return ok(); }
bool tcgen05_kernels_enabled() { return umma_enabled(); }
}  // namespace b2

extern "C" {

const char* b2_last_error(void) { return g_error; }

const char* b2_last_kernel(void) { return g_last_kernel; }

int b2_set_trace(long long* device_buffer) {
  g_trace = device_buffer;
  return ok();
}

int b2_debug_withhold_q(int32_t enable) {
  g_withhold_q = enable ? 1 : 0;
  return ok();
}

int b2_read_status(int32_t* status) {
  if (status == nullptr) return fail(B2_ERR_INVALID, "status pointer is NULL");
  int* dev = device_status_ptr();
  if (dev == nullptr) return fail(B2_ERR_CUDA, "device status word unavailable");
  int value = 0;
  cudaError_t err = cudaMemcpy(&value, dev, sizeof(int), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return cuda_fail(err, "status read");
  const int zero = 0;
  err = cudaMemcpy(dev, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (err != cudaSuccess) return cuda_fail(err, "status reset");
  *status = value;
  return ok();
}

int b2_api_version(void) { return B200ATTN_API_VERSION; }

int b2_build_info(char* buffer, int64_t capacity) {
  if (buffer == nullptr || capacity <= 0) return fail(B2_ERR_INVALID, "build_info buffer is empty");
  snprintf(buffer, static_cast<size_t>(capacity),
           "api=%d;architecture=sm_100a;cuda_build_version=%d;implementation=b200_pisa_fused;block_size=64;"
           "head_dim=128;max_blocks=1024",
           B200ATTN_API_VERSION, CUDART_VERSION);
  return ok();
}

int b2_check_device(int device_index) {
  cudaDeviceProp prop;
  const cudaError_t err = cudaGetDeviceProperties(&prop, device_index);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDeviceProperties");
  if (prop.major != 10) return fail(B2_ERR_DEVICE, "sm_100 (B200) is required, device %d is sm_%d%d", device_index,
                                    prop.major, prop.minor);
  return ok();
}

int64_t b2_stats_workspace_bytes(int32_t batch_heads, int32_t tokens, int32_t head_dim) {
  if (batch_heads <= 0 || tokens <= 0 || head_dim != 128) return -1;
  return stats_partial_bytes(batch_heads, (tokens + kBlock - 1) / kBlock);
}

int b2_pisa_block_stats(const b2_view* q, const b2_view* k, const b2_view* v, int32_t mode, void* q_centroids,
                        float* k_centroids, void* v_stats, float* h_sum, float* h_norm, void* h_bf16,
                        void* workspace, void* stream) {
  int rc = check_stats_call(q, k, v, mode, q_centroids, k_centroids, v_stats, h_sum);
  if (rc) return rc;
  if (!workspace) return fail(B2_ERR_INVALID, "PISA statistics outputs and workspace must be non-NULL");
  const cudaError_t err = run_stats(q, k, v, mode, q_centroids, k_centroids, v_stats, h_sum, h_norm, h_bf16,
                                    static_cast<float*>(workspace), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "PISA block statistics launch");
  return ok();
}

int b2_pisa_route(const void* qc, int32_t qc_dtype, const float* kc, int32_t kc_round, const float* h_norm,
                  int32_t batch_heads, int32_t blocks, int32_t head_dim, int32_t exact_blocks, float scale,
                  int32_t sink_block, int32_t* indices, uint32_t* sel_bits, void* stream) {
  if (!qc || !kc || !indices || !sel_bits) return fail(B2_ERR_INVALID, "routing pointers must be non-NULL");
  if (batch_heads <= 0 || blocks <= 0 || head_dim <= 0) return fail(B2_ERR_INVALID, "routing sizes must be positive");
  if (blocks > 1024) return fail(B2_ERR_UNSUPPORTED, "routing supports at most 1024 blocks");
  if (exact_blocks < 0 || exact_blocks > blocks) return fail(B2_ERR_INVALID, "exact_blocks must be in [0,%d]", blocks);
  if (sink_block != -2 && sink_block != -1 && sink_block != 0)
    return fail(B2_ERR_INVALID, "sink_block must be None, -1, or 0.");
  if (qc_dtype != B2_BF16 && qc_dtype != B2_F32) return fail(B2_ERR_INVALID, "routing centroids must be BF16 or FP32");
  const cudaError_t err = launch_route(qc, qc_dtype, kc, kc_round, h_norm, batch_heads, blocks, head_dim,
                                       exact_blocks, scale, sink_block, indices, sel_bits,
                                       static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "PISA routing launch");
  return ok();
}

int b2_pisa_pair(const uint32_t* sel_bits, int32_t batch_heads, int32_t blocks, int32_t* pairs, void* stream) {
  if (!sel_bits || !pairs) return fail(B2_ERR_INVALID, "pairing pointers must be non-NULL");
  if (batch_heads <= 0 || blocks <= 0) return fail(B2_ERR_INVALID, "pairing sizes must be positive");
  if (!pair_supported(blocks)) return fail(B2_ERR_UNSUPPORTED, "pairing supports at most 608 blocks");
  const cudaError_t err = launch_pair(sel_bits, batch_heads, blocks, pairs, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "PISA pairing launch");
  return ok();
}

int b2_pisa_attention(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out,
                      const int32_t* indices, int32_t exact_blocks, const uint32_t* sel_bits, const int32_t* pairs,
                      const void* kc_bf16, const void* vc_bf16, const void* h_bf16, float scale, float* lse,
                      void* stream) {
  int rc = check_qkv_o(q, k, v, out, true);
  if (rc) return rc;
  if (q->dtype == B2_F32) return fail(B2_ERR_UNSUPPORTED, "PISA attention supports bfloat16 and float16");
  if (q->head_dim != 128) return fail(B2_ERR_UNSUPPORTED, "PISA attention requires D=128");
  const int nb = (q->tokens + kBlock - 1) / kBlock;
  if (exact_blocks < 0 || exact_blocks > nb) return fail(B2_ERR_INVALID, "exact_blocks must be in [0,%d]", nb);
  if (exact_blocks > 0 && indices == nullptr) return fail(B2_ERR_INVALID, "indices are required");
  if (kc_bf16 != nullptr && (vc_bf16 == nullptr || sel_bits == nullptr))
    return fail(B2_ERR_INVALID, "the tail needs centroid values and selection bits");
  AttnParams p = base_params(q, k, v, out, scale);
  p.mode = 1;
  p.pairs = pairs;
  p.indices = indices;
  p.nsel = exact_blocks;
  p.sel_bits = sel_bits;
  p.nb = kc_bf16 ? nb : 0;
  p.kc = kc_bf16;
  p.vc = vc_bf16;
  p.h = h_bf16;
  p.corr_scale = scale / static_cast<float>(q->tokens);
  p.lse = lse;
  const cudaError_t err = run_attention(q, k, v, out, p, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "PISA attention launch");
  return ok();
}

int64_t b2_pisa_workspace_bytes(int32_t batch_heads, int32_t tokens, int32_t head_dim, int32_t exact_blocks) {
  if (batch_heads <= 0 || tokens <= 0 || head_dim != 128 || exact_blocks < 0) return -1;
  return static_cast<int64_t>(carve(nullptr, batch_heads, tokens, head_dim, exact_blocks).total);
}

int b2_pisa_workspace_layout(int32_t batch_heads, int32_t tokens, int32_t head_dim, int32_t exact_blocks,
                             int64_t* offsets, int32_t n) {
  if (batch_heads <= 0 || tokens <= 0 || head_dim != 128 || exact_blocks < 0)
    return fail(B2_ERR_INVALID, "workspace layout needs BH, T > 0, D=128 and exact_blocks >= 0");
  if (offsets == nullptr || n < 0) return fail(B2_ERR_INVALID, "offsets must be non-NULL");
  const PisaWorkspace w = carve(nullptr, batch_heads, tokens, head_dim, exact_blocks);
  for (int i = 0; i < n && i < B2_WS_FIELDS; ++i) offsets[i] = static_cast<int64_t>(w.offset[i]);
  return ok();
}

}  // extern "C"

namespace {
// b2_pisa_forward, optionally storing every output row into n_mirror peer
// copies of the output buffer as well (b2_pisa_forward_mirrored).
int pisa_forward_impl(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out, int32_t exact_blocks,
                      float scale, int32_t sink_block, int32_t stats_mode, int32_t first_order, void* workspace,
                      void* stream, char* const* mirrors, int n_mirror, int multicast) {
  int rc = check_qkv_o(q, k, v, out, true);
  if (rc) return rc;
  if (q->dtype == B2_F32) return fail(B2_ERR_UNSUPPORTED, "PISA supports bfloat16 and float16");
  if (q->head_dim > 128 || q->head_dim % 8 || (stats_mode == B2_STATS_HYD && q->head_dim != 128))
    return fail(B2_ERR_UNSUPPORTED, "PISA requires D=128 (generic PISA: D <= 128, a multiple of 8)");
  if (!(scale > 0.f) || !(scale < 3.4028235e38f))
    return fail(B2_ERR_INVALID, "scale must be representable as a positive finite float32 value.");
  const int nb = (q->tokens + kBlock - 1) / kBlock;
  if (nb > 1024) return fail(B2_ERR_UNSUPPORTED, "PISA supports at most 1024 blocks");
  if (exact_blocks < 0 || exact_blocks > nb) return fail(B2_ERR_INVALID, "exact_blocks must be in [0,%d].", nb);
  if (sink_block != -2 && sink_block != -1 && sink_block != 0)
    return fail(B2_ERR_INVALID, "sink_block must be None, -1, or 0.");
  if (sink_block != -2 && exact_blocks == 0) return fail(B2_ERR_INVALID, "sink_block requires at least one exact block.");
  if (stats_mode != B2_STATS_HYD && stats_mode != B2_STATS_GENERIC) return fail(B2_ERR_INVALID, "unknown stats mode");
  if (stats_mode == B2_STATS_HYD && q->dtype != B2_BF16)
    return fail(B2_ERR_UNSUPPORTED, "HYD PISA requires matching bfloat16 q/k/v.");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int bh = q->batch * q->heads;
  cudaError_t err;
  if (exact_blocks == nb) {
    AttnParams p = base_params(q, k, v, out, scale);
    p.mode = 0;
    set_mirrors(p, mirrors, n_mirror, multicast);
    err = run_attention(q, k, v, out, p, st);
    if (err != cudaSuccess) return cuda_fail(err, "dense attention launch");
    return ok();
  }
  if (workspace == nullptr) return fail(B2_ERR_INVALID, "workspace must be non-NULL");
  // centroids, H and the tail tiles are 128 wide; columns past D stay zero
  PisaWorkspace w = carve(static_cast<char*>(workspace), bh, q->tokens, kTileDim, exact_blocks);
  const bool hyd = stats_mode == B2_STATS_HYD;
  err = run_stats(q, k, v, stats_mode, w.qc, w.kc, w.vstat, w.hsum, hyd ? w.hnorm : nullptr, w.h16, w.partial, st);
  if (err != cudaSuccess) return cuda_fail(err, "PISA statistics launch");
  err = launch_centroid_prep(w.kc, w.vstat, hyd ? 0 : 1, bh, nb, q->tokens, kTileDim, q->dtype, w.kc16, w.vc16, st);
  if (err != cudaSuccess) return cuda_fail(err, "PISA centroid preparation launch");
  const int words = (nb + 31) / 32;
  if (exact_blocks > 0) {
    err = launch_route(w.qc, hyd ? B2_BF16 : B2_F32, w.kc, hyd ? B2_BF16 : B2_F32, hyd ? w.hnorm : nullptr, bh, nb,
                       kTileDim, exact_blocks, scale, hyd ? sink_block : -2, w.indices, w.sel, st);
    if (err != cudaSuccess) return cuda_fail(err, "PISA routing launch");
  } else {
    err = cudaMemsetAsync(w.sel, 0, size_t(bh) * nb * words * 4, st);
    if (err != cudaSuccess) return cuda_fail(err, "selection reset");
  }
  const bool paired = exact_blocks > 0 && pair_supported(nb);  // overlaps must fit in shared memory
  if (paired) {
    err = launch_pair(w.sel, bh, nb, w.pairs, st);
    if (err != cudaSuccess) return cuda_fail(err, "PISA pairing launch");
  }
  AttnParams p = base_params(q, k, v, out, scale);
  p.mode = 1;
  p.pairs = paired ? w.pairs : nullptr;
  p.indices = w.indices;
  p.nsel = exact_blocks;
  p.sel_bits = w.sel;
  p.nb = nb;
  p.kc = w.kc16;
  p.vc = w.vc16;
  p.h = first_order ? w.h16 : nullptr;
  p.corr_scale = scale / static_cast<float>(q->tokens);
  set_mirrors(p, mirrors, n_mirror, multicast);
  err = run_attention(q, k, v, out, p, st);
  if (err != cudaSuccess) return cuda_fail(err, "PISA attention launch");
  return ok();
}
}  // namespace

extern "C" {

int b2_pisa_forward(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out, int32_t exact_blocks,
                    float scale, int32_t sink_block, int32_t stats_mode, int32_t first_order, void* workspace,
                    void* stream) {
  return pisa_forward_impl(q, k, v, out, exact_blocks, scale, sink_block, stats_mode, first_order, workspace, stream,
                           nullptr, 0, 0);
}

}  // extern "C"

namespace {
// Every row a sharded call stores must lie inside [out_buffer, out_buffer +
// bytes): the same offsets are then inside each peer's buffer of that size.
int b2_pisa_forward_mirrored_checks(const b2_view* out, const void* out_buffer, int64_t out_buffer_bytes) {
  int rc = check_view(out, "out");
  if (rc) return rc;
  const int64_t es = esize_of(out->dtype);
  const char* lo_addr = static_cast<const char*>(out->base);
  const int64_t last = (int64_t(out->batch) - 1) * out->stride_b + (int64_t(out->heads) - 1) * out->stride_h +
                       (int64_t(out->tokens) - 1) * out->stride_t + out->head_dim;
  if (out_buffer == nullptr || out_buffer_bytes <= 0 || out->stride_b < 0 || out->stride_h < 0 || out->stride_t < 0 ||
      lo_addr < static_cast<const char*>(out_buffer) ||
      lo_addr + last * es > static_cast<const char*>(out_buffer) + out_buffer_bytes)
    return fail(B2_ERR_INVALID, "out must lie inside [out_buffer, out_buffer + out_buffer_bytes)");
  return B2_OK;
}
}  // namespace

extern "C" {

int b2_pisa_forward_mirrored(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out,
                             int32_t exact_blocks, float scale, int32_t sink_block, int32_t stats_mode,
                             int32_t first_order, const void* out_buffer, int64_t out_buffer_bytes,
                             void* const* mirrors, int32_t n_mirrors, void* workspace, void* stream) {
  if (n_mirrors < 0 || n_mirrors > kMaxMirrors) return fail(B2_ERR_INVALID, "n_mirrors must be in [0,%d]", kMaxMirrors);
  if (n_mirrors > 0 && mirrors == nullptr) return fail(B2_ERR_INVALID, "mirrors must be non-NULL");
  int rc = b2_pisa_forward_mirrored_checks(out, out_buffer, out_buffer_bytes);
  if (rc) return rc;
  const char* lo_addr = static_cast<const char*>(out->base);
  char* peer[kMaxMirrors] = {};
  const int64_t off = lo_addr - static_cast<const char*>(out_buffer);
  for (int i = 0; i < n_mirrors; ++i) {
    if (mirrors[i] == nullptr || reinterpret_cast<uintptr_t>(mirrors[i]) % 16)
      return fail(B2_ERR_INVALID, "mirror buffers must be non-NULL and 16-byte aligned");
    peer[i] = static_cast<char*>(mirrors[i]) + off;
  }
  return pisa_forward_impl(q, k, v, out, exact_blocks, scale, sink_block, stats_mode, first_order, workspace, stream,
                           peer, n_mirrors, 0);
}

int b2_pisa_forward_multicast(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out,
                              int32_t exact_blocks, float scale, int32_t sink_block, int32_t stats_mode,
                              int32_t first_order, const void* out_buffer, int64_t out_buffer_bytes,
                              void* multicast_buffer, void* workspace, void* stream) {
  if (multicast_buffer == nullptr || reinterpret_cast<uintptr_t>(multicast_buffer) % 16)
    return fail(B2_ERR_INVALID, "multicast_buffer must be non-NULL and 16-byte aligned");
  void* const one[1] = {multicast_buffer};
  // the same bounds checks and offset as the mirrored form
  int rc = b2_pisa_forward_mirrored_checks(out, out_buffer, out_buffer_bytes);
  if (rc) return rc;
  char* mc = static_cast<char*>(one[0]) + (static_cast<const char*>(out->base) - static_cast<const char*>(out_buffer));
  return pisa_forward_impl(q, k, v, out, exact_blocks, scale, sink_block, stats_mode, first_order, workspace, stream,
                           &mc, 1, 1);
}

int b2_pisa_forward_spatial_host(const void* q_host, const void* k_host, const void* v_host, void* out_host,
                                 void* q_dev, void* k_dev, void* v_dev, void* out_dev, int32_t batch, int32_t heads,
                                 int32_t grid_h, int32_t grid_w, int32_t head_dim, int32_t dtype,
                                 int32_t exact_blocks, float scale, int32_t sink_block, int32_t heads_per_stage,
                                 void* workspace, void* stream) {
  if (!q_host || !k_host || !v_host || !out_host || !q_dev || !k_dev || !v_dev || !out_dev)
    return fail(B2_ERR_INVALID, "host and device buffers must be non-NULL");
  if (batch <= 0 || heads <= 0 || grid_h <= 0 || grid_w <= 0 || head_dim != 128)
    return fail(B2_ERR_INVALID, "expected B, H > 0, a positive grid and D=128");
  if (dtype != B2_BF16 && dtype != B2_F16) return fail(B2_ERR_UNSUPPORTED, "16-bit q/k/v only");
  if (heads_per_stage <= 0 || heads % heads_per_stage != 0)
    return fail(B2_ERR_INVALID, "heads_per_stage must divide heads");
  if (!is_pinned_host(q_host) || !is_pinned_host(k_host) || !is_pinned_host(v_host) || !is_pinned_host(out_host))
    return fail(B2_ERR_INVALID, "host buffers must be page-locked (pinned)");
  const int32_t tokens = grid_h * grid_w;
  const size_t es = 2;
  const size_t pitch = size_t(heads) * head_dim * es;  // one raster row: all heads of one token
  const size_t width = size_t(heads_per_stage) * head_dim * es;
  const size_t batch_bytes = size_t(tokens) * pitch;
  const int per_batch = heads / heads_per_stage;
  const int stages = batch * per_batch;
  HostPipe* pipe = nullptr;
  cudaError_t err = host_pipe(&pipe);
  if (err != cudaSuccess) return cuda_fail(err, "copy stream set-up");
  // the streams and events are shared by every call on this device: calls
  // from several host threads enqueue one after the other
  std::lock_guard<std::mutex> serial(pipe->enqueue);
  if ((err = host_pipe_events(*pipe, stages)) != cudaSuccess) return cuda_fail(err, "event set-up");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // copies start after the work already queued on the caller's stream
  if ((err = cudaEventRecord(pipe->start, st)) != cudaSuccess) return cuda_fail(err, "event record");
  if ((err = cudaStreamWaitEvent(pipe->h2d, pipe->start, 0)) != cudaSuccess) return cuda_fail(err, "stream wait");
  if ((err = cudaStreamWaitEvent(pipe->d2h, pipe->start, 0)) != cudaSuccess) return cuda_fail(err, "stream wait");
  for (int s = 0; s < stages; ++s) {
    const int b = s / per_batch;
    const int h0 = (s - b * per_batch) * heads_per_stage;
    const size_t off = size_t(b) * batch_bytes + size_t(h0) * head_dim * es;
    cudaEvent_t in = pipe->ev[3 * s], ready = pipe->ev[3 * s + 1];
    const void* srcs[3] = {q_host, k_host, v_host};
    void* dsts[3] = {q_dev, k_dev, v_dev};
    for (int i = 0; i < 3; ++i) {
      err = cudaMemcpy2DAsync(static_cast<char*>(dsts[i]) + off, pitch, static_cast<const char*>(srcs[i]) + off, pitch,
                              width, tokens, cudaMemcpyHostToDevice, pipe->h2d);
      if (err != cudaSuccess) return cuda_fail(err, "input copy");
    }
    if ((err = cudaEventRecord(in, pipe->h2d)) != cudaSuccess) return cuda_fail(err, "event record");
    if ((err = cudaStreamWaitEvent(st, in, 0)) != cudaSuccess) return cuda_fail(err, "stream wait");
    b2_view v[4];
    void* bases[4] = {q_dev, k_dev, v_dev, out_dev};
    for (int i = 0; i < 4; ++i) {
      v[i].base = static_cast<char*>(bases[i]) + off;
      v[i].stride_b = int64_t(tokens) * heads * head_dim;
      v[i].stride_h = head_dim;
      v[i].stride_t = int64_t(heads) * head_dim;
      v[i].batch = 1;
      v[i].heads = heads_per_stage;
      v[i].tokens = tokens;
      v[i].head_dim = head_dim;
      v[i].dtype = dtype;
      v[i].order = B2_ORDER_TILED8;
      v[i].grid_h = grid_h;
      v[i].grid_w = grid_w;
    }
    const int rc = b2_pisa_forward(&v[0], &v[1], &v[2], &v[3], exact_blocks, scale, sink_block, B2_STATS_HYD, 1,
                                   workspace, stream);
    if (rc) return rc;
    if ((err = cudaEventRecord(ready, st)) != cudaSuccess) return cuda_fail(err, "event record");
    if ((err = cudaStreamWaitEvent(pipe->d2h, ready, 0)) != cudaSuccess) return cuda_fail(err, "stream wait");
    err = cudaMemcpy2DAsync(static_cast<char*>(out_host) + off, pitch, static_cast<const char*>(out_dev) + off, pitch,
                            width, tokens, cudaMemcpyDeviceToHost, pipe->d2h);
    if (err != cudaSuccess) return cuda_fail(err, "output copy");
  }
  cudaEvent_t done = pipe->ev[2];
  if ((err = cudaEventRecord(done, pipe->d2h)) != cudaSuccess) return cuda_fail(err, "event record");
  if ((err = cudaStreamWaitEvent(st, done, 0)) != cudaSuccess) return cuda_fail(err, "stream wait");
  return ok();
}

int b2_full_attention(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out, float scale,
                      float* lse, void* stream) {
  int rc = check_qkv_o(q, k, v, out, false);
  if (rc) return rc;
  if (q->dtype == B2_F32) return fail(B2_ERR_UNSUPPORTED, "full attention supports float16 and bfloat16");
  if (q->head_dim > 128 || q->head_dim % 8)
    return fail(B2_ERR_UNSUPPORTED, "full attention supports D <= 128, a multiple of 8");
  AttnParams p = base_params(q, k, v, out, scale);
  p.mode = 0;
  p.lse = lse;
  const cudaError_t err = run_attention(q, k, v, out, p, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "full attention launch");
  return ok();
}

int b2_fixed_block_attention_masked(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out,
                                    float scale, int32_t causal, const float* bias, int64_t bias_bh_stride,
                                    void* stream) {
  int rc = check_qkv_o(q, k, v, out, true);
  if (rc) return rc;
  if (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) % 16 || bias_bh_stride < 0 || bias_bh_stride % 4))
    return fail(B2_ERR_INVALID, "mask bias must be 16-byte aligned with a non-negative stride divisible by 4");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (q->dtype == B2_F32) {
    if (q->head_dim > 128) return fail(B2_ERR_UNSUPPORTED, "FP32 fixed-block attention supports D <= 128");
    err = launch_fixed_f32(make_rows(*q), make_rows(*k), make_rows(*v), make_rows(*out), q->batch * q->heads, scale,
                           causal, bias, bias_bh_stride, st);
  } else {
    if (q->head_dim != 32 && q->head_dim != 64 && q->head_dim != 128)
      return fail(B2_ERR_UNSUPPORTED, "fixed-block attention supports D in {32,64,128}");
    AttnParams p = base_params(q, k, v, out, scale);
    p.mode = 2;
    p.causal = causal ? 1 : 0;
    p.bias = bias;
    p.bias_bh_stride = bias_bh_stride;
    err = run_attention(q, k, v, out, p, st);
  }
  if (err != cudaSuccess) return cuda_fail(err, "fixed-block attention launch");
  return ok();
}

int b2_fixed_block_attention(const b2_view* q, const b2_view* k, const b2_view* v, const b2_view* out, float scale,
                             int32_t causal, void* stream) {
  return b2_fixed_block_attention_masked(q, k, v, out, scale, causal, nullptr, 0, stream);
}

int b2_pack_block_bias(const void* mask, int32_t mask_dtype, int64_t stride_bh, int64_t stride_t, int64_t stride_key,
                       int32_t mask_bh, int32_t tokens, float* bias, void* stream) {
  if (mask == nullptr || bias == nullptr) return fail(B2_ERR_INVALID, "mask and bias must be non-NULL");
  if (mask_bh <= 0 || tokens <= 0) return fail(B2_ERR_INVALID, "mask sizes must be positive");
  if (mask_dtype < B2_MASK_BOOL || mask_dtype > B2_MASK_BF16) return fail(B2_ERR_INVALID, "unknown mask dtype");
  if (stride_bh < 0 || stride_t < 0 || stride_key < 0) return fail(B2_ERR_INVALID, "mask strides must be >= 0");
  if (reinterpret_cast<uintptr_t>(bias) % 16) return fail(B2_ERR_INVALID, "bias must be 16-byte aligned");
  const cudaError_t err = launch_block_bias(mask, mask_dtype, stride_bh, stride_t, stride_key, mask_bh, tokens, bias,
                                            static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "mask bias launch");
  return ok();
}

int b2_pack_rows(const b2_view* src, void* dst, void* stream) {
  int rc = check_view(src, "src");
  if (rc) return rc;
  if (dst == nullptr || reinterpret_cast<uintptr_t>(dst) % 16) return fail(B2_ERR_INVALID, "dst must be 16-byte aligned");
  const cudaError_t err = launch_pack_rows(make_rows(*src), src->batch * src->heads, dst, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "pack launch");
  return ok();
}

int b2_unpack_rows(const void* src, const b2_view* dst, void* stream) {
  int rc = check_view(dst, "dst");
  if (rc) return rc;
  if (src == nullptr || reinterpret_cast<uintptr_t>(src) % 16) return fail(B2_ERR_INVALID, "src must be 16-byte aligned");
  const cudaError_t err = launch_unpack_rows(src, make_rows(*dst), dst->batch * dst->heads, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "unpack launch");
  return ok();
}

int b2_merge_epilogue(const void* exact, const float* exact_lse, const void* approx, const float* approx_lse,
                      const float* correction, const b2_view* dst, void* stream) {
  int rc = check_view(dst, "dst");
  if (rc) return rc;
  if (dst->dtype == B2_F32) return fail(B2_ERR_UNSUPPORTED, "merge epilogue writes bfloat16 or float16");
  if (!exact || !exact_lse || !approx || !approx_lse || !correction)
    return fail(B2_ERR_INVALID, "merge inputs must be non-NULL");
  for (const void* ptr : {exact, approx, static_cast<const void*>(correction)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return fail(B2_ERR_INVALID, "merge inputs must be 16-byte aligned");
  const cudaError_t err = launch_merge(exact, exact_lse, approx, approx_lse, correction, make_rows(*dst), dst->dtype,
                                       dst->batch * dst->heads, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "merge epilogue launch");
  return ok();
}

int b2_h3_pack(const b2_view* views, int32_t n, void* dst, void* stream) {
  if (views == nullptr || n < 1 || n > 3) return fail(B2_ERR_INVALID, "h3 pack takes 1..3 views");
  if (dst == nullptr || reinterpret_cast<uintptr_t>(dst) % 16) return fail(B2_ERR_INVALID, "dst must be 16-byte aligned");
  for (int i = 0; i < n; ++i) {
    int rc = check_view(&views[i], "h3 view");
    if (rc) return rc;
    if (!same_bht(&views[0], &views[i]) || views[i].dtype != views[0].dtype)
      return fail(B2_ERR_INVALID, "h3 views must share shape and dtype");
  }
  const int64_t bytes = int64_t(views[0].batch) * views[0].heads * views[0].tokens * views[0].head_dim *
                        esize_of(views[0].dtype);
  for (int i = 0; i < n; ++i) {
    const cudaError_t err = launch_pack_rows(make_rows(views[i]), views[i].batch * views[i].heads,
                                             static_cast<char*>(dst) + i * bytes, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "h3 pack launch");
  }
  return ok();
}

}  // extern "C"
