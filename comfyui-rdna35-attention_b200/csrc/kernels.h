// Internal launch interface shared by the C ABI layer and the kernels.
#pragma once
#include "common.cuh"

namespace b2 {
constexpr int kMaxMirrors = 7;  // peer copies of an output (head-sharded calls over up to 8 GPUs)
// Parameters of the fused attention kernel (see attn_mma.cu).
struct AttnParams {
  Rows q, k, v, o;
  int tq, tk;
  int mode;
  const int32_t* indices;
  int nsel;
  const uint32_t* sel_bits;
  int nb;
  const void* kc;
  const void* vc;
  const void* h;
  float scale;
  float scale_log2;
  float corr_scale;
  float* lse;
  int causal;
  long long* trace;
  int debug_withhold_q;  // diagnostics: never load Q, so the pipeline's bounded waits run out
  const float* bias;     // fixed-block masks: FP32 [BHm][T][64] additive terms, or NULL
  int64_t bias_bh_stride;  // elements between (batch, head) rows of bias; 0 = one mask for all
  int n_mirror;            // peer copies of the output written with every row (tcgen05 kernel only)
  char* mirror[kMaxMirrors];
  int mirror_multicast;    // 1: mirror[0] is a multicast address reaching every GPU's copy
  const int32_t* pairs;  // optional [BH][ceil(nq/2)][2] query-block pairing (-1: single)
};
// Arguments of the tcgen05 attention kernel (see attn_umma.cu).
struct UmmaArgs {
  int q_kind, kv_kind;  // 0 = linear 4D map, 1 = 8x8-tiled 5D map
  int heads, tq, tk, nqb;
  int frames, tiles_per_row, tiles_per_frame;
  int mode;
  const int32_t* indices;
  int nsel;
  const uint32_t* sel_bits;
  int nb;
  int has_corr;
  float scale_log2, corr_scale, log2_last;
  int causal;
  Rows o;
  float* lse;
  int* status;
  const int32_t* pairs;
  long long* trace;  // optional clock64 timeline of CTA (0,0): [tile][6] + start
  int debug_withhold_q;  // diagnostics (b2_debug_withhold_q): Q is never loaded
  const float* bias;     // fixed-block mask terms (mode DIAG), see AttnParams
  int64_t bias_bh_stride;
  int n_mirror;  // peer output copies, see AttnParams
  char* mirror[kMaxMirrors];
  int mirror_multicast;
};
bool umma_supported(const b2_view& q, const b2_view& k, const b2_view& v, const b2_view& o);
cudaError_t launch_attn_umma(const b2_view& qv, const b2_view& kv, const b2_view& vv, const b2_view& ov,
                             const AttnParams& p, int* status, cudaStream_t stream, bool* launched);
int* device_status_ptr();
// Query-block pairing fits in shared memory for blocks <= 608.
bool pair_supported(int blocks);
cudaError_t launch_pair(const uint32_t* sel_bits, int batch_heads, int blocks, int32_t* pairs, cudaStream_t stream);
cudaError_t launch_stats(const Rows& q, const Rows& k, const Rows& v, int dtype, int mode, int batch_heads,
                         int blocks, void* q_centroids, float* k_centroids, void* v_stats, float* h_sum,
                         float* h_norm, void* h_half, float* partial, cudaStream_t stream);
int64_t stats_partial_bytes(int batch_heads, int blocks);
int stats_group_size(int batch_heads, int blocks);
int stats_group_for_blocks(int blocks);
cudaError_t launch_stats_reduce(const float* partial, int groups, int batch_heads, float* h_sum, void* h_half,
                                int dtype, cudaStream_t stream);
cudaError_t launch_stats_umma(const b2_view& q, const b2_view& k, const b2_view& v, int mode, int group,
                              void* q_centroids, float* k_centroids, void* v_stats, float* h_norm, float* partial,
                              int* status, cudaStream_t stream, bool* launched);
cudaError_t launch_route(const void* qc, int qc_dtype, const float* kc, int kc_round, const float* h_norm,
                         int batch_heads, int blocks, int dim, int k, float scale, int sink, int32_t* indices,
                         uint32_t* sel_bits, cudaStream_t stream);
cudaError_t launch_attn_mma(const AttnParams& p, int dtype, int batch_heads, cudaStream_t stream);
cudaError_t launch_pack_rows(const Rows& src, int batch_heads, void* dst, cudaStream_t stream);
cudaError_t launch_unpack_rows(const void* src, const Rows& dst, int batch_heads, cudaStream_t stream);
cudaError_t launch_merge(const void* exact, const float* exact_lse, const void* approx, const float* approx_lse,
                         const float* corr, const Rows& dst, int dtype, int batch_heads, cudaStream_t stream);
cudaError_t launch_centroid_prep(const float* kc, const void* vstat, int vstat_is_sum, int batch_heads, int blocks,
                                 int tokens, int dim, int dtype, void* kc16, void* vc16, cudaStream_t stream);
cudaError_t launch_fixed_f32(const Rows& q, const Rows& k, const Rows& v, const Rows& o, int batch_heads,
                             float scale, int causal, const float* bias, int64_t bias_bh_stride,
                             cudaStream_t stream);
cudaError_t launch_block_bias(const void* mask, int mask_dtype, int64_t s_bh, int64_t s_row, int64_t s_col,
                              int mask_rows_bh, int tokens, float* bias, cudaStream_t stream);
// Host-side helpers of the C ABI layer (capi.cu): the shared statistics
// argument checks and the thread-local error string behind b2_last_error.
int check_stats_call(const b2_view* q, const b2_view* k, const b2_view* v, int mode, const void* q_centroids,
                     const float* k_centroids, const void* v_stats, const float* h_sum);
int report_error(int code, const char* msg);
int report_cuda_error(cudaError_t err, const char* what);
int report_ok();
bool tcgen05_kernels_enabled();
}  // namespace b2
