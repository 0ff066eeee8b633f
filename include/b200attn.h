/*
 * b200attn.h -- C ABI of the B200 (sm_100a) attention hot path.
 *
 * Every entry point takes plain device pointers, element strides and a
 * cudaStream_t passed as void*, launches asynchronously on that stream and
 * returns 0 on success or a B2_ERR_* code.  b2_last_error() returns a
 * thread-local message describing the most recent failure.  No entry point
 * synchronises the stream or allocates device memory; callers own every
 * buffer (outputs and the scratch workspace sized by b2_pisa_workspace_bytes).
 *
 * Reference interfaces replaced (paths inside the ComfyUI-RDNA35-Attention
 * project):
 *   native/rdna35_pisa_ck/csrc/pisa_kernels.cu:563-594  pisa_block_stats
 *   native/rdna35_pisa_ck/csrc/pisa_kernels.cu:597-635  pisa_block_stats_hyd
 *   native/rdna35_pisa_ck/csrc/pisa_kernels.cu:638-676  pisa_pack_spatial_qkv
 *   native/rdna35_pisa_ck/csrc/pisa_kernels.cu:679-707  pisa_unpack_spatial_output
 *   native/rdna35_pisa_ck/csrc/pisa_kernels.cu:710-773  pisa_fuse_spatial_epilogue
 *   native/rdna35_pisa_ck/csrc/bindings.cpp:70-82       build_info
 *   native/rdna35_pisa_ck/rdna35_pisa_ck/__init__.py:233-316 _forward_impl
 *       (routing + FlexAttention exact/tail + correction GEMM + merge)
 *   rdna35_block_attention/triton_kernel.py:53-100,200-244 fixed-block kernel
 *   rdna35_block_attention/triton_kernel.py:113-197      full attention kernel
 *   rdna35_block_attention/minimax_h3_gfx1151_attention.py:64-74 H3 pack
 *   rdna35_block_attention/pisa_kernel.py:49-131         Triton PISA stats
 */
#ifndef B200ATTN_H
#define B200ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200ATTN_API_VERSION 7

enum b2_status {
  B2_OK = 0,
  B2_ERR_INVALID = 1,      /* bad shape, stride, alignment or argument */
  B2_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement */
  B2_ERR_CUDA = 3,         /* a CUDA runtime call or launch failed */
  B2_ERR_DEVICE = 4        /* the current device is not sm_100 */
};

enum b2_dtype { B2_BF16 = 0, B2_F16 = 1, B2_F32 = 2 };

/* Token order of a row view.  B2_ORDER_LINEAR: row t is token t.
 * B2_ORDER_TILED8: row t walks 8x8 spatial tiles of a grid_h x grid_w raster
 * (per frame, frames = tokens / (grid_h*grid_w)); within a tile rows go
 * row-major.  This is the block-major order of pisa_kernels.cu:55-64
 * (ordered_to_raster) and generic_pisa.py:17-52. */
enum b2_order { B2_ORDER_LINEAR = 0, B2_ORDER_TILED8 = 1 };

/* A [B,H,T,D] tensor view addressed by element strides.  Row (b,h,t) starts
 * at base + b*stride_b + h*stride_h + map(t)*stride_t, where map is given by
 * order/grid_h/grid_w; the D elements of a row are contiguous. */
typedef struct b2_view {
  void* base;
  int64_t stride_b, stride_h, stride_t;
  int32_t batch, heads, tokens, head_dim;
  int32_t dtype;   /* enum b2_dtype */
  int32_t order;   /* enum b2_order */
  int32_t grid_h, grid_w;
} b2_view;

/* Statistic semantics. B2_STATS_HYD follows pisa_kernels.cu:167-244 (sums
 * times 1/len, BF16 q/v centroids, FP32-centred K).  B2_STATS_GENERIC follows
 * generic_pisa.py:106-138 + pisa_kernel.py:49-84 (sums divided by len, FP32
 * centroids, BF16-rounded centred K, V sums). */
enum b2_stats_mode { B2_STATS_HYD = 0, B2_STATS_GENERIC = 1, B2_STATS_SCALED = 2 };
/* B2_STATS_SCALED: centroids only, each element times 1/len before the sum so
 * extreme BF16 inputs cannot overflow (pisa_kernels.cu:130-164, block_stats). */

const char* b2_last_error(void);
/* Name of the attention kernel the calling thread launched last:
 * "tcgen05" (TMA + tcgen05.mma + TMEM) or "mma_sync" (warp-level MMA, used
 * for views the TMA maps cannot express or when B200ATTN_KERNEL=mma). */
const char* b2_last_kernel(void);
/* Synchronously reads and clears the current device's kernel status word:
 * 0 when every kernel finished normally, else (1 << 8 | site) after a
 * pipeline wait timed out (the kernel then ends early; outputs are invalid).
 * This is the one entry point that synchronises (it copies 4 bytes). */
int b2_read_status(int32_t* status);
/* Diagnostics: when device_buffer is not NULL, later tcgen05 attention
 * launches of this process record clock64() timestamps of CTA (0,0) into it
 * ([256 tiles][6 events] + start + [256] P.V issue times + [256][4] P arrival
 * times of the four softmax warps + [256] S issue-return times, int64: 3073
 * entries; see attn_umma.cu).  NULL disables. */
int b2_set_trace(long long* device_buffer);
/* Diagnostics (no counterpart in the reference): while enabled, later
 * tcgen05 attention launches of this process never load their Q tile, so
 * their pipelines stall on a barrier that nothing completes.  Every wait of
 * the kernel is bounded (about 2^31 cycles): the CTAs then record
 * (1 << 8 | site) in the status word, wait for their own loads in flight,
 * free TMEM and return, leaving the context usable.  Used by the tests of
 * that timeout path; outputs of such launches are invalid. */
int b2_debug_withhold_q(int32_t enable);
int b2_api_version(void);
/* Writes a NUL-terminated "key=value;..." build description. */
int b2_build_info(char* buffer, int64_t capacity);
/* Fails with B2_ERR_DEVICE unless device_index is an sm_100 GPU. */
int b2_check_device(int device_index);

/* ---- PISA block statistics (pisa_kernels.cu:597-635, pisa_kernel.py:90-131).
 * q,k,v: [BH,T,D] views (D=128).  Outputs are contiguous:
 *   q_centroids [BH,nb,D] (BF16 for HYD, FP32 for GENERIC),
 *   k_centroids [BH,nb,D] FP32,
 *   v_stats     [BH,nb,D] (HYD: BF16 means; GENERIC: FP32 sums),
 *   h_sum       [BH,D,D] FP32, h_norm [BH,nb] FP32 (may be NULL),
 *   h_bf16      [BH,D,D] BF16 copy of h_sum (may be NULL).
 * workspace: b2_stats_workspace_bytes() bytes of scratch. */
int64_t b2_stats_workspace_bytes(int32_t batch_heads, int32_t tokens, int32_t head_dim);
int b2_pisa_block_stats(const b2_view* q, const b2_view* k, const b2_view* v,
                        int32_t mode, void* q_centroids, float* k_centroids,
                        void* v_stats, float* h_sum, float* h_norm,
                        void* h_bf16, void* workspace, void* stream);

/* ---- Allocation-free block statistics.  No counterpart in the reference.
 * Same inputs, outputs and argument checks as b2_pisa_block_stats, but the
 * partial H sums go to an 8 MiB array compiled into the library (one copy per
 * GPU, held until the process exits) instead of a caller workspace, for
 * callers that cannot allocate device memory when they run (allocator
 * callbacks, fixed memory pools, plugin hosts that only hand out input/output
 * buffers).
 * Limit: batch*heads*ceil(nb/group) partials of 64 KiB must fit in 8 MiB,
 * i.e. batch*heads <= 128; larger requests fail with B2_ERR_UNSUPPORTED.
 * Blocks are grouped as in b2_pisa_block_stats (so h_sum/h_bf16 match it bit
 * for bit) unless the array forces larger groups; then H is summed in another
 * order and matches only within FP32 reassociation.  Centroids and h_norm
 * always match bit for bit.
 * Every call looks up the array's device address in the current device's
 * context (cudaGetSymbolAddress; make the first call on a device before any
 * stream capture).  Every call shares the array and overwrites all of it that
 * it reads, so no clearing is needed, but calls whose kernels overlap on the
 * same GPU (different streams, or host threads) race on it.  Errors are
 * reported by b2_last_error(); b2_noalloc_last_error() returns the same
 * string. */
int b2_pisa_block_stats_noalloc(const b2_view* q, const b2_view* k,
                                const b2_view* v, int32_t mode,
                                void* q_centroids, float* k_centroids,
                                void* v_stats, float* h_sum, float* h_norm,
                                void* h_bf16, void* stream);
const char* b2_noalloc_last_error(void);

/* ---- HYD routing + top-k (rdna35_pisa_ck/__init__.py:258-269; generic
 * routing without the h_norm bias: generic_pisa.py:172-184).
 * scores[i,j] = dot(qc_i, kc_j)*scale (+ log(h_norm_j + 1e-5) when h_norm is
 * not NULL); sink_block in {-2 (none), -1, 0} forces that column to +inf.
 * qc: [BH,nb,D] (qc_dtype BF16 or FP32); kc: [BH,nb,D] FP32, rounded to the
 * routing dtype kc_round (B2_BF16 rounds to BF16 first, B2_F32 keeps FP32).
 * Writes indices [BH,nb,k] int32 sorted ascending and sel_bits
 * [BH,nb,ceil(nb/32)] uint32 (bit j set when block j is exact). */
int b2_pisa_route(const void* qc, int32_t qc_dtype, const float* kc,
                  int32_t kc_round, const float* h_norm, int32_t batch_heads,
                  int32_t blocks, int32_t head_dim, int32_t exact_blocks,
                  float scale, int32_t sink_block, int32_t* indices,
                  uint32_t* sel_bits, void* stream);

/* ---- Fused PISA attention: exact block-sparse softmax attention over the
 * selected KV blocks + centroid tail (logits q.kc*scale + log len, selected
 * masked) + first-order correction q.H*scale/T weighted by the tail mass,
 * merged in one online softmax (rdna35_pisa_ck/__init__.py:272-316,
 * pisa_kernels.cu:296-340).  The output view may be tiled (raster write).
 * kc_bf16/vc_bf16: [BH,nb,D] centroid rows in the input's 16-bit type
 * (kc NULL: no tail); h_bf16 [BH,D,D] in the same type or NULL to skip the
 * correction; lse: [BH,T] FP32 or NULL; pairs: b2_pisa_pair output or NULL
 * (query blocks 2p, 2p+1 share a CTA).  q/k/v/out share [B,H,T,D=128]. */
int b2_pisa_attention(const b2_view* q, const b2_view* k, const b2_view* v,
                      const b2_view* out, const int32_t* indices,
                      int32_t exact_blocks, const uint32_t* sel_bits,
                      const int32_t* pairs, const void* kc_bf16,
                      const void* vc_bf16, const void* h_bf16, float scale,
                      float* lse, void* stream);

/* ---- Query-block pairing for the attention CTAs: pairs[bh][p] = (a, b) with
 * b = -1 for an unpaired block; blocks are matched greedily (ascending a) with
 * the unpaired block of largest selection overlap, so each CTA's union of
 * exact key blocks is small.  No counterpart in the reference (its
 * FlexAttention visits each query block's list separately).  nb <= 608. */
int b2_pisa_pair(const uint32_t* sel_bits, int32_t batch_heads, int32_t blocks,
                 int32_t* pairs, void* stream);

/* ---- Whole PISA forward in one call: stats, routing, fused attention.
 * stats_mode B2_STATS_HYD: rdna35_pisa_ck forward / forward_spatial_bhtd
 * (__init__.py:233-316); B2_STATS_GENERIC: generic_pisa_attention
 * (generic_pisa.py:141-232, sink_block must be -2).  first_order=0 drops the
 * correction term (generic_pisa.py:226-228).  exact_blocks == nb runs dense
 * attention.  workspace: b2_pisa_workspace_bytes() bytes. */
int64_t b2_pisa_workspace_bytes(int32_t batch_heads, int32_t tokens,
                                int32_t head_dim, int32_t exact_blocks);
int b2_pisa_forward(const b2_view* q, const b2_view* k, const b2_view* v,
                    const b2_view* out, int32_t exact_blocks, float scale,
                    int32_t sink_block, int32_t stats_mode,
                    int32_t first_order, void* workspace, void* stream);

/* ---- Byte offsets of the buffers b2_pisa_forward carves out of its
 * workspace, so a caller can read the routing it used (no counterpart in the
 * reference, whose forward keeps its indices internal;
 * rdna35_pisa_ck/__init__.py:262-264 computes them).  Writes up to n offsets,
 * indexed by the B2_WS_* constants below, and returns 0, or B2_ERR_INVALID
 * for sizes b2_pisa_workspace_bytes rejects.  After a sparse b2_pisa_forward
 * (0 < exact_blocks < nb) on `stream` completes:
 *   B2_WS_INDICES  int32  [BH,nb,exact_blocks] routed key blocks, ascending;
 *   B2_WS_SEL      uint32 [BH,nb,ceil(nb/32)] the same sets as bitsets;
 *   B2_WS_HNORM    FP32   [BH,nb] HYD covariance norms;
 *   B2_WS_QC/KC    query (BF16 HYD / FP32 generic) and FP32 key centroids
 *                  [BH,nb,D]; B2_WS_HSUM FP32 [BH,D,D]. */
enum {
  B2_WS_QC = 0, B2_WS_KC = 1, B2_WS_VSTAT = 2, B2_WS_HSUM = 3, B2_WS_H16 = 4,
  B2_WS_HNORM = 5, B2_WS_KC16 = 6, B2_WS_VC16 = 7, B2_WS_INDICES = 8,
  B2_WS_SEL = 9, B2_WS_PAIRS = 10, B2_WS_PARTIAL = 11, B2_WS_FIELDS = 12
};
int b2_pisa_workspace_layout(int32_t batch_heads, int32_t tokens,
                             int32_t head_dim, int32_t exact_blocks,
                             int64_t* offsets, int32_t n);

/* ---- b2_pisa_forward for one rank of a head-sharded call (no counterpart in
 * the reference, whose path runs on one device).  `out` is this rank's head
 * slice inside the output buffer [out_buffer, out_buffer + out_buffer_bytes)
 * (e.g. the BHTD view of columns [h0*D, h1*D) of a [B,T,H*D] raster); every
 * output row is stored there and, in the same kernel epilogue, at the same
 * byte offset inside each of the n_mirrors (<= 7) peer buffers mirrors[i],
 * which are other GPUs' copies of that buffer mapped into this process
 * (peer-to-peer stores over NVLink).  All ranks writing their slices this way
 * assemble the full output on every GPU without a separate all-gather; the
 * caller synchronises the ranks before reading it.  Rejects an `out` view
 * that reaches outside the buffer.  tcgen05 path only (D = 128 views TMA can
 * address); other requests fail with B2_ERR_CUDA. */
int b2_pisa_forward_mirrored(const b2_view* q, const b2_view* k,
                             const b2_view* v, const b2_view* out,
                             int32_t exact_blocks, float scale,
                             int32_t sink_block, int32_t stats_mode,
                             int32_t first_order, const void* out_buffer,
                             int64_t out_buffer_bytes, void* const* mirrors,
                             int32_t n_mirrors, void* workspace, void* stream);

/* ---- b2_pisa_forward_mirrored with one multicast address instead of peer
 * pointers (no counterpart in the reference): multicast_buffer is an NVLink
 * multicast mapping of every GPU's copy of the output buffer (NVSwitch
 * SHARP), so each output row is stored once (multimem.st) and the switch
 * writes it into every copy, this GPU's included.  Same bounds checks;
 * one-warpgroup tcgen05 layout only. */
int b2_pisa_forward_multicast(const b2_view* q, const b2_view* k,
                              const b2_view* v, const b2_view* out,
                              int32_t exact_blocks, float scale,
                              int32_t sink_block, int32_t stats_mode,
                              int32_t first_order, const void* out_buffer,
                              int64_t out_buffer_bytes, void* multicast_buffer,
                              void* workspace, void* stream);

/* ---- Pipelined PISA HYD forward from host memory.  No counterpart in the
 * reference (its forward_spatial_bhtd, rdna35_pisa_ck/__init__.py:406-433,
 * takes device tensors).  q/k/v_host and out_host: page-locked raster
 * buffers [B, grid_h*grid_w, H, 128] (BF16/FP16); q/k/v/out_dev: device
 * buffers of the same layout.  The call runs as B*H/heads_per_stage stages
 * of heads_per_stage heads of one batch: the inputs of a stage are copied in
 * on a copy stream, the stage's forward (the semantics of b2_pisa_forward,
 * B2_STATS_HYD, first-order on, tiled 8x8 token order) runs on `stream`, and
 * its output is copied out on a second copy stream, so transfers overlap the
 * compute of neighbouring stages.  `stream` waits for the last copy; the
 * host output is valid once `stream` has been synchronised.  workspace:
 * b2_pisa_workspace_bytes(heads_per_stage, T, 128, exact_blocks) bytes. */
int b2_pisa_forward_spatial_host(const void* q_host, const void* k_host,
                                 const void* v_host, void* out_host,
                                 void* q_dev, void* k_dev, void* v_dev,
                                 void* out_dev, int32_t batch, int32_t heads,
                                 int32_t grid_h, int32_t grid_w,
                                 int32_t head_dim, int32_t dtype,
                                 int32_t exact_blocks, float scale,
                                 int32_t sink_block, int32_t heads_per_stage,
                                 void* workspace, void* stream);

/* ---- Exact full attention (triton_kernel.py:113-197): out = softmax(q k^T
 * scale) v over all Tk keys, no mask.  q: [B,H,Tq,D], k/v: [B,H,Tk,D]
 * views, D in {64,128}, BF16 or FP16.  lse may be NULL. */
int b2_full_attention(const b2_view* q, const b2_view* k, const b2_view* v,
                      const b2_view* out, float scale, float* lse, void* stream);

/* ---- Fixed 64-token block-diagonal attention (triton_kernel.py:53-100 and
 * reference.py:159-200): each query block attends to its own key block.
 * BF16/FP16 (D in {32,64,128}) or FP32 (D <= 128).  causal: 0/1. */
int b2_fixed_block_attention(const b2_view* q, const b2_view* k,
                             const b2_view* v, const b2_view* out, float scale,
                             int32_t causal, void* stream);

/* ---- Masked fixed-block attention (reference.py:114-200: the diagonal
 * 64x64 block of a [T,T] / [N,T,T] / [B,H,T,T] mask, boolean masks keeping
 * True entries, other masks added to the scores).
 * b2_pack_block_bias reads a mask as [mask_bh, T, T] through element strides
 * (stride_bh may be 0 for one mask shared by every (batch, head)) and writes
 * bias [mask_bh, T, 64] FP32: entry (bh, t, c) is the mask term of query t
 * and key start(t)+c of t's own block (bool: 0 or -inf; float: the value;
 * -inf past a ragged last block).  b2_fixed_block_attention_masked is
 * b2_fixed_block_attention with bias[bh * bias_bh_stride + t * 64 + c] added
 * to the scaled score (after the causal mask); bias_bh_stride is T*64, or 0
 * for a shared mask.  A query row with every key masked yields NaN, as the
 * reference's softmax does. */
enum b2_mask_dtype { B2_MASK_BOOL = 0, B2_MASK_F32 = 1, B2_MASK_F16 = 2, B2_MASK_BF16 = 3 };
int b2_pack_block_bias(const void* mask, int32_t mask_dtype, int64_t stride_bh,
                       int64_t stride_t, int64_t stride_key, int32_t mask_bh,
                       int32_t tokens, float* bias, void* stream);
int b2_fixed_block_attention_masked(const b2_view* q, const b2_view* k,
                                    const b2_view* v, const b2_view* out,
                                    float scale, int32_t causal,
                                    const float* bias, int64_t bias_bh_stride,
                                    void* stream);

/* ---- Layout kernels. */
/* pisa_kernels.cu:247-272: [B,H,T,D] tiled views -> contiguous [BH,T,D]. */
int b2_pack_rows(const b2_view* src, void* dst, void* stream);
/* pisa_kernels.cu:275-293: contiguous [BH,T,D] -> view (e.g. raster). */
int b2_unpack_rows(const void* src, const b2_view* dst, void* stream);
/* pisa_kernels.cu:296-340: LSE-weighted merge, block-major -> dst view.
 * exact/approx: [BH,T,D] BF16, lses [BH,T] FP32, correction [BH,T,D] FP32. */
int b2_merge_epilogue(const void* exact, const float* exact_lse,
                      const void* approx, const float* approx_lse,
                      const float* correction, const b2_view* dst,
                      void* stream);
/* minimax_h3_gfx1151_attention.py:64-74: copy n views (n in 1..3) of equal
 * shape into one contiguous [n,B,H,T,D] allocation at dst. */
int b2_h3_pack(const b2_view* views, int32_t n, void* dst, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B200ATTN_H */
