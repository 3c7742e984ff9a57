/*
 * gdn_recoverssm_b200.h -- C ABI of the B200 (sm_100a) RecoverSSM verify +
 * grouped-commit path.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * launches on the given CUDA stream (a cudaStream_t passed as void*, NULL =
 * legacy default stream), never synchronises and never allocates device
 * memory.  Arguments are validated on the host before any launch; a rejected
 * call returns GDN_RSSM_EINVAL and leaves a message for gdn_rssm_last_error().
 * Strides are in ELEMENTS of the tensor they describe, as in the reference's
 * tiling ABI (plugin/gdn_recoverssm_ascend/csrc/common.h:5-6).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   gdn_rssm_abi_version   <- torch op gdn_recoverssm_ac::abi_version
 *                             (csrc/ops.cpp:244, kAbiVersion csrc/common.h:64)
 *   gdn_rssm_verify        <- torch op gdn_recoverssm_ac::verify
 *                             (csrc/ops.cpp:87-154,245) and the Triton launch
 *                             of _gdn_recoverssm_verify_kernel
 *                             (kernels.py:491-697, host wrapper :700-928)
 *   gdn_rssm_fold          <- torch op gdn_recoverssm_ac::fold
 *                             (csrc/ops.cpp:170-239,246), Triton
 *                             _grouped_commit_gdn_state_kernel
 *                             (grouped_commit.py:325-480) and
 *                             _commit_gdn_state_kernel (kernels.py:1172-1324)
 *   gdn_rssm_commit_plan   <- Triton _prepare_commit_plan_kernel
 *                             (kernels.py:936-1072)
 *   gdn_rssm_grouped_plan  <- Triton _grouped_plan_kernel
 *                             (grouped_commit.py:31-222)
 *   gdn_rssm_publish_align <- Triton _publish_grouped_align_kernel
 *                             (grouped_commit.py:531-560)
 *   gdn_rssm_compact_conv  <- Triton _grouped_compact_conv_state_kernel
 *                             (grouped_commit.py:225-322) and
 *                             _compact_conv_state_kernel (kernels.py:1075-1169)
 *   gdn_rssm_verify_gated  <- the gating op in front of verify, fused as in
 *                             the upstream verify
 *                             (docs/reference/recoverssm_gdn_upstream.py:39-175)
 */
#ifndef GDN_RECOVERSSM_B200_H
#define GDN_RECOVERSSM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_RSSM_ABI_VERSION 1

/* Only the entry points below are exported from the shared library. */
#if defined(__GNUC__)
#define GDN_RSSM_API __attribute__((visibility("default")))
#else
#define GDN_RSSM_API
#endif

/* Element type codes. */
enum {
  GDN_RSSM_F32 = 0,
  GDN_RSSM_BF16 = 1,
  GDN_RSSM_F16 = 2,
  GDN_RSSM_I32 = 3,
  GDN_RSSM_I64 = 4
};

/* Status codes. */
enum {
  GDN_RSSM_OK = 0,
  GDN_RSSM_EINVAL = 1,      /* argument rejected before launch          */
  GDN_RSSM_ECUDA = 2,       /* CUDA runtime / driver call failed        */
  GDN_RSSM_EUNSUPPORTED = 3 /* shape or dtype outside the built kernels */
};

/* gdn_rssm_verify flags. */
#define GDN_RSSM_RECORD_PACKED 1u /* correction/key/decay point into one   \
                                     packed fp32 [R,HV,Q,V+K+1] record      \
                                     (key = corr + V, decay = corr + V + K; \
                                     the key is per value head)            */
#define GDN_RSSM_NORMALIZE_QK 2u  /* q,k <- x * rsqrt(sum(x^2) + 1e-6)    */
/* Test hook for failure detection: the tensor-core verify kernel (K = V = 128,
 * fp32 pool) starts no state-tile copy, so its bounded wait for the tile runs
 * out after 1 s; the kernel then records status 1 (copy timeout) in the word
 * gdn_rssm_device_status() reads, releases its tensor memory and exits, and
 * the context stays usable.  Ignored by the other kernels. */
#define GDN_RSSM_VERIFY_TEST_NO_TILE 0x10000u
/* Accuracy comparisons: run the CUDA-core verify kernel (fp32 FMAs over the
 * whole state tile) where the tensor-core kernel would run (K = V = 128, fp32
 * pool).  Same results within fp32 rounding, slower. */
#define GDN_RSSM_VERIFY_CUDA_CORES 0x20000u

/* gdn_rssm_fold flags. */
#define GDN_RSSM_FOLD_PACKED 1u /* records are packed fp32 [R,HV,Q,V+K+1] */

/* Number of int64 fields of the verify / fold configuration arrays.  The
 * field ORDER is the reference's tiling ABI (csrc/common.h:8-54):
 *   verify: rows, tokens, heads, value_heads, query_len, blocks, record_rows,
 *     null_block, q_token_stride, k_token_stride, v_token_stride,
 *     g_token_stride, beta_token_stride, state_block_stride,
 *     state_head_stride, state_v_stride, corr_row_stride, corr_head_stride,
 *     corr_token_stride, key_row_stride, key_head_stride, key_token_stride,
 *     decay_row_stride, decay_head_stride, decay_token_stride,
 *     out_token_stride, qsl_stride, index_stride
 *   fold: rows, layers, heads, key_heads, query_len, blocks, record_rows,
 *     plan_capacity, null_block, state_head_stride, state_v_stride,
 *     corr_head_stride, corr_token_stride, key_head_stride,
 *     key_token_stride, decay_head_stride, decay_token_stride          */
#define GDN_RSSM_VERIFY_FIELDS 28
#define GDN_RSSM_FOLD_FIELDS 17

/* A read-only 1-D integer array on the device: element i is
 * data[i * stride] of type dtype (GDN_RSSM_I32 or GDN_RSSM_I64); valid
 * indices are 0 <= i < length.  data == NULL means "absent".            */
typedef struct {
  const void *data;
  int64_t stride;
  int64_t length;
  int32_t dtype;
} gdn_rssm_index_view;

/* A writable 1-D integer array on the device. */
typedef struct {
  void *data;
  int64_t stride;
  int64_t length;
  int32_t dtype;
} gdn_rssm_out_view;

/* A read-only 2-D integer table (block table) on the device. */
typedef struct {
  const void *data;
  int64_t rows;
  int64_t cols;
  int64_t row_stride;
  int64_t col_stride;
  int32_t dtype;
} gdn_rssm_table_view;

/* One KV-cache group of the grouped commit plan. */
typedef struct {
  gdn_rssm_index_view state_indices;   /* [rows] source pages            */
  gdn_rssm_index_view query_start_loc; /* [rows + 1]                     */
  gdn_rssm_index_view request_indices; /* [rows] row -> request          */
  gdn_rssm_index_view num_computed;    /* [requests], align mode only    */
  gdn_rssm_table_view block_table;     /* [requests, W], align mode only */
  int64_t num_blocks;                  /* pool size of this group        */
  int64_t block_size;                  /* tokens per cache block (align) */
} gdn_rssm_plan_group;

/* ABI version of this library (GDN_RSSM_ABI_VERSION). */
GDN_RSSM_API int64_t gdn_rssm_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
GDN_RSSM_API const char *gdn_rssm_last_error(void);

/* Read and clear the device-side status word of the current device (set when
 * an in-kernel wait ran out; 0 = no error).  Synchronises `stream`. */
GDN_RSSM_API int gdn_rssm_device_status(int32_t *status, void *stream);

/* Speculative verify.  q, k [1,T,H,K] (head-contiguous); v, out [1,T,HV,V];
 * g [T,HV] fp32 log-decay; beta [T,HV] (fp32 or activation dtype); state
 * [blocks,HV,V,K] read-only checkpoint pool; records as described by the
 * config strides (typed: correction [R,HV,Q,V] fp32, key [R,H,Q,K], decay
 * [R,HV,Q] fp32; packed: see GDN_RSSM_RECORD_PACKED); qsl [rows+1] and
 * indices [rows] of dtype qsl_dtype / index_dtype (I32 or I64).
 * Supported: K == V in {32, 64, 128} (bf16 state: {64, 128}), 1 <= Q <= 8,
 * activation bf16/fp16/fp32, state fp32/bf16, null_block == 0. */
GDN_RSSM_API int gdn_rssm_verify(const void *q, const void *k, const void *v, const float *g,
                    const void *beta, const void *state, float *correction,
                    void *key, float *decay, void *out, const void *qsl,
                    const void *indices, const int64_t *config,
                    int64_t config_len, float scale, int32_t activation_dtype,
                    int32_t state_dtype, int32_t beta_dtype, int32_t key_dtype,
                    int32_t qsl_dtype, int32_t index_dtype, int32_t key_dim,
                    int32_t value_dim, uint32_t flags, void *stream);

/* Verify with the gates computed in the kernel prologue.  Replaces the
 * separate gating op in front of verify: the reference plugin's upstream
 * verify (docs/reference/recoverssm_gdn_upstream.py:39-175, host wrapper
 * :178-330) fuses it the same way; its own torch op has no counterpart.
 * Same as gdn_rssm_verify except that the raw gate inputs replace g and beta:
 * a [T,HV] (dtype gate_dtype, token stride = config field g_token_stride),
 * b [T,HV] (dtype b_dtype, stride = beta_token_stride), A_log [HV] and
 * dt_bias [HV] fp32, and per token and value head
 *   g    = -exp(A_log) * softplus(a + dt_bias),
 *   softplus(x) = log(1 + exp(sb * x)) / sb  if sb * x <= threshold, else x,
 *   beta = sigmoid(b),
 * with sb = softplus_beta, threshold = softplus_threshold (the upstream
 * defaults are 1 and 20).  The decay record is exp(g) as multiplied. */
GDN_RSSM_API int gdn_rssm_verify_gated(const void *q, const void *k, const void *v, const void *a,
                    const void *b, const float *A_log, const float *dt_bias,
                    const void *state, float *correction, void *key, float *decay,
                    void *out, const void *qsl, const void *indices,
                    const int64_t *config, int64_t config_len, float scale,
                    float softplus_beta, float softplus_threshold,
                    int32_t activation_dtype, int32_t state_dtype, int32_t gate_dtype,
                    int32_t b_dtype, int32_t key_dtype, int32_t qsl_dtype,
                    int32_t index_dtype, int32_t key_dim, int32_t value_dim,
                    uint32_t flags, void *stream);

/* Multi-layer accepted-prefix fold.  Per layer l: state_addrs[l] is the
 * layer's state pool base, state_block_strides[l] its page stride (elements);
 * the corr/key/decay tables give each layer's record bases and ROW strides.
 * Head/v/token strides come from the config and are shared by all layers.
 * Plan arrays (int32, plan_len entries): plan row = layer_groups[l] *
 * plan_capacity + row; `source` may be any index view (the per-context
 * commit passes the raw state indices).  Only `state` pages are written.
 * The kernel bounds every page index by config field `blocks` and every
 * record row by `record_rows`; the library cannot see the sizes behind the
 * address tables, so the caller guarantees that each layer's pool holds the
 * pages its plan rows name (at least `blocks` pages, or, in a grouped
 * commit, its own group's pool size, which the grouped plan enforces) and
 * that each layer's records hold `record_rows` rows. */
GDN_RSSM_API int gdn_rssm_fold(const int64_t *state_addrs, const int64_t *state_block_strides,
                  const int64_t *corr_addrs, const int64_t *corr_block_strides,
                  const int64_t *key_addrs, const int64_t *key_block_strides,
                  const int64_t *decay_addrs,
                  const int64_t *decay_block_strides,
                  const int32_t *layer_groups, gdn_rssm_index_view source,
                  const int32_t *lengths, const int32_t *final_indices,
                  const int32_t *boundary_indices,
                  const int32_t *boundary_lengths, int64_t plan_len,
                  const int64_t *config, int64_t config_len,
                  int32_t state_dtype, int32_t key_dtype, int32_t key_dim,
                  int32_t value_dim, uint32_t flags, void *stream);

/* Per-context commit plan (none mode when block_table.data == NULL).
 * Outputs are int32 [rows]. */
GDN_RSSM_API int gdn_rssm_commit_plan(gdn_rssm_index_view num_accepted,
                         gdn_rssm_index_view request_indices,
                         gdn_rssm_index_view state_indices,
                         gdn_rssm_index_view query_start_loc,
                         gdn_rssm_table_view block_table,
                         gdn_rssm_index_view num_computed, int32_t *commit_lens,
                         int32_t *final_indices, int32_t *boundary_indices,
                         int32_t *boundary_lengths, int32_t *align_valid,
                         int32_t *align_col, int64_t rows,
                         int64_t spec_query_len, int64_t num_blocks,
                         int64_t block_size, int64_t null_block, void *stream);

/* Grouped commit plan over 1..3 groups.  Outputs are int32
 * [num_groups * plan_capacity]; when align && publish, rows whose groups are
 * all valid and agree on column and request write persistent_cols[slot] =
 * col and persistent_accepted[slot] = 1, slot = idx_mapping[request]. */
GDN_RSSM_API int gdn_rssm_grouped_plan(gdn_rssm_index_view sampled,
                          const gdn_rssm_plan_group *groups, int32_t num_groups,
                          int32_t *source, int32_t *length, int32_t *final_indices,
                          int32_t *boundary_indices, int32_t *boundary_lengths,
                          int32_t *valid, int32_t *col,
                          gdn_rssm_index_view idx_mapping,
                          gdn_rssm_out_view persistent_cols,
                          gdn_rssm_out_view persistent_accepted, int64_t rows,
                          int64_t plan_capacity, int64_t spec_query_len,
                          int64_t null_block, int32_t align, int32_t publish,
                          void *stream);

/* Cross-bucket align publication.  descriptors: device int64 [buckets * 4] =
 * (valid ptr, col ptr, capacity, group count) per bucket. */
GDN_RSSM_API int gdn_rssm_publish_align(const int64_t *descriptors, int32_t num_buckets,
                           gdn_rssm_index_view request_indices,
                           gdn_rssm_index_view idx_mapping,
                           gdn_rssm_out_view persistent_cols,
                           gdn_rssm_out_view persistent_accepted, int64_t rows,
                           void *stream);

/* Conv-history compaction for every layer: final[:, h] = src[:, n - 1 + h]
 * and, in align mode, boundary[:, h] = src[:, blen - 1 + h], h < history.
 * Per-layer tables give base address, page / dim / token strides (elements);
 * `window` is the conv state length (history + Q - 1): rows whose lengths
 * would read past it are skipped.  elem_dtype selects the element size
 * (bit-exact copy). */
GDN_RSSM_API int gdn_rssm_compact_conv(const int64_t *conv_addrs,
                          const int64_t *conv_block_strides,
                          const int64_t *conv_dim_strides,
                          const int64_t *conv_token_strides,
                          const int32_t *layer_groups, gdn_rssm_index_view source,
                          const int32_t *lengths, const int32_t *final_indices,
                          const int32_t *boundary_indices,
                          const int32_t *boundary_lengths, int64_t plan_len,
                          int64_t rows, int64_t layers, int64_t plan_capacity,
                          int64_t conv_dim, int64_t history, int64_t window,
                          int64_t num_blocks, int64_t null_block,
                          int32_t elem_dtype, int32_t align, void *stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* GDN_RECOVERSSM_B200_H */
