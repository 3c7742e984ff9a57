// Kernel parameter blocks (passed by value) shared by the launchers in
// fold.cu and the argument checks in capi.cu.
#pragma once

#include "common.cuh"

namespace gdn_rssm {

struct FoldParams {
  const int64_t *state_addrs, *state_bs;
  const int64_t *corr_addrs, *corr_bs;
  const int64_t *key_addrs, *key_bs;
  const int64_t *decay_addrs, *decay_bs;
  const int32_t *layer_groups;
  gdn_rssm_index_view source;
  const int32_t *lengths, *finals, *boundaries, *boundary_lens;
  int64_t plan_len;
  int64_t rows, layers, heads, key_heads, query_len, blocks, record_rows, plan_capacity, null_block;
  int64_t state_hs, state_vs, corr_hs, corr_ts, key_hs, key_ts, decay_hs, decay_ts;
  uint32_t flags;
  int32_t *status;  // device status word of the fold translation unit
};

struct CommitPlanParams {
  gdn_rssm_index_view accepted, request, state, qsl, computed;
  gdn_rssm_table_view table;
  int32_t *lens, *finals, *boundaries, *boundary_lens, *valid, *col;
  int64_t rows, Q, num_blocks, block_size, null_block;
};

struct GroupedPlanParams {
  gdn_rssm_index_view sampled;
  gdn_rssm_plan_group groups[3];
  int32_t num_groups;
  int32_t *source, *length, *finals, *boundaries, *boundary_lens, *valid, *col;
  gdn_rssm_index_view idx_mapping;
  gdn_rssm_out_view cols_out, accepted_out;
  int64_t rows, capacity, Q, null_block;
  int32_t align, publish;
};

struct PublishParams {
  const int64_t *descriptors;
  int32_t num_buckets;
  gdn_rssm_index_view request, idx_mapping;
  gdn_rssm_out_view cols_out, accepted_out;
  int64_t rows;
};

struct ConvParams {
  const int64_t *addrs, *block_strides, *dim_strides, *token_strides;
  const int32_t *layer_groups;
  gdn_rssm_index_view source;
  const int32_t *lengths, *finals, *boundaries, *boundary_lens;
  int64_t plan_len, rows, layers, capacity, conv_dim, history, window, num_blocks, null_block;
  int32_t align;
  int32_t chunk;      // channels per CTA (blockIdx.y)
  int32_t vec;        // 1: stage whole chunks through shared memory with 16-byte copies
  int32_t elem_size;  // bytes per conv element (2 or 4)
  int32_t *status;    // device status word of the fold translation unit
};

}  // namespace gdn_rssm
