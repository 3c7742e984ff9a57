// extern "C" entry points of libgdn_rssm_b200.so: argument validation (before
// any launch), TMA descriptor encoding and template dispatch.  The checks
// mirror the reference's host-side checks (csrc/ops.cpp:87-154,170-239 and
// kernels.py:700-928) plus the alignment rules of the sm_100a data paths.
#include <cstring>
#include <mutex>
#include <string>

#include "params.cuh"
#include "verify_launch.cuh"

namespace gdn_rssm {

static thread_local std::string t_error;
void set_error(const std::string &msg) { t_error = msg; }
const char *get_error() { return t_error.c_str(); }

bool host_dtype_is_float(int32_t d) { return d == GDN_RSSM_F32 || d == GDN_RSSM_BF16 || d == GDN_RSSM_F16; }
int host_dtype_size(int32_t d) {
  switch (d) {
    case GDN_RSSM_F32: return 4;
    case GDN_RSSM_BF16: return 2;
    case GDN_RSSM_F16: return 2;
    case GDN_RSSM_I32: return 4;
    case GDN_RSSM_I64: return 8;
  }
  return 0;
}

int launch_verify_bf16(VerifyLaunch &L);
int launch_verify_f16(VerifyLaunch &L);
int launch_verify_f32(VerifyLaunch &L);
int read_status_bf16(int32_t *out, cudaStream_t stream);
int read_status_f16(int32_t *out, cudaStream_t stream);
int read_status_f32(int32_t *out, cudaStream_t stream);
int read_status_fold(int32_t *out, cudaStream_t stream);
int launch_fold(const FoldParams &p, int dim, int32_t state_dtype, int32_t key_dtype, cudaStream_t stream);
int launch_commit_plan(const CommitPlanParams &p, cudaStream_t stream);
int launch_grouped_plan(const GroupedPlanParams &p, cudaStream_t stream);
int launch_publish_align(const PublishParams &p, cudaStream_t stream);
int launch_compact_conv(const ConvParams &p, int elem_size, cudaStream_t stream);

// ------------------------------------------------------------- TMA encode --- //
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  });
  return fn;
}

int encode_state_map(CUtensorMap *map, const void *base, int32_t state_dtype, int dim, int box_rows,
                     int64_t value_heads, int64_t blocks, int64_t state_bs, int64_t state_hs, int64_t state_vs) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("GDN RecoverSSM: cuTensorMapEncodeTiled is unavailable from the driver");
    return GDN_RSSM_ECUDA;
  }
  const int es = host_dtype_size(state_dtype);
  const cuuint64_t gdim[4] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(dim),
                              static_cast<cuuint64_t>(value_heads), static_cast<cuuint64_t>(blocks)};
  const cuuint64_t gstride[3] = {static_cast<cuuint64_t>(state_vs * es), static_cast<cuuint64_t>(state_hs * es),
                                 static_cast<cuuint64_t>(state_bs * es)};
  // one box = 128 bytes of K (one swizzle row) x box_rows rows
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(box_rows), 1, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUresult r = fn(map,
                        state_dtype == GDN_RSSM_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        4, const_cast<void *>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("GDN RecoverSSM: cuTensorMapEncodeTiled rejected the state pool layout (code " + std::to_string(r) +
              "); base and strides must be 16-byte aligned");
    return GDN_RSSM_ECUDA;
  }
  return GDN_RSSM_OK;
}

static bool index_dtype_ok(int32_t d) { return d == GDN_RSSM_I32 || d == GDN_RSSM_I64; }
static bool view_ok(const gdn_rssm_index_view &v) { return v.data != nullptr && index_dtype_ok(v.dtype) && v.length >= 0; }
static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace gdn_rssm

using namespace gdn_rssm;

extern "C" {

int64_t gdn_rssm_abi_version(void) { return GDN_RSSM_ABI_VERSION; }

const char *gdn_rssm_last_error(void) { return get_error(); }

int gdn_rssm_device_status(int32_t *status, void *stream) {
  GDN_REQUIRE(status != nullptr, "status output pointer is null");
  auto s = static_cast<cudaStream_t>(stream);
  int32_t a = 0, b = 0, c = 0, d = 0;
  int rc;
  if ((rc = read_status_bf16(&a, s)) != GDN_RSSM_OK) return rc;
  if ((rc = read_status_f16(&b, s)) != GDN_RSSM_OK) return rc;
  if ((rc = read_status_f32(&c, s)) != GDN_RSSM_OK) return rc;
  if ((rc = read_status_fold(&d, s)) != GDN_RSSM_OK) return rc;
  *status = a | b | c | d;
  return GDN_RSSM_OK;
}

static int verify_impl(const void *q, const void *k, const void *v, const void *g, const void *beta,
                       const void *state, float *correction, void *key, float *decay, void *out, const void *qsl,
                       const void *indices, const int64_t *config, int64_t config_len, float scale,
                       int32_t activation_dtype, int32_t state_dtype, int32_t gate_dtype, int32_t beta_dtype,
                       int32_t key_dtype, int32_t qsl_dtype, int32_t index_dtype, int32_t key_dim, int32_t value_dim,
                       uint32_t flags, const float *A_log, const float *dt_bias, float softplus_beta,
                       float softplus_threshold, void *stream) {
  const bool gated = A_log != nullptr;
  GDN_REQUIRE(config != nullptr && config_len == GDN_RSSM_VERIFY_FIELDS, "verify config must have 28 fields");
  int64_t f[GDN_RSSM_VERIFY_FIELDS];
  std::memcpy(f, config, sizeof(f));
  VerifyLaunch L{};
  VerifyParams &p = L.p;
  p.rows = f[0];
  p.tokens = f[1];
  p.heads = f[2];
  p.value_heads = f[3];
  p.query_len = f[4];
  p.blocks = f[5];
  p.record_rows = f[6];
  p.null_block = f[7];
  p.q_ts = f[8];
  p.k_ts = f[9];
  p.v_ts = f[10];
  p.g_ts = f[11];
  p.beta_ts = f[12];
  L.state_bs = f[13];
  L.state_hs = f[14];
  L.state_vs = f[15];
  p.corr_rs = f[16];
  p.corr_hs = f[17];
  p.corr_ts = f[18];
  p.key_rs = f[19];
  p.key_hs = f[20];
  p.key_ts = f[21];
  p.decay_rs = f[22];
  p.decay_hs = f[23];
  p.decay_ts = f[24];
  p.out_ts = f[25];
  p.qsl_stride = f[26];
  p.index_stride = f[27];

  const bool packed = (flags & GDN_RSSM_RECORD_PACKED) != 0;
  const bool normalize = (flags & GDN_RSSM_NORMALIZE_QK) != 0;
  GDN_REQUIRE((flags & ~(GDN_RSSM_RECORD_PACKED | GDN_RSSM_NORMALIZE_QK | GDN_RSSM_VERIFY_TEST_NO_TILE |
                          GDN_RSSM_VERIFY_CUDA_CORES)) == 0,
              "unknown verify flags");
  GDN_REQUIRE(p.null_block == 0, "the null block id must be 0 (page zero is reserved)");
  GDN_REQUIRE(key_dim == value_dim && (key_dim == 32 || key_dim == 64 || key_dim == 128),
              "K and V must be equal and one of 32, 64, 128");
  GDN_REQUIRE(activation_dtype == GDN_RSSM_F32 || activation_dtype == GDN_RSSM_BF16 || activation_dtype == GDN_RSSM_F16,
              "activations must be FP32, BF16 or FP16");
  GDN_REQUIRE(state_dtype == GDN_RSSM_F32 || (state_dtype == GDN_RSSM_BF16 && key_dim >= 64),
              "state must be FP32 (or BF16 with K >= 64)");
  GDN_REQUIRE(beta_dtype == GDN_RSSM_F32 || beta_dtype == activation_dtype, "beta must be FP32 or the activation dtype");
  GDN_REQUIRE(gate_dtype == GDN_RSSM_F32 || (gated && gate_dtype == activation_dtype),
              "the gate must be FP32 (or, raw, the activation dtype)");
  if (gated) {
    GDN_REQUIRE(dt_bias != nullptr && softplus_beta > 0.f, "gating needs A_log, dt_bias and softplus_beta > 0");
  }
  if (packed) {
    GDN_REQUIRE(key_dtype == GDN_RSSM_F32, "packed records must remain FP32");
  } else {
    GDN_REQUIRE(key_dtype == GDN_RSSM_F32 || (!normalize && key_dtype == activation_dtype),
                "low-precision key records require already-normalized input dtype");
  }
  GDN_REQUIRE(index_dtype_ok(qsl_dtype) && index_dtype_ok(index_dtype), "qsl / state indices must be int32 or int64");
  GDN_REQUIRE(p.rows >= 0 && p.tokens >= 0 && p.heads > 0 && p.value_heads >= p.heads && p.value_heads % p.heads == 0,
              "value heads must be a positive multiple of the q/k heads");
  GDN_REQUIRE(p.query_len >= 1 && p.query_len <= kMaxWindow, "spec_query_len must be in [1, 8]");
  GDN_REQUIRE(p.tokens <= p.rows * p.query_len, "speculative decode input exceeds its activation capacity");
  // the kernels keep row, token and page indices in 32 bits
  GDN_REQUIRE(p.rows < (int64_t{1} << 31) - 1 && p.tokens < (int64_t{1} << 31) - 16 && p.blocks < (int64_t{1} << 31),
              "rows, tokens and checkpoint blocks must stay below 2^31");
  GDN_REQUIRE(p.blocks > 0 && p.record_rows >= 1, "state pool and record rows must be non-empty");
  GDN_REQUIRE(p.rows * p.value_heads < (int64_t(1) << 31), "rows x value heads exceeds the launch grid");
  // the tensor-core walk packs a unit's key head above its 8-bit token mask
  GDN_REQUIRE(p.value_heads < (int64_t(1) << 23), "value heads must stay below 2^23");
  if (p.rows == 0 || p.tokens == 0) return GDN_RSSM_OK;
  GDN_REQUIRE(q && k && v && g && beta && state && correction && key && decay && out && qsl && indices,
              "verify tensor pointer is null");
  const int es = host_dtype_size(state_dtype);
  const int64_t epc = 16 / es;
  GDN_REQUIRE(aligned16(state) && L.state_vs % epc == 0 && L.state_hs % epc == 0 && L.state_bs % epc == 0 &&
                  L.state_vs >= key_dim,
              "state pool base and strides must be 16-byte aligned with contiguous K rows");

  p.q = q;
  p.k = k;
  p.v = v;
  p.g = g;
  p.beta = beta;
  p.A_log = A_log;
  p.dt_bias = dt_bias;
  p.softplus_beta = softplus_beta;
  p.softplus_threshold = softplus_threshold;
  p.gate_dtype = gate_dtype;
  p.corr = correction;
  p.key = key;
  p.decay = decay;
  p.out = out;
  p.qsl = qsl;
  p.indices = indices;
  p.scale = scale;
  p.beta_dtype = beta_dtype;
  p.key_dtype = key_dtype;
  p.qsl_dtype = qsl_dtype;
  p.index_dtype = index_dtype;
  p.flags = flags | (gated ? kGateInKernel : 0u);
  L.state = state;
  L.state_dtype = state_dtype;
  L.dim = key_dim;
  L.stream = static_cast<cudaStream_t>(stream);
  switch (activation_dtype) {
    case GDN_RSSM_BF16: return launch_verify_bf16(L);
    case GDN_RSSM_F16: return launch_verify_f16(L);
    default: return launch_verify_f32(L);
  }
}

int gdn_rssm_verify(const void *q, const void *k, const void *v, const float *g, const void *beta, const void *state,
                    float *correction, void *key, float *decay, void *out, const void *qsl, const void *indices,
                    const int64_t *config, int64_t config_len, float scale, int32_t activation_dtype,
                    int32_t state_dtype, int32_t beta_dtype, int32_t key_dtype, int32_t qsl_dtype,
                    int32_t index_dtype, int32_t key_dim, int32_t value_dim, uint32_t flags, void *stream) {
  return verify_impl(q, k, v, g, beta, state, correction, key, decay, out, qsl, indices, config, config_len, scale,
                     activation_dtype, state_dtype, GDN_RSSM_F32, beta_dtype, key_dtype, qsl_dtype, index_dtype,
                     key_dim, value_dim, flags, nullptr, nullptr, 0.f, 0.f, stream);
}

int gdn_rssm_verify_gated(const void *q, const void *k, const void *v, const void *a, const void *b, const float *A_log,
                          const float *dt_bias, const void *state, float *correction, void *key, float *decay,
                          void *out, const void *qsl, const void *indices, const int64_t *config, int64_t config_len,
                          float scale, float softplus_beta, float softplus_threshold, int32_t activation_dtype,
                          int32_t state_dtype, int32_t gate_dtype, int32_t b_dtype, int32_t key_dtype,
                          int32_t qsl_dtype, int32_t index_dtype, int32_t key_dim, int32_t value_dim, uint32_t flags,
                          void *stream) {
  GDN_REQUIRE(A_log != nullptr, "gdn_rssm_verify_gated needs A_log");
  return verify_impl(q, k, v, a, b, state, correction, key, decay, out, qsl, indices, config, config_len, scale,
                     activation_dtype, state_dtype, gate_dtype, b_dtype, key_dtype, qsl_dtype, index_dtype, key_dim,
                     value_dim, flags, A_log, dt_bias, softplus_beta, softplus_threshold, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Validation of the commit-side arguments, shared by the separate entry points
// and the fused ones: each fills its parameter block or returns the error.
// ---------------------------------------------------------------------------
namespace gdn_rssm {

// The fold's configuration and per-layer tables (everything but the plan).
static int prepare_fold(FoldParams &p, const int64_t *state_addrs, const int64_t *state_block_strides,
                        const int64_t *corr_addrs, const int64_t *corr_block_strides, const int64_t *key_addrs,
                        const int64_t *key_block_strides, const int64_t *decay_addrs,
                        const int64_t *decay_block_strides, const int32_t *layer_groups, const int64_t *config,
                        int64_t config_len, int32_t state_dtype, int32_t key_dtype, int32_t key_dim,
                        int32_t value_dim, uint32_t flags) {
  GDN_REQUIRE(config != nullptr && config_len == GDN_RSSM_FOLD_FIELDS, "fold config must have 17 fields");
  int64_t f[GDN_RSSM_FOLD_FIELDS];
  std::memcpy(f, config, sizeof(f));
  p = FoldParams{};
  p.rows = f[0];
  p.layers = f[1];
  p.heads = f[2];
  p.key_heads = f[3];
  p.query_len = f[4];
  p.blocks = f[5];
  p.record_rows = f[6];
  p.plan_capacity = f[7];
  p.null_block = f[8];
  p.state_hs = f[9];
  p.state_vs = f[10];
  p.corr_hs = f[11];
  p.corr_ts = f[12];
  p.key_hs = f[13];
  p.key_ts = f[14];
  p.decay_hs = f[15];
  p.decay_ts = f[16];
  const bool packed = (flags & GDN_RSSM_FOLD_PACKED) != 0;
  GDN_REQUIRE((flags & ~GDN_RSSM_FOLD_PACKED) == 0, "unknown fold flags");
  GDN_REQUIRE(p.null_block == 0, "the null block id must be 0 (page zero is reserved)");
  GDN_REQUIRE(key_dim == value_dim && (key_dim == 32 || key_dim == 64 || key_dim == 128),
              "K and V must be equal and one of 32, 64, 128");
  GDN_REQUIRE(state_dtype == GDN_RSSM_F32 || state_dtype == GDN_RSSM_BF16, "fold state must be FP32 or BF16");
  GDN_REQUIRE(packed ? key_dtype == GDN_RSSM_F32
                     : (key_dtype == GDN_RSSM_F32 || key_dtype == GDN_RSSM_BF16 || key_dtype == GDN_RSSM_F16),
              "record keys require FP16, BF16 or FP32 (packed: FP32)");
  GDN_REQUIRE(p.layers > 0 && p.rows >= 0 && p.plan_capacity > 0 && p.rows <= p.plan_capacity,
              "fold geometry: rows must fit the plan capacity");
  GDN_REQUIRE(p.heads > 0 && p.key_heads > 0 && p.heads % p.key_heads == 0, "fold head geometry");
  GDN_REQUIRE(p.query_len >= 1 && p.query_len <= kMaxWindow, "spec_query_len must be in [1, 8]");
  GDN_REQUIRE(p.layers * p.rows * p.heads < (int64_t(1) << 31), "fold launch grid too large");
  if (p.rows == 0) return GDN_RSSM_OK;
  GDN_REQUIRE(state_addrs && state_block_strides && corr_addrs && corr_block_strides && layer_groups,
              "fold table pointer is null");
  GDN_REQUIRE(packed || (key_addrs && key_block_strides && decay_addrs && decay_block_strides),
              "typed records need key and decay tables");
  const int64_t epc = 16 / host_dtype_size(state_dtype);
  GDN_REQUIRE(p.state_hs % epc == 0 && p.state_vs % epc == 0 && p.state_vs >= key_dim,
              "state head / row strides must be 16-byte aligned with contiguous K rows");
  p.state_addrs = state_addrs;
  p.state_bs = state_block_strides;
  p.corr_addrs = corr_addrs;
  p.corr_bs = corr_block_strides;
  p.key_addrs = key_addrs;
  p.key_bs = key_block_strides;
  p.decay_addrs = decay_addrs;
  p.decay_bs = decay_block_strides;
  p.layer_groups = layer_groups;
  p.flags = flags;
  return GDN_RSSM_OK;
}

static int prepare_commit_plan(CommitPlanParams &p, gdn_rssm_index_view num_accepted,
                               gdn_rssm_index_view request_indices, gdn_rssm_index_view state_indices,
                               gdn_rssm_index_view query_start_loc, gdn_rssm_table_view block_table,
                               gdn_rssm_index_view num_computed, int32_t *commit_lens, int32_t *final_indices,
                               int32_t *boundary_indices, int32_t *boundary_lengths, int32_t *align_valid,
                               int32_t *align_col, int64_t rows, int64_t spec_query_len, int64_t num_blocks,
                               int64_t block_size, int64_t null_block) {
  GDN_REQUIRE(null_block == 0, "the null block id must be 0 (page zero is reserved)");
  GDN_REQUIRE(rows >= 0 && spec_query_len >= 1 && spec_query_len <= kMaxWindow, "plan geometry");
  if (rows == 0) return GDN_RSSM_OK;
  GDN_REQUIRE(view_ok(num_accepted) && view_ok(state_indices) && view_ok(query_start_loc), "plan inputs must be int views");
  GDN_REQUIRE(state_indices.length >= rows && query_start_loc.length >= rows + 1, "plan inputs are shorter than rows");
  GDN_REQUIRE(request_indices.data == nullptr || (view_ok(request_indices) && request_indices.length >= rows),
              "request mapping is too short");
  GDN_REQUIRE(request_indices.data != nullptr || num_accepted.length >= rows, "accepted-token counts are too short");
  GDN_REQUIRE(commit_lens && final_indices && boundary_indices && boundary_lengths && align_valid && align_col,
              "plan output pointer is null");
  const bool align = block_table.data != nullptr;
  if (align) {
    GDN_REQUIRE(index_dtype_ok(block_table.dtype) && block_table.rows >= 0 && block_table.cols > 0,
                "block table must be two-dimensional with a positive width");
    GDN_REQUIRE(view_ok(num_computed), "align mode needs num_computed_tokens");
    GDN_REQUIRE(block_size >= spec_query_len, "align block size must cover one speculative window");
    // the per-context plan does its align arithmetic in 32 bits, as the reference does
    GDN_REQUIRE(block_size < (int64_t{1} << 31) && block_table.cols < (int64_t{1} << 31),
                "align block size and block table width must stay below 2^31");
  }
  p = CommitPlanParams{};
  p.accepted = num_accepted;
  p.request = request_indices;
  p.state = state_indices;
  p.qsl = query_start_loc;
  p.computed = num_computed;
  p.table = block_table;
  p.lens = commit_lens;
  p.finals = final_indices;
  p.boundaries = boundary_indices;
  p.boundary_lens = boundary_lengths;
  p.valid = align_valid;
  p.col = align_col;
  p.rows = rows;
  p.Q = spec_query_len;
  p.num_blocks = num_blocks;
  p.block_size = align ? block_size : 1;
  p.null_block = null_block;
  return GDN_RSSM_OK;
}

static int prepare_grouped_plan(GroupedPlanParams &p, gdn_rssm_index_view sampled, const gdn_rssm_plan_group *groups,
                                int32_t num_groups, int32_t *source, int32_t *length, int32_t *final_indices,
                                int32_t *boundary_indices, int32_t *boundary_lengths, int32_t *valid, int32_t *col,
                                gdn_rssm_index_view idx_mapping, gdn_rssm_out_view persistent_cols,
                                gdn_rssm_out_view persistent_accepted, int64_t rows, int64_t plan_capacity,
                                int64_t spec_query_len, int64_t null_block, int32_t align, int32_t publish) {
  GDN_REQUIRE(null_block == 0, "the null block id must be 0 (page zero is reserved)");
  GDN_REQUIRE(groups != nullptr && num_groups >= 1 && num_groups <= 3, "one recovery bucket supports one to three groups");
  GDN_REQUIRE(rows > 0 && rows <= plan_capacity, "grouped recovery rows out of range");
  GDN_REQUIRE(spec_query_len >= 1 && spec_query_len <= kMaxWindow, "spec_query_len must be in [1, 8]");
  GDN_REQUIRE(view_ok(sampled), "sampled counts must be an int view");
  GDN_REQUIRE(source && length && final_indices && boundary_indices && boundary_lengths && valid && col,
              "plan output pointer is null");
  p = GroupedPlanParams{};
  for (int i = 0; i < num_groups; ++i) {
    const gdn_rssm_plan_group &g = groups[i];
    GDN_REQUIRE(view_ok(g.state_indices) && g.state_indices.length >= rows, "group state indices are too short");
    GDN_REQUIRE(view_ok(g.query_start_loc) && g.query_start_loc.length >= rows + 1,
                "grouped recovery offsets are shorter than their rows");
    GDN_REQUIRE(view_ok(g.request_indices) && g.request_indices.length >= rows,
                "grouped recovery requires an explicit native row mapping");
    if (align) {
      GDN_REQUIRE(g.block_table.data != nullptr && index_dtype_ok(g.block_table.dtype) && g.block_table.cols > 0,
                  "align block table has no columns");
      GDN_REQUIRE(view_ok(g.num_computed), "align mode needs num_computed_tokens");
      GDN_REQUIRE(g.block_size >= spec_query_len, "align blocks must cover the speculative window");
    }
    p.groups[i] = g;
    if (!align) p.groups[i].block_size = 1;
  }
  if (align && publish) {
    GDN_REQUIRE(view_ok(idx_mapping), "publication needs idx_mapping");
    GDN_REQUIRE(persistent_cols.data && persistent_accepted.data && index_dtype_ok(persistent_cols.dtype) &&
                    index_dtype_ok(persistent_accepted.dtype),
                "publication needs persistent column / acceptance outputs");
    GDN_REQUIRE(!(persistent_accepted.data == sampled.data), "sampled counts must not alias persistent acceptance output");
  }
  p.sampled = sampled;
  p.num_groups = num_groups;
  p.source = source;
  p.length = length;
  p.finals = final_indices;
  p.boundaries = boundary_indices;
  p.boundary_lens = boundary_lengths;
  p.valid = valid;
  p.col = col;
  p.idx_mapping = idx_mapping;
  p.cols_out = persistent_cols;
  p.accepted_out = persistent_accepted;
  p.rows = rows;
  p.capacity = plan_capacity;
  p.Q = spec_query_len;
  p.null_block = null_block;
  p.align = align;
  p.publish = align && publish;
  return GDN_RSSM_OK;
}

// The conv compaction's tables and geometry (not its plan arrays).
static int prepare_conv(ConvParams &p, const int64_t *conv_addrs, const int64_t *conv_block_strides,
                        const int64_t *conv_dim_strides, const int64_t *conv_token_strides, int64_t rows,
                        int64_t layers, int64_t plan_capacity, int64_t conv_dim, int64_t history, int64_t window,
                        int64_t num_blocks, int64_t null_block, int32_t elem_dtype, int32_t align) {
  GDN_REQUIRE(null_block == 0, "the null block id must be 0 (page zero is reserved)");
  GDN_REQUIRE(rows >= 0 && layers > 0 && plan_capacity > 0 && rows <= plan_capacity, "conv geometry");
  GDN_REQUIRE(conv_dim > 0 && history > 0 && window >= history, "conv state is shorter than its window");
  GDN_REQUIRE(history <= 8, "conv history longer than 8 tokens");
  GDN_REQUIRE(conv_dim <= int64_t{65535} * 64, "conv state has too many channels");
  GDN_REQUIRE(window <= 64, "conv state window longer than 64 tokens");
  GDN_REQUIRE(layers * rows < (int64_t(1) << 31), "conv launch grid too large");
  const int es = host_dtype_size(elem_dtype);
  GDN_REQUIRE(host_dtype_is_float(elem_dtype) && (es == 2 || es == 4), "conv state must be FP32, BF16 or FP16");
  if (rows == 0) return GDN_RSSM_OK;
  GDN_REQUIRE(conv_addrs && conv_block_strides && conv_dim_strides && conv_token_strides, "conv table pointer is null");
  p = ConvParams{};
  p.addrs = conv_addrs;
  p.block_strides = conv_block_strides;
  p.dim_strides = conv_dim_strides;
  p.token_strides = conv_token_strides;
  p.rows = rows;
  p.layers = layers;
  p.capacity = plan_capacity;
  p.conv_dim = conv_dim;
  p.history = history;
  p.window = window;
  p.num_blocks = num_blocks;
  p.null_block = null_block;
  p.align = align;
  p.elem_size = es;
  return GDN_RSSM_OK;
}

// The plan arrays a separate fold / conv compaction reads.
static int plan_arrays_ok(const gdn_rssm_index_view &source, const int32_t *lengths, const int32_t *final_indices,
                          const int32_t *boundary_indices, const int32_t *boundary_lengths, int64_t plan_len) {
  GDN_REQUIRE(lengths && final_indices && boundary_indices && boundary_lengths && plan_len > 0,
              "plan array pointer is null");
  GDN_REQUIRE(view_ok(source), "source indices must be an int32/int64 view");
  return GDN_RSSM_OK;
}

#define GDN_TRY(call)              \
  do {                             \
    const int _rc = (call);        \
    if (_rc != GDN_RSSM_OK) return _rc; \
  } while (0)

}  // namespace gdn_rssm

extern "C" {

int gdn_rssm_fold(const int64_t *state_addrs, const int64_t *state_block_strides, const int64_t *corr_addrs,
                  const int64_t *corr_block_strides, const int64_t *key_addrs, const int64_t *key_block_strides,
                  const int64_t *decay_addrs, const int64_t *decay_block_strides, const int32_t *layer_groups,
                  gdn_rssm_index_view source, const int32_t *lengths, const int32_t *final_indices,
                  const int32_t *boundary_indices, const int32_t *boundary_lengths, int64_t plan_len,
                  const int64_t *config, int64_t config_len, int32_t state_dtype, int32_t key_dtype, int32_t key_dim,
                  int32_t value_dim, uint32_t flags, void *stream) {
  FoldParams p{};
  GDN_TRY(prepare_fold(p, state_addrs, state_block_strides, corr_addrs, corr_block_strides, key_addrs,
                       key_block_strides, decay_addrs, decay_block_strides, layer_groups, config, config_len,
                       state_dtype, key_dtype, key_dim, value_dim, flags));
  if (p.rows == 0) return GDN_RSSM_OK;
  GDN_TRY(plan_arrays_ok(source, lengths, final_indices, boundary_indices, boundary_lengths, plan_len));
  p.source = source;
  p.lengths = lengths;
  p.finals = final_indices;
  p.boundaries = boundary_indices;
  p.boundary_lens = boundary_lengths;
  p.plan_len = plan_len;
  const bool packed = (flags & GDN_RSSM_FOLD_PACKED) != 0;
  return launch_fold(p, key_dim, state_dtype, packed ? GDN_RSSM_F32 : key_dtype, static_cast<cudaStream_t>(stream));
}

int gdn_rssm_commit_plan(gdn_rssm_index_view num_accepted, gdn_rssm_index_view request_indices,
                         gdn_rssm_index_view state_indices, gdn_rssm_index_view query_start_loc,
                         gdn_rssm_table_view block_table, gdn_rssm_index_view num_computed, int32_t *commit_lens,
                         int32_t *final_indices, int32_t *boundary_indices, int32_t *boundary_lengths,
                         int32_t *align_valid, int32_t *align_col, int64_t rows, int64_t spec_query_len,
                         int64_t num_blocks, int64_t block_size, int64_t null_block, void *stream) {
  CommitPlanParams p{};
  GDN_TRY(prepare_commit_plan(p, num_accepted, request_indices, state_indices, query_start_loc, block_table,
                              num_computed, commit_lens, final_indices, boundary_indices, boundary_lengths,
                              align_valid, align_col, rows, spec_query_len, num_blocks, block_size, null_block));
  if (rows == 0) return GDN_RSSM_OK;
  return launch_commit_plan(p, static_cast<cudaStream_t>(stream));
}

int gdn_rssm_grouped_plan(gdn_rssm_index_view sampled, const gdn_rssm_plan_group *groups, int32_t num_groups,
                          int32_t *source, int32_t *length, int32_t *final_indices, int32_t *boundary_indices,
                          int32_t *boundary_lengths, int32_t *valid, int32_t *col, gdn_rssm_index_view idx_mapping,
                          gdn_rssm_out_view persistent_cols, gdn_rssm_out_view persistent_accepted, int64_t rows,
                          int64_t plan_capacity, int64_t spec_query_len, int64_t null_block, int32_t align,
                          int32_t publish, void *stream) {
  GroupedPlanParams p{};
  GDN_TRY(prepare_grouped_plan(p, sampled, groups, num_groups, source, length, final_indices, boundary_indices,
                               boundary_lengths, valid, col, idx_mapping, persistent_cols, persistent_accepted, rows,
                               plan_capacity, spec_query_len, null_block, align, publish));
  return launch_grouped_plan(p, static_cast<cudaStream_t>(stream));
}

int gdn_rssm_publish_align(const int64_t *descriptors, int32_t num_buckets, gdn_rssm_index_view request_indices,
                           gdn_rssm_index_view idx_mapping, gdn_rssm_out_view persistent_cols,
                           gdn_rssm_out_view persistent_accepted, int64_t rows, void *stream) {
  GDN_REQUIRE(descriptors != nullptr && num_buckets >= 1, "publication needs at least one bucket descriptor");
  GDN_REQUIRE(rows >= 0, "rows must be non-negative");
  if (rows == 0) return GDN_RSSM_OK;
  GDN_REQUIRE(view_ok(request_indices) && request_indices.length >= rows && view_ok(idx_mapping),
              "publication needs request indices and idx_mapping");
  GDN_REQUIRE(persistent_cols.data && persistent_accepted.data && index_dtype_ok(persistent_cols.dtype) &&
                  index_dtype_ok(persistent_accepted.dtype),
              "publication needs persistent column / acceptance outputs");
  PublishParams p{};
  p.descriptors = descriptors;
  p.num_buckets = num_buckets;
  p.request = request_indices;
  p.idx_mapping = idx_mapping;
  p.cols_out = persistent_cols;
  p.accepted_out = persistent_accepted;
  p.rows = rows;
  return launch_publish_align(p, static_cast<cudaStream_t>(stream));
}

int gdn_rssm_compact_conv(const int64_t *conv_addrs, const int64_t *conv_block_strides,
                          const int64_t *conv_dim_strides, const int64_t *conv_token_strides,
                          const int32_t *layer_groups, gdn_rssm_index_view source, const int32_t *lengths,
                          const int32_t *final_indices, const int32_t *boundary_indices,
                          const int32_t *boundary_lengths, int64_t plan_len, int64_t rows, int64_t layers,
                          int64_t plan_capacity, int64_t conv_dim, int64_t history, int64_t window,
                          int64_t num_blocks, int64_t null_block, int32_t elem_dtype, int32_t align, void *stream) {
  ConvParams p{};
  GDN_TRY(prepare_conv(p, conv_addrs, conv_block_strides, conv_dim_strides, conv_token_strides, rows, layers,
                       plan_capacity, conv_dim, history, window, num_blocks, null_block, elem_dtype, align));
  if (rows == 0) return GDN_RSSM_OK;
  GDN_REQUIRE(layer_groups != nullptr, "conv table pointer is null");
  GDN_TRY(plan_arrays_ok(source, lengths, final_indices, boundary_indices, boundary_lengths, plan_len));
  p.layer_groups = layer_groups;
  p.source = source;
  p.lengths = lengths;
  p.finals = final_indices;
  p.boundaries = boundary_indices;
  p.boundary_lens = boundary_lengths;
  p.plan_len = plan_len;
  return launch_compact_conv(p, p.elem_size, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
