// Torch custom ops over the C ABI (libgdn_rssm_b200.so).
//
// Registers the reference's native schemas unchanged under the same namespace
// -- gdn_recoverssm_ac::{abi_version, verify, fold} (csrc/ops.cpp:243-257) --
// with CUDA and Meta implementations, plus the ops the Triton half of the
// reference path provided: verify_ext (packed records / in-kernel L2),
// fold_ext (packed records, any source index view), commit_plan,
// grouped_plan, publish_align and compact_conv.  Every op validates its
// tensors (TORCH_CHECK -> RuntimeError before launch), launches on the current
// CUDA stream, allocates nothing and never synchronises.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <vector>

#include "gdn_recoverssm_b200.h"

namespace {

using at::Tensor;

int32_t code_of(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return GDN_RSSM_F32;
    case at::kBFloat16: return GDN_RSSM_BF16;
    case at::kHalf: return GDN_RSSM_F16;
    case at::kInt: return GDN_RSSM_I32;
    case at::kLong: return GDN_RSSM_I64;
    default: TORCH_CHECK(false, "GDN RecoverSSM: unsupported dtype ", t);
  }
}

void check_rc(int rc) { TORCH_CHECK(rc == GDN_RSSM_OK, gdn_rssm_last_error()); }

void same_cuda(const Tensor &t, const Tensor &ref, const char *name) {
  TORCH_CHECK(t.defined() && t.is_cuda() && t.device() == ref.device(), "GDN RecoverSSM: ", name,
              " must be a CUDA tensor on the same device");
}

gdn_rssm_index_view index_view(const Tensor &t, const Tensor &ref, const char *name) {
  same_cuda(t, ref, name);
  TORCH_CHECK(t.dim() == 1 && (t.scalar_type() == at::kInt || t.scalar_type() == at::kLong),
              "GDN RecoverSSM: ", name, " must be a 1-D int32/int64 tensor");
  return gdn_rssm_index_view{t.data_ptr(), t.stride(0), t.size(0), code_of(t.scalar_type())};
}

gdn_rssm_index_view opt_index_view(const std::optional<Tensor> &t, const Tensor &ref, const char *name) {
  if (!t.has_value() || !t->defined()) return gdn_rssm_index_view{nullptr, 0, 0, GDN_RSSM_I32};
  return index_view(*t, ref, name);
}

gdn_rssm_out_view out_view(const Tensor &t, const Tensor &ref, const char *name) {
  same_cuda(t, ref, name);
  TORCH_CHECK(t.dim() == 1 && (t.scalar_type() == at::kInt || t.scalar_type() == at::kLong),
              "GDN RecoverSSM: ", name, " must be a 1-D int32/int64 tensor");
  return gdn_rssm_out_view{t.data_ptr(), t.stride(0), t.size(0), code_of(t.scalar_type())};
}

gdn_rssm_table_view table_view(const std::optional<Tensor> &t, const Tensor &ref, const char *name) {
  if (!t.has_value() || !t->defined()) return gdn_rssm_table_view{nullptr, 0, 0, 0, 0, GDN_RSSM_I32};
  same_cuda(*t, ref, name);
  TORCH_CHECK(t->dim() == 2 && (t->scalar_type() == at::kInt || t->scalar_type() == at::kLong),
              "GDN RecoverSSM: block table must be a 2-D int32/int64 tensor");
  return gdn_rssm_table_view{t->data_ptr(), t->size(0), t->size(1), t->stride(0), t->stride(1),
                             code_of(t->scalar_type())};
}

void check_plan_out(const Tensor &t, const Tensor &ref, int64_t n, const char *name) {
  same_cuda(t, ref, name);
  TORCH_CHECK(t.scalar_type() == at::kInt && t.dim() == 1 && t.is_contiguous() && t.numel() >= n,
              "GDN RecoverSSM: plan tensor ", name, " must be contiguous int32 with at least ", n, " entries");
}

void check_table(const Tensor &t, const Tensor &ref, int64_t layers, at::ScalarType dtype, const char *name) {
  same_cuda(t, ref, name);
  TORCH_CHECK(t.scalar_type() == dtype && t.dim() == 1 && t.is_contiguous() && t.numel() == layers,
              "GDN RecoverSSM: invalid layer table ", name);
}

// verify with explicit flags: packed records (correction == key == decay ==
// the packed fp32 record tensor) and/or in-kernel q/k normalisation.
// Gate inputs of verify_gated_ext: g / beta slots carry the raw a / b.
struct GateArgs {
  const Tensor &A_log;
  const Tensor &dt_bias;
  double softplus_beta, softplus_threshold;
};

void verify_common(const Tensor &q, const Tensor &k, const Tensor &v, const Tensor &g, const Tensor &beta,
                   const Tensor &state, const Tensor &correction, const Tensor &key, const Tensor &decay,
                   const Tensor &out, const Tensor &qsl, const Tensor &indices, at::IntArrayRef config, double scale,
                   int64_t flags, const GateArgs *gate) {
  TORCH_CHECK(config.size() == GDN_RSSM_VERIFY_FIELDS, "GDN RecoverSSM: verify config must have 28 fields");
  TORCH_CHECK(q.is_cuda(), "GDN RecoverSSM: verify requires CUDA tensors");
  for (auto *t : {&k, &v, &g, &beta, &state, &correction, &key, &decay, &out, &qsl, &indices}) same_cuda(*t, q, "input");
  TORCH_CHECK(q.dim() == 4 && k.sizes() == q.sizes() && v.dim() == 4 && out.sizes() == v.sizes() && q.size(0) == 1 &&
                  q.size(1) == v.size(1),
              "GDN RecoverSSM: activation shape");
  TORCH_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type() &&
                  out.scalar_type() == q.scalar_type(),
              "GDN RecoverSSM: q/k/v/out dtypes differ");
  TORCH_CHECK(q.stride(3) == 1 && q.stride(2) == q.size(3) && k.stride(3) == 1 && k.stride(2) == k.size(3) &&
                  v.stride(3) == 1 && v.stride(2) == v.size(3) && out.stride(3) == 1 && out.stride(2) == out.size(3),
              "GDN RecoverSSM: q/k/v/out heads must be contiguous");
  TORCH_CHECK((g.scalar_type() == at::kFloat || (gate && g.scalar_type() == q.scalar_type())) &&
                  correction.scalar_type() == at::kFloat && decay.scalar_type() == at::kFloat,
              "GDN RecoverSSM: FP32 gate/correction/decay required");
  if (gate) {
    for (const Tensor *t : {&gate->A_log, &gate->dt_bias}) {
      same_cuda(*t, q, "A_log / dt_bias");
      TORCH_CHECK(t->dim() == 1 && t->size(0) == v.size(2) && t->stride(0) == 1 && t->scalar_type() == at::kFloat,
                  "GDN RecoverSSM: A_log and dt_bias must be contiguous FP32 [value heads]");
    }
  }
  TORCH_CHECK(g.dim() == 2 && beta.dim() == 2 && g.stride(1) == 1 && beta.stride(1) == 1,
              "GDN RecoverSSM: gate and beta must be [tokens, value heads] with contiguous heads");
  TORCH_CHECK(state.dim() == 4 && state.stride(3) == 1, "GDN RecoverSSM: state must be [blocks, HV, V, K]");
  TORCH_CHECK(config[1] == q.size(1) && config[2] == q.size(2) && config[3] == v.size(2) &&
                  config[5] == state.size(0) && state.size(1) == v.size(2) && state.size(2) == v.size(3) &&
                  state.size(3) == q.size(3),
              "GDN RecoverSSM: verify config does not match the tensors");
  TORCH_CHECK(qsl.dim() == 1 && indices.dim() == 1 && qsl.numel() >= config[0] + 1 && indices.numel() >= config[0],
              "GDN RecoverSSM: row capacity");
  TORCH_CHECK(config[8] == q.stride(1) && config[9] == k.stride(1) && config[10] == v.stride(1) &&
                  config[11] == g.stride(0) && config[12] == beta.stride(0) && config[13] == state.stride(0) &&
                  config[14] == state.stride(1) && config[15] == state.stride(2) && config[25] == out.stride(1) &&
                  config[26] == qsl.stride(0) && config[27] == indices.stride(0),
              "GDN RecoverSSM: verify config does not match tensor strides");
  const bool packed = (flags & GDN_RSSM_RECORD_PACKED) != 0;
  const int64_t V = v.size(3), K = q.size(3);
  float *corr_ptr = correction.data_ptr<float>();
  void *key_ptr = key.data_ptr();
  float *decay_ptr = decay.data_ptr<float>();
  if (packed) {
    TORCH_CHECK(correction.dim() == 4 && correction.size(3) == V + K + 1 && correction.stride(3) == 1 &&
                    correction.size(0) == config[6],
                "GDN RecoverSSM: packed record geometry");
    key_ptr = corr_ptr + V;
    decay_ptr = corr_ptr + V + K;
  } else {
    TORCH_CHECK(correction.dim() == 4 && key.dim() == 4 && decay.dim() == 3 && correction.size(0) == config[6] &&
                    key.size(0) == config[6] && decay.size(0) == config[6] && correction.stride(3) == 1 &&
                    key.stride(3) == 1 && decay.stride(2) == 1,
                "GDN RecoverSSM: record geometry");
  }
  const c10::cuda::CUDAGuard guard(q.device());
  const auto stream = at::cuda::getCurrentCUDAStream(q.get_device()).stream();
  std::vector<int64_t> cfg(config.begin(), config.end());
  const int32_t key_code = packed ? GDN_RSSM_F32 : code_of(key.scalar_type());
  if (gate == nullptr) {
    check_rc(gdn_rssm_verify(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(), beta.data_ptr(),
                             state.data_ptr(), corr_ptr, key_ptr, decay_ptr, out.data_ptr(), qsl.data_ptr(),
                             indices.data_ptr(), cfg.data(), static_cast<int64_t>(cfg.size()),
                             static_cast<float>(scale), code_of(q.scalar_type()), code_of(state.scalar_type()),
                             code_of(beta.scalar_type()), key_code, code_of(qsl.scalar_type()),
                             code_of(indices.scalar_type()), static_cast<int32_t>(K), static_cast<int32_t>(V),
                             static_cast<uint32_t>(flags), stream));
  } else {
    check_rc(gdn_rssm_verify_gated(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), gate->A_log.data_ptr<float>(),
        gate->dt_bias.data_ptr<float>(), state.data_ptr(), corr_ptr, key_ptr, decay_ptr, out.data_ptr(),
        qsl.data_ptr(), indices.data_ptr(), cfg.data(), static_cast<int64_t>(cfg.size()), static_cast<float>(scale),
        static_cast<float>(gate->softplus_beta), static_cast<float>(gate->softplus_threshold),
        code_of(q.scalar_type()), code_of(state.scalar_type()), code_of(g.scalar_type()), code_of(beta.scalar_type()),
        key_code, code_of(qsl.scalar_type()), code_of(indices.scalar_type()), static_cast<int32_t>(K),
        static_cast<int32_t>(V), static_cast<uint32_t>(flags), stream));
  }
}

void verify_ext(const Tensor &q, const Tensor &k, const Tensor &v, const Tensor &g, const Tensor &beta,
                const Tensor &state, const Tensor &correction, const Tensor &key, const Tensor &decay,
                const Tensor &out, const Tensor &qsl, const Tensor &indices, at::IntArrayRef config, double scale,
                int64_t flags) {
  verify_common(q, k, v, g, beta, state, correction, key, decay, out, qsl, indices, config, scale, flags, nullptr);
}

// verify with the gates computed in the kernel from the raw inputs a, b and
// the per-head A_log, dt_bias (the upstream fused form).
void verify_gated_ext(const Tensor &q, const Tensor &k, const Tensor &v, const Tensor &a, const Tensor &b,
                      const Tensor &A_log, const Tensor &dt_bias, const Tensor &state, const Tensor &correction,
                      const Tensor &key, const Tensor &decay, const Tensor &out, const Tensor &qsl,
                      const Tensor &indices, at::IntArrayRef config, double scale, double softplus_beta,
                      double softplus_threshold, int64_t flags) {
  const GateArgs gate{A_log, dt_bias, softplus_beta, softplus_threshold};
  verify_common(q, k, v, a, b, state, correction, key, decay, out, qsl, indices, config, scale, flags, &gate);
}

// The reference schema: typed records, q/k already normalised.
void verify(const Tensor &q, const Tensor &k, const Tensor &v, const Tensor &g, const Tensor &beta,
            const Tensor &state, const Tensor &correction, const Tensor &key, const Tensor &decay, const Tensor &out,
            const Tensor &qsl, const Tensor &indices, at::IntArrayRef config, double scale) {
  verify_ext(q, k, v, g, beta, state, correction, key, decay, out, qsl, indices, config, scale, 0);
}

// Checks of the fold's tensors and configuration (everything but the plan
// arrays), shared by fold_ext and the fused commits.
struct FoldTables {
  const int64_t *state_addrs, *state_bs, *corr_addrs, *corr_bs, *key_addrs, *key_bs, *decay_addrs, *decay_bs;
  const int32_t *layer_groups;
  int32_t state_code, key_code, K, V;
};

FoldTables check_fold_tensors(const Tensor &state, const Tensor &correction, const Tensor &key, const Tensor &decay,
                              const Tensor &state_addrs, const Tensor &state_block_strides, const Tensor &corr_addrs,
                              const Tensor &corr_block_strides, const Tensor &key_addrs,
                              const Tensor &key_block_strides, const Tensor &decay_addrs,
                              const Tensor &decay_block_strides, const Tensor &layer_groups, at::IntArrayRef config,
                              int64_t flags) {
  TORCH_CHECK(config.size() == GDN_RSSM_FOLD_FIELDS, "GDN RecoverSSM: fold config must have 17 fields");
  TORCH_CHECK(state.is_cuda(), "GDN RecoverSSM: fold requires CUDA tensors");
  const int64_t layers = config[1];
  const bool packed = (flags & GDN_RSSM_FOLD_PACKED) != 0;
  for (auto *t : {&correction, &key, &decay}) same_cuda(*t, state, "record");
  check_table(state_addrs, state, layers, at::kLong, "state_addrs");
  check_table(state_block_strides, state, layers, at::kLong, "state_block_strides");
  check_table(corr_addrs, state, layers, at::kLong, "corr_addrs");
  check_table(corr_block_strides, state, layers, at::kLong, "corr_block_strides");
  if (!packed) {
    check_table(key_addrs, state, layers, at::kLong, "key_addrs");
    check_table(key_block_strides, state, layers, at::kLong, "key_block_strides");
    check_table(decay_addrs, state, layers, at::kLong, "decay_addrs");
    check_table(decay_block_strides, state, layers, at::kLong, "decay_block_strides");
  }
  check_table(layer_groups, state, layers, at::kInt, "layer_groups");
  TORCH_CHECK(state.dim() == 4 && state.stride(3) == 1 && state.size(1) == config[2] && config[9] == state.stride(1) &&
                  config[10] == state.stride(2),
              "GDN RecoverSSM: fold config does not match the state geometry");
  TORCH_CHECK(correction.scalar_type() == at::kFloat && correction.dim() == 4 && correction.stride(3) == 1 &&
                  config[11] == correction.stride(1) && config[12] == correction.stride(2),
              "GDN RecoverSSM: fold config does not match the correction records");
  // the kernel bounds pages by config[5] and record rows by config[6]: both
  // must lie inside the tensors this op was given (the address tables of the
  // other layers are trusted to describe pools and records at least as large)
  TORCH_CHECK(config[5] > 0 && config[5] <= state.size(0),
              "GDN RecoverSSM: fold page bound exceeds the state pool (", config[5], " > ", state.size(0), ")");
  TORCH_CHECK(config[6] > 0 && config[6] <= correction.size(0) && config[0] <= config[7],
              "GDN RecoverSSM: fold record rows exceed the correction records or rows exceed the plan capacity");
  const int64_t V = state.size(2), K = state.size(3);
  if (packed) {
    TORCH_CHECK(correction.size(3) == V + K + 1, "GDN RecoverSSM: packed record width must be V + K + 1");
  } else {
    TORCH_CHECK(decay.scalar_type() == at::kFloat && key.dim() == 4 && decay.dim() == 3 && key.stride(3) == 1 &&
                    decay.stride(2) == 1 && config[13] == key.stride(1) && config[14] == key.stride(2) &&
                    config[15] == decay.stride(1) && config[16] == decay.stride(2) && key.size(1) == config[3],
                "GDN RecoverSSM: fold config does not match the typed records");
    TORCH_CHECK(config[6] <= key.size(0) && config[6] <= decay.size(0),
                "GDN RecoverSSM: fold record rows exceed the key / decay records");
  }
  auto ptr64 = [](const Tensor &t) { return t.defined() && t.numel() ? t.data_ptr<int64_t>() : nullptr; };
  FoldTables f{};
  f.state_addrs = state_addrs.data_ptr<int64_t>();
  f.state_bs = state_block_strides.data_ptr<int64_t>();
  f.corr_addrs = corr_addrs.data_ptr<int64_t>();
  f.corr_bs = corr_block_strides.data_ptr<int64_t>();
  f.key_addrs = packed ? nullptr : ptr64(key_addrs);
  f.key_bs = packed ? nullptr : ptr64(key_block_strides);
  f.decay_addrs = packed ? nullptr : ptr64(decay_addrs);
  f.decay_bs = packed ? nullptr : ptr64(decay_block_strides);
  f.layer_groups = layer_groups.data_ptr<int32_t>();
  f.state_code = code_of(state.scalar_type());
  f.key_code = packed ? GDN_RSSM_F32 : code_of(key.scalar_type());
  f.K = static_cast<int32_t>(K);
  f.V = static_cast<int32_t>(V);
  return f;
}

void fold_ext(const Tensor &state, const Tensor &correction, const Tensor &key, const Tensor &decay,
              const Tensor &state_addrs, const Tensor &state_block_strides, const Tensor &corr_addrs,
              const Tensor &corr_block_strides, const Tensor &key_addrs, const Tensor &key_block_strides,
              const Tensor &decay_addrs, const Tensor &decay_block_strides, const Tensor &layer_groups,
              const Tensor &source, const Tensor &lengths, const Tensor &final_indices,
              const Tensor &boundary_indices, const Tensor &boundary_lengths, at::IntArrayRef config,
              int64_t flags) {
  const FoldTables f = check_fold_tensors(state, correction, key, decay, state_addrs, state_block_strides, corr_addrs,
                                          corr_block_strides, key_addrs, key_block_strides, decay_addrs,
                                          decay_block_strides, layer_groups, config, flags);
  const int64_t plan = lengths.numel();
  TORCH_CHECK(config[7] > 0 && plan % config[7] == 0 && plan / config[7] > 0, "GDN RecoverSSM: invalid plan tensor");
  for (auto *t : {&lengths, &final_indices, &boundary_indices, &boundary_lengths}) check_plan_out(*t, state, plan, "plan");
  auto src = index_view(source, state, "source");
  const c10::cuda::CUDAGuard guard(state.device());
  const auto stream = at::cuda::getCurrentCUDAStream(state.get_device()).stream();
  std::vector<int64_t> cfg(config.begin(), config.end());
  check_rc(gdn_rssm_fold(f.state_addrs, f.state_bs, f.corr_addrs, f.corr_bs, f.key_addrs, f.key_bs, f.decay_addrs,
                         f.decay_bs, f.layer_groups, src, lengths.data_ptr<int32_t>(), final_indices.data_ptr<int32_t>(),
                         boundary_indices.data_ptr<int32_t>(), boundary_lengths.data_ptr<int32_t>(), plan, cfg.data(),
                         static_cast<int64_t>(cfg.size()), f.state_code, f.key_code, f.K, f.V,
                         static_cast<uint32_t>(flags), stream));
}

void fold(const Tensor &state, const Tensor &correction, const Tensor &key, const Tensor &decay,
          const Tensor &state_addrs, const Tensor &state_block_strides, const Tensor &corr_addrs,
          const Tensor &corr_block_strides, const Tensor &key_addrs, const Tensor &key_block_strides,
          const Tensor &decay_addrs, const Tensor &decay_block_strides, const Tensor &layer_groups,
          const Tensor &source, const Tensor &lengths, const Tensor &final_indices, const Tensor &boundary_indices,
          const Tensor &boundary_lengths, at::IntArrayRef config) {
  fold_ext(state, correction, key, decay, state_addrs, state_block_strides, corr_addrs, corr_block_strides, key_addrs,
           key_block_strides, decay_addrs, decay_block_strides, layer_groups, source, lengths, final_indices,
           boundary_indices, boundary_lengths, config, 0);
}

void commit_plan(const Tensor &num_accepted, const std::optional<Tensor> &request_indices,
                 const Tensor &state_indices, const Tensor &qsl, const std::optional<Tensor> &block_table,
                 const std::optional<Tensor> &num_computed, const Tensor &commit_lens, const Tensor &final_indices,
                 const Tensor &boundary_indices, const Tensor &boundary_lengths, const Tensor &align_valid,
                 const Tensor &align_col, int64_t spec_query_len, int64_t num_blocks, int64_t block_size) {
  const Tensor &ref = state_indices;
  TORCH_CHECK(ref.is_cuda(), "GDN RecoverSSM: commit plan requires CUDA tensors");
  const int64_t rows = state_indices.size(0);
  for (auto *t : {&commit_lens, &final_indices, &boundary_indices, &boundary_lengths, &align_valid, &align_col})
    check_plan_out(*t, ref, rows, "plan output");
  const c10::cuda::CUDAGuard guard(ref.device());
  const auto stream = at::cuda::getCurrentCUDAStream(ref.get_device()).stream();
  check_rc(gdn_rssm_commit_plan(index_view(num_accepted, ref, "num_accepted"),
                                opt_index_view(request_indices, ref, "request_indices"),
                                index_view(state_indices, ref, "state_indices"), index_view(qsl, ref, "query_start_loc"),
                                table_view(block_table, ref, "block_table"),
                                opt_index_view(num_computed, ref, "num_computed_tokens"),
                                commit_lens.data_ptr<int32_t>(), final_indices.data_ptr<int32_t>(),
                                boundary_indices.data_ptr<int32_t>(), boundary_lengths.data_ptr<int32_t>(),
                                align_valid.data_ptr<int32_t>(), align_col.data_ptr<int32_t>(), rows, spec_query_len,
                                num_blocks, block_size, 0, stream));
}

void grouped_plan(const Tensor &sampled, at::TensorList state_indices, at::TensorList qsl,
                  at::TensorList request_indices, const c10::List<std::optional<Tensor>> &block_tables,
                  const c10::List<std::optional<Tensor>> &num_computed, at::IntArrayRef num_blocks,
                  at::IntArrayRef block_sizes, const Tensor &source, const Tensor &length, const Tensor &final_indices,
                  const Tensor &boundary_indices, const Tensor &boundary_lengths, const Tensor &valid,
                  const Tensor &col, const std::optional<Tensor> &idx_mapping,
                  const std::optional<Tensor> &persistent_cols, const std::optional<Tensor> &persistent_accepted,
                  int64_t rows, int64_t plan_capacity, int64_t spec_query_len, bool align, bool publish) {
  const int64_t groups = static_cast<int64_t>(state_indices.size());
  TORCH_CHECK(groups >= 1 && groups <= 3, "GDN RecoverSSM: one recovery bucket supports one to three groups");
  TORCH_CHECK(qsl.size() == state_indices.size() && request_indices.size() == state_indices.size() &&
                  static_cast<int64_t>(block_tables.size()) == groups &&
                  static_cast<int64_t>(num_computed.size()) == groups &&
                  static_cast<int64_t>(num_blocks.size()) == groups && static_cast<int64_t>(block_sizes.size()) == groups,
              "GDN RecoverSSM: per-group argument lists differ in length");
  const Tensor &ref = sampled;
  TORCH_CHECK(ref.is_cuda(), "GDN RecoverSSM: grouped plan requires CUDA tensors");
  for (auto *t : {&source, &length, &final_indices, &boundary_indices, &boundary_lengths, &valid, &col})
    check_plan_out(*t, ref, groups * plan_capacity, "plan output");
  gdn_rssm_plan_group g[3];
  for (int64_t i = 0; i < groups; ++i) {
    g[i].state_indices = index_view(state_indices[i], ref, "state_indices");
    g[i].query_start_loc = index_view(qsl[i], ref, "query_start_loc");
    g[i].request_indices = index_view(request_indices[i], ref, "request_indices");
    g[i].num_computed = opt_index_view(num_computed.get(i), ref, "num_computed_tokens");
    g[i].block_table = table_view(block_tables.get(i), ref, "block_table");
    g[i].num_blocks = num_blocks[i];
    g[i].block_size = block_sizes[i];
  }
  gdn_rssm_out_view cols{nullptr, 0, 0, GDN_RSSM_I32}, acc{nullptr, 0, 0, GDN_RSSM_I32};
  if (persistent_cols.has_value() && persistent_cols->defined()) cols = out_view(*persistent_cols, ref, "persistent_cols");
  if (persistent_accepted.has_value() && persistent_accepted->defined())
    acc = out_view(*persistent_accepted, ref, "persistent_accepted");
  const c10::cuda::CUDAGuard guard(ref.device());
  const auto stream = at::cuda::getCurrentCUDAStream(ref.get_device()).stream();
  check_rc(gdn_rssm_grouped_plan(index_view(sampled, ref, "sampled"), g, static_cast<int32_t>(groups),
                                 source.data_ptr<int32_t>(), length.data_ptr<int32_t>(),
                                 final_indices.data_ptr<int32_t>(), boundary_indices.data_ptr<int32_t>(),
                                 boundary_lengths.data_ptr<int32_t>(), valid.data_ptr<int32_t>(),
                                 col.data_ptr<int32_t>(), opt_index_view(idx_mapping, ref, "idx_mapping"), cols, acc,
                                 rows, plan_capacity, spec_query_len, 0, align ? 1 : 0, publish ? 1 : 0, stream));
}

void publish_align(const Tensor &descriptors, const Tensor &request_indices, const Tensor &idx_mapping,
                   const Tensor &persistent_cols, const Tensor &persistent_accepted, int64_t rows) {
  const Tensor &ref = descriptors;
  TORCH_CHECK(ref.is_cuda() && descriptors.scalar_type() == at::kLong && descriptors.dim() == 1 &&
                  descriptors.is_contiguous() && descriptors.numel() % 4 == 0 && descriptors.numel() > 0,
              "GDN RecoverSSM: publication descriptors must be int64 [buckets * 4]");
  const c10::cuda::CUDAGuard guard(ref.device());
  const auto stream = at::cuda::getCurrentCUDAStream(ref.get_device()).stream();
  check_rc(gdn_rssm_publish_align(descriptors.data_ptr<int64_t>(), static_cast<int32_t>(descriptors.numel() / 4),
                                  index_view(request_indices, ref, "request_indices"),
                                  index_view(idx_mapping, ref, "idx_mapping"),
                                  out_view(persistent_cols, ref, "persistent_cols"),
                                  out_view(persistent_accepted, ref, "persistent_accepted"), rows, stream));
}

void compact_conv(const Tensor &conv_ref, const Tensor &conv_addrs, const Tensor &block_strides,
                  const Tensor &dim_strides, const Tensor &token_strides, const Tensor &layer_groups,
                  const Tensor &source, const Tensor &lengths, const Tensor &final_indices,
                  const Tensor &boundary_indices, const Tensor &boundary_lengths, int64_t rows, int64_t plan_capacity,
                  int64_t conv_dim, int64_t history, int64_t window, int64_t num_blocks, bool align) {
  const Tensor &ref = conv_ref;
  TORCH_CHECK(ref.is_cuda(), "GDN RecoverSSM: conv compaction requires CUDA tensors");
  const int64_t layers = conv_addrs.numel();
  check_table(conv_addrs, ref, layers, at::kLong, "conv_addrs");
  check_table(block_strides, ref, layers, at::kLong, "conv_block_strides");
  check_table(dim_strides, ref, layers, at::kLong, "conv_dim_strides");
  check_table(token_strides, ref, layers, at::kLong, "conv_token_strides");
  check_table(layer_groups, ref, layers, at::kInt, "layer_groups");
  const int64_t plan = lengths.numel();
  for (auto *t : {&lengths, &final_indices, &boundary_indices, &boundary_lengths}) check_plan_out(*t, ref, plan, "plan");
  auto src = index_view(source, ref, "source");
  const c10::cuda::CUDAGuard guard(ref.device());
  const auto stream = at::cuda::getCurrentCUDAStream(ref.get_device()).stream();
  check_rc(gdn_rssm_compact_conv(conv_addrs.data_ptr<int64_t>(), block_strides.data_ptr<int64_t>(),
                                 dim_strides.data_ptr<int64_t>(), token_strides.data_ptr<int64_t>(),
                                 layer_groups.data_ptr<int32_t>(), src, lengths.data_ptr<int32_t>(),
                                 final_indices.data_ptr<int32_t>(), boundary_indices.data_ptr<int32_t>(),
                                 boundary_lengths.data_ptr<int32_t>(), plan, rows, layers, plan_capacity, conv_dim,
                                 history, window, num_blocks, 0, code_of(conv_ref.scalar_type()), align ? 1 : 0,
                                 stream));
}

int64_t device_status() {
  int32_t status = 0;
  const auto stream = at::cuda::getCurrentCUDAStream().stream();
  check_rc(gdn_rssm_device_status(&status, stream));
  return status;
}

}  // namespace

TORCH_LIBRARY(gdn_recoverssm_ac, m) {
  m.def("abi_version() -> int", []() -> int64_t { return gdn_rssm_abi_version(); });
  m.def(
      "verify(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor state, Tensor(a!) correction, "
      "Tensor(b!) key, Tensor(c!) decay, Tensor(d!) out, Tensor qsl, Tensor indices, int[] config, float scale) -> ()");
  m.def(
      "fold(Tensor(a!) state, Tensor correction, Tensor key, Tensor decay, Tensor state_addrs, "
      "Tensor state_block_strides, Tensor corr_addrs, Tensor corr_block_strides, Tensor key_addrs, "
      "Tensor key_block_strides, Tensor decay_addrs, Tensor decay_block_strides, Tensor layer_groups, "
      "Tensor source, Tensor lengths, Tensor final_indices, Tensor boundary_indices, Tensor boundary_lengths, "
      "int[] config) -> ()");
  m.def(
      "verify_ext(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor state, Tensor(a!) correction, "
      "Tensor(b!) key, Tensor(c!) decay, Tensor(d!) out, Tensor qsl, Tensor indices, int[] config, float scale, "
      "int flags) -> ()");
  m.def(
      "verify_gated_ext(Tensor q, Tensor k, Tensor v, Tensor a, Tensor b, Tensor A_log, Tensor dt_bias, "
      "Tensor state, Tensor(a!) correction, Tensor(b!) key, Tensor(c!) decay, Tensor(d!) out, Tensor qsl, "
      "Tensor indices, int[] config, float scale, float softplus_beta, float softplus_threshold, int flags) -> ()");
  m.def(
      "fold_ext(Tensor(a!) state, Tensor correction, Tensor key, Tensor decay, Tensor state_addrs, "
      "Tensor state_block_strides, Tensor corr_addrs, Tensor corr_block_strides, Tensor key_addrs, "
      "Tensor key_block_strides, Tensor decay_addrs, Tensor decay_block_strides, Tensor layer_groups, "
      "Tensor source, Tensor lengths, Tensor final_indices, Tensor boundary_indices, Tensor boundary_lengths, "
      "int[] config, int flags) -> ()");
  m.def(
      "commit_plan(Tensor num_accepted, Tensor? request_indices, Tensor state_indices, Tensor qsl, "
      "Tensor? block_table, Tensor? num_computed, Tensor(a!) commit_lens, Tensor(b!) final_indices, "
      "Tensor(c!) boundary_indices, Tensor(d!) boundary_lengths, Tensor(e!) align_valid, Tensor(f!) align_col, "
      "int spec_query_len, int num_blocks, int block_size) -> ()");
  m.def(
      "grouped_plan(Tensor sampled, Tensor[] state_indices, Tensor[] qsl, Tensor[] request_indices, "
      "Tensor?[] block_tables, Tensor?[] num_computed, int[] num_blocks, int[] block_sizes, Tensor(a!) source, "
      "Tensor(b!) length, Tensor(c!) final_indices, Tensor(d!) boundary_indices, Tensor(e!) boundary_lengths, "
      "Tensor(f!) valid, Tensor(g!) col, Tensor? idx_mapping, Tensor(h!)? persistent_cols, "
      "Tensor(i!)? persistent_accepted, int rows, int plan_capacity, int spec_query_len, bool align, "
      "bool publish) -> ()");
  m.def(
      "publish_align(Tensor descriptors, Tensor request_indices, Tensor idx_mapping, Tensor(a!) persistent_cols, "
      "Tensor(b!) persistent_accepted, int rows) -> ()");
  m.def(
      "compact_conv(Tensor(a!) conv_ref, Tensor conv_addrs, Tensor block_strides, Tensor dim_strides, "
      "Tensor token_strides, Tensor layer_groups, Tensor source, Tensor lengths, Tensor final_indices, "
      "Tensor boundary_indices, Tensor boundary_lengths, int rows, int plan_capacity, int conv_dim, int history, "
      "int window, int num_blocks, bool align) -> ()");
  m.def("device_status() -> int", &device_status);
}

TORCH_LIBRARY_IMPL(gdn_recoverssm_ac, CUDA, m) {
  m.impl("verify", TORCH_FN(verify));
  m.impl("fold", TORCH_FN(fold));
  m.impl("verify_ext", TORCH_FN(verify_ext));
  m.impl("verify_gated_ext", TORCH_FN(verify_gated_ext));
  m.impl("fold_ext", TORCH_FN(fold_ext));
  m.impl("commit_plan", TORCH_FN(commit_plan));
  m.impl("grouped_plan", TORCH_FN(grouped_plan));
  m.impl("publish_align", TORCH_FN(publish_align));
  m.impl("compact_conv", TORCH_FN(compact_conv));
}

// Meta: shape-only tracing; every op mutates caller-owned buffers in place.
TORCH_LIBRARY_IMPL(gdn_recoverssm_ac, Meta, m) {
  m.impl("verify", [](const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                      const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                      at::IntArrayRef, double) {});
  m.impl("verify_ext", [](const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                          const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                          const Tensor &, const Tensor &, at::IntArrayRef, double, int64_t) {});
  m.impl("verify_gated_ext", [](const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                                const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                                const Tensor &, const Tensor &, const Tensor &, const Tensor &, at::IntArrayRef,
                                double, double, double, int64_t) {});
  m.impl("fold", [](const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                    const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                    const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                    at::IntArrayRef) {});
  m.impl("fold_ext", [](const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                        const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                        const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &,
                        const Tensor &, at::IntArrayRef, int64_t) {});
}
