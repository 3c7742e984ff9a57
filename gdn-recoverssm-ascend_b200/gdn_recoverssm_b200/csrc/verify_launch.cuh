// Host launcher for the verify kernel, instantiated once per activation dtype
// (verify_bf16.cu, verify_f16.cu, verify_f32.cu) so the template variants
// compile in parallel.  Each instantiating translation unit owns one device
// status word.
#pragma once

#include <algorithm>
#include <type_traits>

#include "verify.cuh"
#include "verify_tc.cuh"

namespace gdn_rssm {

// Everything the launcher needs besides the kernel parameters.
struct VerifyLaunch {
  VerifyParams p;
  const void *state;
  int64_t state_bs, state_hs, state_vs;  // element strides of the pool
  int32_t state_dtype;
  int dim;
  cudaStream_t stream;
};

// Encodes the 4-D tiled tensor map of the state pool (defined in capi.cu).
// Box: 128 bytes of K x box_rows rows.
int encode_state_map(CUtensorMap *map, const void *base, int32_t state_dtype, int dim, int box_rows,
                     int64_t value_heads, int64_t blocks, int64_t state_bs, int64_t state_hs, int64_t state_vs);

// K = V = 128 with an fp32 pool runs the tensor-core kernel (verify_tc.cuh);
// other shapes the CUDA-core kernel (verify.cuh).
#ifndef GDN_RSSM_VERIFY_TENSOR_CORES
#define GDN_RSSM_VERIFY_TENSOR_CORES 1
#endif

template <int DIM, typename St>
constexpr bool verify_uses_tensor_cores() {
  return GDN_RSSM_VERIFY_TENSOR_CORES && DIM == 128 && std::is_same<St, float>::value;
}

// TC: the tensor-core kernel (verify_tc.cuh), else the CUDA-core kernel.
template <int DIM, int QT, typename Act, typename St, bool TC>
int launch_verify_kernel(VerifyLaunch &L) {
  // tensor-core kernel: whole-height boxes (4 copies per tile); CUDA-core
  // kernel: 32-row quarters, each on its own mbarrier
  CUtensorMap map;
  int rc = encode_state_map(&map, L.state, L.state_dtype, DIM, TC ? DIM : 32, L.p.value_heads, L.p.blocks,
                            L.state_bs, L.state_hs, L.state_vs);
  if (rc != GDN_RSSM_OK) return rc;
  // the tensor-core kernel has separate instantiations for the fused gating
  // prologue (so the plain form keeps its register budget) and for exact
  // operands: bf16 / fp16 q, k used as given are exact tf32 values
  const int gated = (L.p.flags & kGateInKernel) ? 1 : 0;
  constexpr bool low_precision = !std::is_same<Act, float>::value;
  // at Q = 8 the exact form stages q / k / v rows with 16-byte cp.async: it
  // needs 16-byte aligned rows (else the split form runs, same results)
  auto rows16 = [&]() {
    const int64_t es = static_cast<int64_t>(sizeof(Act));
    return ((reinterpret_cast<uintptr_t>(L.p.q) | reinterpret_cast<uintptr_t>(L.p.k) |
             reinterpret_cast<uintptr_t>(L.p.v)) & 15) == 0 &&
           (L.p.q_ts * es) % 16 == 0 && (L.p.k_ts * es) % 16 == 0 && (L.p.v_ts * es) % 16 == 0;
  };
  const int exact =
      (TC && low_precision && !(L.p.flags & GDN_RSSM_NORMALIZE_QK) && (QT < 8 || rows16())) ? 1 : 0;
  void (*kernel)(const CUtensorMap, const VerifyParams) = nullptr;
  int smem = 0;
  if constexpr (TC) {
    if constexpr (low_precision) {
      if (exact) {
        kernel = gated ? verify_tc_kernel<QT, Act, true, true> : verify_tc_kernel<QT, Act, false, true>;
        smem = verify_tc_smem_bytes<QT, Act, true>();
      }
    }
    if (!exact) {
      kernel = gated ? verify_tc_kernel<QT, Act, true, false> : verify_tc_kernel<QT, Act, false, false>;
      smem = verify_tc_smem_bytes<QT, Act, false>();
    }
  } else {
    kernel = verify_kernel<DIM, QT, Act, St>;
    smem = verify_smem_bytes<DIM, QT, Act, St>();
  }
  static bool configured[2][2][64] = {};
  int dev = 0;
  GDN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("GDN RecoverSSM: device ordinal out of range");
    return GDN_RSSM_EUNSUPPORTED;
  }
  if (!configured[gated][exact][dev]) {
    GDN_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[gated][exact][dev] = true;
  }
  const int64_t units = L.p.rows * L.p.value_heads;
  if (units <= 0) return GDN_RSSM_OK;
  int64_t grid = units;  // CUDA-core kernel: one CTA per (row, value head) unit
  if constexpr (TC) {
    // tensor-core kernel: as many CTAs as fit at once, each walking units
    // blockIdx.x + k * gridDim.x
    grid = std::min<int64_t>(units, static_cast<int64_t>(sm_count_current_device()) * verify_tc_min_blocks<QT>());
  }
  kernel<<<static_cast<unsigned>(grid), kVerifyThreads, smem, L.stream>>>(map, L.p);
  GDN_CUDA(cudaGetLastError());
  return GDN_RSSM_OK;
}

template <int DIM, int QT, typename Act, typename St>
int launch_verify_variant(VerifyLaunch &L) {
  if constexpr (verify_uses_tensor_cores<DIM, St>()) {
    if (L.p.flags & GDN_RSSM_VERIFY_CUDA_CORES) return launch_verify_kernel<DIM, QT, Act, St, false>(L);
    return launch_verify_kernel<DIM, QT, Act, St, true>(L);
  } else {
    return launch_verify_kernel<DIM, QT, Act, St, false>(L);
  }
}

template <int DIM, typename Act, typename St>
int launch_verify_qt(VerifyLaunch &L) {
  const int64_t Q = L.p.query_len;
  if (Q <= 1) return launch_verify_variant<DIM, 1, Act, St>(L);
  if (Q <= 2) return launch_verify_variant<DIM, 2, Act, St>(L);
  if (Q <= 4) return launch_verify_variant<DIM, 4, Act, St>(L);
  return launch_verify_variant<DIM, 8, Act, St>(L);
}

template <typename Act>
int launch_verify_act(VerifyLaunch &L) {
  if (L.state_dtype == GDN_RSSM_F32) {
    switch (L.dim) {
      case 32: return launch_verify_qt<32, Act, float>(L);
      case 64: return launch_verify_qt<64, Act, float>(L);
      case 128: return launch_verify_qt<128, Act, float>(L);
    }
  } else if (L.state_dtype == GDN_RSSM_BF16) {
    switch (L.dim) {
      case 64: return launch_verify_qt<64, Act, __nv_bfloat16>(L);
      case 128: return launch_verify_qt<128, Act, __nv_bfloat16>(L);
    }
  }
  set_error("GDN RecoverSSM: unsupported verify state dtype / head dim");
  return GDN_RSSM_EUNSUPPORTED;
}

}  // namespace gdn_rssm

// Defines, for activation type ACT and suffix NAME, a device status word
// (GDN_RSSM_STATUS_WORD) and int gdn_rssm::launch_verify_NAME(VerifyLaunch&).
#define GDN_RSSM_VERIFY_TU(ACT, NAME)                                    \
  GDN_RSSM_STATUS_WORD(NAME)                                             \
  namespace gdn_rssm {                                                   \
  int launch_verify_##NAME(VerifyLaunch &L) {                            \
    L.p.status = status_ptr_for_device<symbol_##NAME>();                 \
    if (L.p.status == nullptr) {                                         \
      set_error("GDN RecoverSSM: cannot resolve the device status word"); \
      return GDN_RSSM_ECUDA;                                             \
    }                                                                    \
    return launch_verify_act<ACT>(L);                                    \
  }                                                                      \
  }
