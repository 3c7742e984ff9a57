// Shared device/host helpers for the RecoverSSM sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "gdn_recoverssm_b200.h"

namespace gdn_rssm {

constexpr int kMaxWindow = 8;  // spec_query_len bound (kernels.py:101, verify.h:21)
constexpr int kVerifyThreads = 256;
constexpr int kFoldThreads = 256;

// ---------------------------------------------------------------- errors ---
// Thread-local message of the last failed C-ABI call.
void set_error(const std::string &msg);
const char *get_error();

#define GDN_REQUIRE(cond, msg)                       \
  do {                                               \
    if (!(cond)) {                                   \
      ::gdn_rssm::set_error(std::string("GDN RecoverSSM: ") + (msg)); \
      return GDN_RSSM_EINVAL;                        \
    }                                                \
  } while (0)

#define GDN_CUDA(call)                                                      \
  do {                                                                      \
    cudaError_t _e = (call);                                                \
    if (_e != cudaSuccess) {                                                \
      ::gdn_rssm::set_error(std::string("GDN RecoverSSM CUDA error: ") +   \
                            cudaGetErrorString(_e) + " at " #call);         \
      return GDN_RSSM_ECUDA;                                                \
    }                                                                       \
  } while (0)

// Status codes written by kernels whose bounded wait gave up (see the
// translation units that own a device status word; gdn_rssm_device_status()
// reads and clears all of them).
constexpr int32_t kStatusTmaTimeout = 1;
constexpr int32_t kStatusMisaligned = 2;
constexpr int32_t kStatusMmaTimeout = 4;

// Resolve (once per device) the device address of a translation unit's status
// word; GetSymbol wraps cudaGetSymbolAddress for that word.
template <int32_t *(*GetSymbol)()>
int32_t *status_ptr_for_device() {
  static int32_t *ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (ptrs[dev] == nullptr) ptrs[dev] = GetSymbol();
  return ptrs[dev];
}

// Defines a status word g_status_NAME private to this translation unit,
// gdn_rssm::symbol_NAME() (its device address) and
// gdn_rssm::read_status_NAME(int32_t*, cudaStream_t) (read, then clear).
#define GDN_RSSM_STATUS_WORD(NAME)                                                    \
  namespace gdn_rssm {                                                                \
  static __device__ int32_t g_status_##NAME = 0;                                      \
  static int32_t *symbol_##NAME() {                                                   \
    void *ptr = nullptr;                                                              \
    if (cudaGetSymbolAddress(&ptr, g_status_##NAME) != cudaSuccess) return nullptr;   \
    return static_cast<int32_t *>(ptr);                                               \
  }                                                                                   \
  int read_status_##NAME(int32_t *out, cudaStream_t stream) {                         \
    int32_t value = 0, zero = 0;                                                      \
    GDN_CUDA(cudaMemcpyFromSymbolAsync(&value, g_status_##NAME, sizeof(int32_t), 0,   \
                                       cudaMemcpyDeviceToHost, stream));              \
    GDN_CUDA(cudaMemcpyToSymbolAsync(g_status_##NAME, &zero, sizeof(int32_t), 0,      \
                                     cudaMemcpyHostToDevice, stream));                \
    GDN_CUDA(cudaStreamSynchronize(stream));                                          \
    *out = value;                                                                     \
    return GDN_RSSM_OK;                                                               \
  }                                                                                   \
  }

// ------------------------------------------------------------- conversion ---
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Runtime-typed scalar load (float element types).
__device__ __forceinline__ float load_float(const void *p, int64_t i, int32_t dtype) {
  switch (dtype) {
    case GDN_RSSM_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    case GDN_RSSM_F16: return __half2float(static_cast<const __half *>(p)[i]);
    default: return static_cast<const float *>(p)[i];
  }
}

// Runtime-typed integer load from an index view (I32 / I64).
__device__ __forceinline__ int64_t load_index(const gdn_rssm_index_view &v, int64_t i) {
  const int64_t off = i * v.stride;
  return v.dtype == GDN_RSSM_I64 ? static_cast<const int64_t *>(v.data)[off]
                                 : static_cast<int64_t>(static_cast<const int32_t *>(v.data)[off]);
}

// Bounded index-view read: out-of-range -> `fallback`, ok=false.
__device__ __forceinline__ int64_t load_index_checked(const gdn_rssm_index_view &v, int64_t i, bool &ok,
                                                      int64_t fallback = 0) {
  if (v.data == nullptr || i < 0 || i >= v.length) {
    ok = false;
    return fallback;
  }
  return load_index(v, i);
}

__device__ __forceinline__ void store_index(const gdn_rssm_out_view &v, int64_t i, int64_t value) {
  const int64_t off = i * v.stride;
  if (v.dtype == GDN_RSSM_I64) {
    static_cast<int64_t *>(v.data)[off] = value;
  } else {
    static_cast<int32_t *>(v.data)[off] = static_cast<int32_t>(value);
  }
}

__device__ __forceinline__ int64_t load_table(const gdn_rssm_table_view &t, int64_t r, int64_t c) {
  const int64_t off = r * t.row_stride + c * t.col_stride;
  return t.dtype == GDN_RSSM_I64 ? static_cast<const int64_t *>(t.data)[off]
                                 : static_cast<int64_t>(static_cast<const int32_t *>(t.data)[off]);
}

// Python-style floor division for the plan arithmetic on possibly negative
// numerators (Triton `//` of the reference plans on nonnegative operands).
__device__ __forceinline__ int64_t floordiv(int64_t a, int64_t b) {
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
  return q;
}

// SM count of the current device (cached per device).
inline int sm_count_current_device() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    counts[dev] = n;
  }
  return counts[dev];
}

// Host helpers.
bool host_dtype_is_float(int32_t d);
int host_dtype_size(int32_t d);

}  // namespace gdn_rssm
