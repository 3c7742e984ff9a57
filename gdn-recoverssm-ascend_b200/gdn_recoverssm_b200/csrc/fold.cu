// Fold / plan / conv-compaction launchers.
#include "fold.cuh"
#include "plan.cuh"

GDN_RSSM_STATUS_WORD(fold)

namespace gdn_rssm {

// CTAs per unit: fp32 tiles at K = V = 128 are folded in two 64-row halves.
#ifndef GDN_RSSM_FOLD_PARTS
#define GDN_RSSM_FOLD_PARTS 2
#endif
template <int DIM, typename St>
constexpr int fold_parts() {
  return (DIM == 128 && sizeof(St) == 4) ? GDN_RSSM_FOLD_PARTS : 1;
}

template <int DIM, typename St, typename Kt, int PARTS>
int launch_fold_variant(FoldParams p, cudaStream_t stream) {
  p.status = status_ptr_for_device<symbol_fold>();
  if (p.status == nullptr) {
    set_error("GDN RecoverSSM: cannot resolve the device status word");
    return GDN_RSSM_ECUDA;
  }
  constexpr int smem = fold_smem_bytes<DIM, St, PARTS>();
  static bool configured[64] = {false};
  int dev = 0;
  GDN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("GDN RecoverSSM: device ordinal out of range");
    return GDN_RSSM_EUNSUPPORTED;
  }
  if (!configured[dev]) {
    GDN_CUDA(cudaFuncSetAttribute(fold_kernel<DIM, St, Kt, PARTS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  // one CTA per (layer, row, value head) unit, launched as a programmatic
  // dependent of the kernel before it (the plan): its CTAs become resident
  // while the plan runs and wait in the kernel for the plan's results
  const int64_t grid = p.layers * p.rows * p.heads * PARTS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(FoldShape<DIM, St, PARTS>::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GDN_CUDA(cudaLaunchKernelEx(&cfg, fold_kernel<DIM, St, Kt, PARTS>, p));
  return GDN_RSSM_OK;
}

template <int DIM, typename St>
int launch_fold_key(const FoldParams &p, int32_t key_dtype, cudaStream_t stream) {
  switch (key_dtype) {
    case GDN_RSSM_F32: return launch_fold_variant<DIM, St, float, fold_parts<DIM, St>()>(p, stream);
    case GDN_RSSM_BF16: return launch_fold_variant<DIM, St, __nv_bfloat16, fold_parts<DIM, St>()>(p, stream);
    case GDN_RSSM_F16: return launch_fold_variant<DIM, St, __half, fold_parts<DIM, St>()>(p, stream);
  }
  set_error("GDN RecoverSSM: unsupported record key dtype");
  return GDN_RSSM_EUNSUPPORTED;
}

template <typename St>
int launch_fold_dim(const FoldParams &p, int dim, int32_t key_dtype, cudaStream_t stream) {
  switch (dim) {
    case 32: return launch_fold_key<32, St>(p, key_dtype, stream);
    case 64: return launch_fold_key<64, St>(p, key_dtype, stream);
    case 128: return launch_fold_key<128, St>(p, key_dtype, stream);
  }
  set_error("GDN RecoverSSM: unsupported fold head dim");
  return GDN_RSSM_EUNSUPPORTED;
}

int launch_fold(const FoldParams &p, int dim, int32_t state_dtype, int32_t key_dtype, cudaStream_t stream) {
  if (state_dtype == GDN_RSSM_F32) return launch_fold_dim<float>(p, dim, key_dtype, stream);
  if (state_dtype == GDN_RSSM_BF16) return launch_fold_dim<__nv_bfloat16>(p, dim, key_dtype, stream);
  set_error("GDN RecoverSSM: fold state must be FP32 or BF16");
  return GDN_RSSM_EUNSUPPORTED;
}

static unsigned blocks_for(int64_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

// Launch as a programmatic dependent of the previous kernel in the stream: the
// kernel waits in its prologue (griddepcontrol.wait) for that grid's
// completion and memory, so only the launch latency overlaps.
template <typename Params>
static int launch_dependent(void (*kernel)(Params), const Params &p, dim3 grid, unsigned threads,
                            cudaStream_t stream, unsigned smem = 0) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GDN_CUDA(cudaLaunchKernelEx(&cfg, kernel, p));
  return GDN_RSSM_OK;
}

int launch_commit_plan(const CommitPlanParams &p, cudaStream_t stream) {
  return launch_dependent(commit_plan_kernel, p, blocks_for(p.rows, 128), 128, stream);
}

int launch_grouped_plan(const GroupedPlanParams &p, cudaStream_t stream) {
  return launch_dependent(grouped_plan_kernel, p, blocks_for(p.rows, 128), 128, stream);
}

int launch_publish_align(const PublishParams &p, cudaStream_t stream) {
  publish_align_kernel<<<blocks_for(p.rows, 128), 128, 0, stream>>>(p);
  GDN_CUDA(cudaGetLastError());
  return GDN_RSSM_OK;
}

int launch_compact_conv(const ConvParams &params, int elem_size, cudaStream_t stream) {
  ConvParams p = params;
  // chunk of channels per CTA: the largest that lets the contiguous path
  // stage three chunks in the default 48 KB of shared memory
  p.chunk = kConvChannelsPerCta;
  const int64_t row_bytes = p.window * elem_size;
  while (p.chunk > 64 && 3 * p.chunk * row_bytes > kConvSmemLimit) p.chunk /= 2;
  p.vec = (3 * p.chunk * row_bytes <= kConvSmemLimit && (p.chunk * row_bytes) % 16 == 0) ? 1 : 0;
  const unsigned smem = p.vec ? static_cast<unsigned>(3 * p.chunk * row_bytes) : 0u;
  // x: (layer, row); y: chunks of channels
  const dim3 grid(static_cast<unsigned>(p.layers * p.rows), static_cast<unsigned>((p.conv_dim + p.chunk - 1) / p.chunk));
  p.status = status_ptr_for_device<symbol_fold>();
  if (p.status == nullptr) {
    set_error("GDN RecoverSSM: cannot resolve the device status word");
    return GDN_RSSM_ECUDA;
  }
  // shared memory first (four 48 KB CTAs per SM), and room for the staging
  // chunks beside the kernel's static mbarrier
  static bool configured[2][64] = {};
  int dev = 0;
  GDN_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && (elem_size == 2 || elem_size == 4) && !configured[elem_size / 4][dev]) {
    if (elem_size == 2) {
      GDN_CUDA(cudaFuncSetAttribute(compact_conv_kernel<uint16_t>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared));
      GDN_CUDA(cudaFuncSetAttribute(compact_conv_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kConvSmemLimit));
    } else {
      GDN_CUDA(cudaFuncSetAttribute(compact_conv_kernel<uint32_t>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared));
      GDN_CUDA(cudaFuncSetAttribute(compact_conv_kernel<uint32_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kConvSmemLimit));
    }
    configured[elem_size / 4][dev] = true;
  }
  switch (elem_size) {  // a programmatic dependent of the plan, as the fold behind it is of this kernel
    case 2: return launch_dependent(compact_conv_kernel<uint16_t>, p, grid, kConvThreads, stream, smem);
    case 4: return launch_dependent(compact_conv_kernel<uint32_t>, p, grid, kConvThreads, stream, smem);
    default:
      set_error("GDN RecoverSSM: conv state element size must be 2 or 4 bytes");
      return GDN_RSSM_EUNSUPPORTED;
  }
}

}  // namespace gdn_rssm
