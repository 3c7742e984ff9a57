// Accepted-prefix fold (grouped commit) kernel, sm_100a.
//
// Semantics: reference grouped fold (grouped_commit.py:325-480), per-context
// fold (kernels.py:1172-1324) and AscendC FoldEngine (fold.h:192-237).  Per
// (layer, row, value head): plan row p = layer_groups[layer]*capacity + row;
// if 0 < src < blocks, 0 < final < blocks, 0 < n <= Q and row < record_rows:
//     h = S[src];  for t < n: h = fma(corr_t, k_t, h * decay_t)
//     (store h to the boundary page when t + 1 == boundary_len, the boundary
//      page is valid and differs from the final page)
//     store h to the final page.
// The update is the reference's exact arithmetic order (tl.fma(c, k, h*d)).
//
// B200 design.  Pure HBM streaming: one CTA per unit, each thread owns a fixed
// 16-byte column chunk (so its key slice lives in registers for the whole
// window) and a strided set of rows; all of a thread's state chunks are
// loaded before any is folded, so ~64 KiB per CTA is in flight.  The corr
// vectors of the window are staged in shared memory and read as broadcasts.
// Every element is read and written by the same thread, so in-place commits
// and a boundary page that aliases the source page are race-free.
#pragma once

#include "params.cuh"

namespace gdn_rssm {


template <typename T>
struct Chunk16 {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ void unpack16(const uint4 raw, float *out, float) {
  out[0] = __uint_as_float(raw.x);
  out[1] = __uint_as_float(raw.y);
  out[2] = __uint_as_float(raw.z);
  out[3] = __uint_as_float(raw.w);
}
__device__ __forceinline__ void unpack16(const uint4 raw, float *out, __nv_bfloat16) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void unpack16(const uint4 raw, float *out, __half) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 hh = *reinterpret_cast<const __half2 *>(&w[i]);
    const float2 f = __half22float2(hh);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack16(const float *in, float) {
  return make_uint4(__float_as_uint(in[0]), __float_as_uint(in[1]), __float_as_uint(in[2]), __float_as_uint(in[3]));
}
__device__ __forceinline__ uint4 pack16(const float *in, __nv_bfloat16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t *>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int DIM, typename St, typename Kt>
__global__ void __launch_bounds__(kFoldThreads, 2) fold_kernel(const FoldParams p) {
  constexpr int EPC = Chunk16<St>::N;      // state elements per 16-B chunk
  constexpr int CPR = DIM / EPC;           // chunks per state row
  constexpr int RSTEP = kFoldThreads / CPR;  // rows between a thread's chunks
  constexpr int CPT = (DIM + RSTEP - 1) / RSTEP;  // chunks per thread (last may be empty)
  static_assert(kFoldThreads % CPR == 0, "fold layout");
  __shared__ float s_corr[kMaxWindow][DIM];
  __shared__ float s_decay[kMaxWindow];

  const int64_t HV = p.heads;
  const int64_t unit = blockIdx.x;
  const int head = static_cast<int>(unit % HV);
  const int64_t row = (unit / HV) % p.rows;
  const int64_t layer = unit / (HV * p.rows);
  if (row >= p.record_rows) return;
  const int64_t prow = static_cast<int64_t>(p.layer_groups[layer]) * p.plan_capacity + row;
  if (prow < 0 || prow >= p.plan_len) return;
  bool ok = true;
  const int64_t src = load_index_checked(p.source, prow, ok);
  const int n = p.lengths[prow];
  const int64_t fin = p.finals[prow];
  if (!ok || src <= p.null_block || src >= p.blocks || fin <= p.null_block || fin >= p.blocks || n <= 0 ||
      n > p.query_len || n > kMaxWindow)
    return;
  const int64_t bidx = p.boundaries[prow];
  const int blen = p.boundary_lens[prow];
  const bool store_b = bidx > p.null_block && bidx < p.blocks && bidx != fin && blen > 0;

  const bool packed = (p.flags & GDN_RSSM_FOLD_PACKED) != 0;
  St *state = reinterpret_cast<St *>(p.state_addrs[layer]);
  const int64_t sbs = p.state_bs[layer];
  // 16-byte vector access needs a 16-byte aligned page base (the head / row
  // strides were checked on the host); refuse the unit instead of faulting.
  if ((reinterpret_cast<uintptr_t>(state) & 15) != 0 || sbs % EPC != 0) {
    if (threadIdx.x == 0) atomicExch(p.status, kStatusMisaligned);
    return;
  }
  const float *corr = reinterpret_cast<const float *>(p.corr_addrs[layer]) + row * p.corr_bs[layer] + head * p.corr_hs;
  const Kt *keyp;
  const float *decp;
  int64_t key_ts, dec_ts;
  if (packed) {
    keyp = reinterpret_cast<const Kt *>(corr + DIM);
    decp = corr + 2 * DIM;
    key_ts = p.corr_ts;
    dec_ts = p.corr_ts;
  } else {
    const int64_t kh = head / (HV / p.key_heads);
    keyp = reinterpret_cast<const Kt *>(p.key_addrs[layer]) + row * p.key_bs[layer] + kh * p.key_hs;
    decp = reinterpret_cast<const float *>(p.decay_addrs[layer]) + row * p.decay_bs[layer] + head * p.decay_hs;
    key_ts = p.key_ts;
    dec_ts = p.decay_ts;
  }

  const int tid = threadIdx.x;
  const int col = tid % CPR;      // fixed 16-B column chunk of this thread
  const int rbase = tid / CPR;    // rows rbase, rbase + RSTEP, ...
  const St *src_tile = state + src * sbs + head * p.state_hs;

  // issue every state load of this thread first
  uint4 raw[CPT];
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int r = rbase + i * RSTEP;
    if (DIM % RSTEP == 0 || r < DIM) raw[i] = __ldcs(reinterpret_cast<const uint4 *>(src_tile + r * p.state_vs + col * EPC));
  }
  // window records: corr -> shared, decay -> shared, key slice -> registers
  for (int i = tid; i < n * DIM; i += kFoldThreads) {
    const int t = i / DIM, e = i % DIM;
    s_corr[t][e] = corr[t * p.corr_ts + e];
  }
  if (tid < n) s_decay[tid] = decp[tid * dec_ts];
  float kk[kMaxWindow][EPC];
#pragma unroll
  for (int t = 0; t < kMaxWindow; ++t) {
#pragma unroll
    for (int e = 0; e < EPC; ++e) kk[t][e] = t < n ? to_f32<Kt>(keyp[t * key_ts + col * EPC + e]) : 0.f;
  }
  __syncthreads();

  St *fin_tile = state + fin * sbs + head * p.state_hs;
  St *b_tile = state + bidx * sbs + head * p.state_hs;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int r = rbase + i * RSTEP;
    if (DIM % RSTEP != 0 && r >= DIM) break;
    float hcur[EPC];
    unpack16(raw[i], hcur, St());
#pragma unroll
    for (int t = 0; t < kMaxWindow; ++t) {
      if (t < n) {
        const float c = s_corr[t][r];
        const float d = s_decay[t];
#pragma unroll
        for (int e = 0; e < EPC; ++e) hcur[e] = fmaf(c, kk[t][e], hcur[e] * d);
        if (store_b && t + 1 == blen) {
          *reinterpret_cast<uint4 *>(b_tile + r * p.state_vs + col * EPC) = pack16(hcur, St());
        }
      }
    }
    *reinterpret_cast<uint4 *>(fin_tile + r * p.state_vs + col * EPC) = pack16(hcur, St());
  }
}

}  // namespace gdn_rssm
