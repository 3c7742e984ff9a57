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
// B200 design: one CTA (256 threads) per unit, three resident per SM -- or,
// for fp32 tiles at K = V = 128, two CTAs of 128 threads per unit, each
// folding 64 of the 128 state rows, six resident per SM (PARTS below).
// Thread 0 starts one bulk copy (cp.async.bulk, completion on an mbarrier) of
// the CTA's rows of the source state tile into shared memory -- 64 (or 32)
// KiB in flight per CTA without holding registers -- while all threads stage
// the window's corr / decay records in shared memory and their key slice in
// registers (each thread owns one 16-byte column chunk of the tile and a
// strided set of rows).  The fold then streams the final state, and the
// boundary snapshot mid-fold, straight to HBM with 16-byte stores.  The
// CTA's whole source rows are in shared memory before any of its stores, and
// no two CTAs share a row, so in-place commits and a boundary page that
// aliases the source page are safe.
#pragma once

#include "params.cuh"
#include "ptx.cuh"

namespace gdn_rssm {

constexpr uint64_t kFoldWaitLimitNs = 1000000000ull;  // 1 s

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

// PARTS: the unit's V x K tile is folded by PARTS CTAs of DIM / PARTS state
// rows each (kFoldThreads / PARTS threads): the same work per thread and per
// SM in smaller pieces, so the last wave of a small batch is shorter.
template <int DIM, typename St, int PARTS = 1>
struct FoldShape {
  static constexpr int ROWS = DIM / PARTS;                // state rows of one CTA
  static constexpr int THREADS = kFoldThreads / PARTS;
  static constexpr int EPC = Chunk16<St>::N;             // state elements per 16-byte chunk
  static constexpr int CPR = DIM / EPC;                  // chunks per state row
  static constexpr int RSTEP = THREADS / CPR;            // rows between a thread's chunks
  static constexpr int CPT = (ROWS + RSTEP - 1) / RSTEP;  // chunks per thread (last may be empty)
  static constexpr int TILE = ROWS * DIM * sizeof(St);
  static constexpr int CORR = kMaxWindow * ROWS * 4;
  static constexpr int SMEM = 128 /* alignment slack */ + TILE + CORR + 64;
  static_assert(THREADS % CPR == 0 && DIM % PARTS == 0, "fold layout");
};

template <int DIM, typename St, int PARTS = 1>
constexpr int fold_smem_bytes() {
  return FoldShape<DIM, St, PARTS>::SMEM;
}

// Three resident CTAs per SM (times PARTS); two for 2-byte state tiles, whose
// 8-wide key slices need more registers.
template <typename St, int PARTS = 1>
constexpr int fold_min_blocks() {
  return (sizeof(St) == 4 ? 3 : 2) * PARTS;
}

template <int DIM, typename St, typename Kt, int PARTS>
__global__ void __launch_bounds__(FoldShape<DIM, St, PARTS>::THREADS, fold_min_blocks<St, PARTS>())
    fold_kernel(const FoldParams p) {
  using Sh = FoldShape<DIM, St, PARTS>;
  constexpr int EPC = Sh::EPC, CPR = Sh::CPR, RSTEP = Sh::RSTEP, CPT = Sh::CPT, ROWS = Sh::ROWS;
  constexpr int NT = Sh::THREADS;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  unsigned char *tile = smem;
  float(*s_corr)[ROWS] = reinterpret_cast<float(*)[ROWS]>(smem + Sh::TILE);
  float *s_decay = reinterpret_cast<float *>(smem + Sh::TILE + Sh::CORR);
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + Sh::TILE + Sh::CORR + 32);

  const int64_t HV = p.heads;
  const int64_t unit = blockIdx.x / PARTS;
  const int r0 = static_cast<int>(blockIdx.x % PARTS) * ROWS;  // first state row of this CTA
  const int head = static_cast<int>(unit % HV);
  const int64_t row = (unit / HV) % p.rows;
  const int64_t layer = unit / (HV * p.rows);
  if (row >= p.record_rows) return;
  // launched programmatically behind the plan (or the conv compaction behind
  // it, itself behind the plan): wait for that grid and its memory before
  // reading plans, records or pages
  ptx::wait_prerequisite_grid();
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
  St *state = reinterpret_cast<St *>(p.state_addrs[layer]);
  const int64_t sbs = p.state_bs[layer];
  // 16-byte copies and stores need a 16-byte aligned page base (head / row
  // strides were checked on the host): refuse the unit instead of faulting.
  if ((reinterpret_cast<uintptr_t>(state) & 15) != 0 || sbs % EPC != 0) {
    if (threadIdx.x == 0) atomicExch(p.status, kStatusMisaligned);
    return;
  }
  const int tid = threadIdx.x;
  const St *src_tile = state + src * sbs + head * p.state_hs + r0 * p.state_vs;
  if (tid < 32) {
    if (tid == 0) {
      ptx::mbar_init(bar, 1);
      ptx::fence_mbar_init();
      ptx::mbar_arrive_expect_tx(bar, Sh::TILE);
    }
    __syncwarp();
    if (p.state_vs == DIM) {
      if (tid == 0) ptx::bulk_load(tile, src_tile, Sh::TILE, bar);
    } else {
      for (int r = tid; r < ROWS; r += 32)
        ptx::bulk_load(tile + r * DIM * sizeof(St), src_tile + r * p.state_vs, DIM * sizeof(St), bar);
    }
  }
  // window records: corr -> shared, decay -> shared, this thread's key slice -> registers
  const bool packed = (p.flags & GDN_RSSM_FOLD_PACKED) != 0;
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
  const int col = tid % CPR;    // fixed 16-byte column chunk of this thread
  const int rbase = tid / CPR;  // rows rbase, rbase + RSTEP, ...
  float cv[kMaxWindow * ROWS / NT + 1];
  {
    // issue every record load before any store (one memory round trip); the
    // corrections of this CTA's rows only
    constexpr int PER = (kMaxWindow * ROWS + NT - 1) / NT;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int idx = tid + c * NT;
      const int t = idx / ROWS, e = idx % ROWS;
      cv[c] = (t < n) ? corr[t * p.corr_ts + r0 + e] : 0.f;
    }
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int idx = tid + c * NT;
      const int t = idx / ROWS, e = idx % ROWS;
      if (t < n) s_corr[t][e] = cv[c];
    }
  }
  float kk[kMaxWindow][EPC];
  float dd[kMaxWindow];
#pragma unroll
  for (int t = 0; t < kMaxWindow; ++t) {
    dd[t] = t < n ? decp[t * dec_ts] : 1.f;
#pragma unroll
    for (int e = 0; e < EPC; ++e) kk[t][e] = t < n ? to_f32<Kt>(keyp[t * key_ts + col * EPC + e]) : 0.f;
  }
  (void)s_decay;
  __syncthreads();  // corr staged; barrier initialised
  if (!ptx::mbar_wait_bounded(bar, 0, kFoldWaitLimitNs)) {
    if (tid == 0) atomicExch(p.status, kStatusTmaTimeout);
    ptx::mbar_wait_bounded(bar, 0, kFoldWaitLimitNs);  // let an in-flight copy land before exiting
    return;
  }
  St *fin_tile = state + fin * sbs + head * p.state_hs + r0 * p.state_vs;
  St *b_tile = state + bidx * sbs + head * p.state_hs + r0 * p.state_vs;
#pragma unroll 4
  for (int i = 0; i < CPT; ++i) {
    const int r = rbase + i * RSTEP;  // row of this CTA's slab
    if (ROWS % RSTEP != 0 && r >= ROWS) break;
    const uint4 raw = *reinterpret_cast<const uint4 *>(tile + (r * DIM + col * EPC) * sizeof(St));
    float h[EPC];
    unpack16(raw, h, St());
#pragma unroll
    for (int t = 0; t < kMaxWindow; ++t) {
      if (t < n) {
        const float c = s_corr[t][r];
#pragma unroll
        for (int e = 0; e < EPC; ++e) h[e] = fmaf(c, kk[t][e], h[e] * dd[t]);
        if (store_b && t + 1 == blen)
          *reinterpret_cast<uint4 *>(b_tile + r * p.state_vs + col * EPC) = pack16(h, St());
      }
    }
    *reinterpret_cast<uint4 *>(fin_tile + r * p.state_vs + col * EPC) = pack16(h, St());
  }
}

}  // namespace gdn_rssm
