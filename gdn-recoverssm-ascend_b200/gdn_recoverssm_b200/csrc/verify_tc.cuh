// Tensor-core verify kernel for K = V = 128 with an fp32 state pool (sm_100a).
//
// Same semantics and the same chunked form of the Q-step recurrence as
// verify_kernel (verify.cuh): the only O(V K) work is P = S_0 X^T, the 2Q dot
// products of every state row with the window's k_hat / q_tilde vectors.  Here
// that product runs on the 5th-generation tensor cores (tcgen05.mma,
// kind::tf32, M = 128 state rows, accumulators in tensor memory) instead of
// 2Q x 128 FMAs per row on the CUDA cores.
//
// fp32 accuracy from tf32 operands (three-product split): every operand x is
// written as x = hi(x) + lo(x) with hi(x) = x with its low 13 mantissa bits
// cleared (exactly a tf32 value) and lo(x) = x - hi(x) (exact in fp32).  The
// B operand holds the rows [hi(X); lo(X)] (2 x 2Q rows, padded to a multiple
// of 16), so one MMA pass over the tile as loaded gives S_hi X_hi and S_hi
// X_lo side by side in tensor memory (the tensor core reads an fp32 operand
// as tf32 by dropping the same 13 bits).  The tile is then rewritten in place
// as lo(S) and a second pass accumulates lo(S) X_hi and lo(S) X_lo into the
// same columns.  Column j plus column 2Q + j is the dot product with only the
// lo x lo truncation left out: relative error ~2^-21, the size of fp32
// rounding over a 128-term sum.
//
// CTA flow (256 threads, one unit = one (row, value head)):
//   thread 0: TMA of the 64 KiB tile (4-D tensor map, 128-byte swizzle: the
//             layout the MMA's K-major descriptor reads directly);
//   warp 0:   allocates 32 tensor-memory columns;
//   all:      stage hi/lo(X) into the B operand, v, g, beta, key and decay
//             records; Gram coefficients while the tile is in flight;
//   thread 0: MMA pass 1 -> commit; all: rewrite the tile as lo(S);
//   thread 0: MMA pass 2 -> commit; every warp loads its 32 rows' sums from
//             tensor memory (one row per lane) and runs the recurrence: warps
//             0-3 write the correction records, warps 4-7 the outputs.
// Every wait is bounded (1 s) and reported through the status word; tensor
// memory is released on every path after it was allocated.
#pragma once

#include "verify.cuh"

namespace gdn_rssm {

template <int QT, typename Act>
struct VerifyTcShape {
  static constexpr int DIM = 128;
  static constexpr int NJ = 2 * QT;                    // dot products per state row
  static constexpr int NB = (2 * NJ + 15) / 16 * 16;   // B operand rows: hi(X), lo(X), zero padding
  static constexpr int TMEM_COLS = 32;                 // accumulator columns (>= NB, power of two)
  static constexpr int SLAB = DIM * 128;               // one 32-column K slab of the tile (bytes)
  static constexpr int TILE = DIM * DIM * 4;
  static constexpr int B_SLAB = NB * 128;
  static constexpr int B_BYTES = 4 * B_SLAB;
  static constexpr int V_BYTES = (QT * DIM * static_cast<int>(sizeof(Act)) + 15) / 16 * 16;
  struct Small {
    uint64_t tile_bar;
    uint64_t mma_bar;
    uint32_t tmem;
    float A[QT];
    float beta[QT];
    float dec[QT];
    float mkk[QT][QT];  // D[t][s] * (k_s . k_t), s < t
    float mkq[QT][QT];  // D[t][s] * (k_s . q_t), s <= t
  };
  static constexpr int SMEM = 1024 /* alignment slack */ + TILE + B_BYTES + V_BYTES + static_cast<int>(sizeof(Small));
  static_assert(NB <= TMEM_COLS && (NB == 16 || NB == 32), "accumulator columns");
  static_assert(B_SLAB % 1024 == 0, "B operand slabs must stay 1024-byte aligned");
};

template <int QT, typename Act>
constexpr int verify_tc_smem_bytes() {
  return VerifyTcShape<QT, Act>::SMEM;
}

// Three resident CTAs per SM up to Q = 4 (75 KB of shared memory each), two at
// Q = 8.
template <int QT>
constexpr int verify_tc_min_blocks() {
  return QT >= 8 ? 2 : 3;
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

// Gram coefficients of the window from the B operand ([hi(X); lo(X)], rows
// 128 bytes apart in 4 K slabs of B_SLAB bytes, 16-byte chunk c of row n at
// chunk c ^ (n % 8)):
//     mkk[t][s] = D[t][s] (k_s . k_t)  for s < t,
//     mkq[t][s] = D[t][s] (k_s . q_t)  for s <= t,   D[t][s] = prod_{s<r<=t} dec[r].
// One task = (pair, K slab): 32 elements, x = hi + lo (exact); the 4 tasks of
// a pair sit on 4 consecutive lanes and are summed with two shuffles.  Lanes
// of one pair walk the slab's chunks in rotated order so that they read
// different banks.
template <int QT, int NJ, int B_SLAB>
__device__ __forceinline__ void gram_coefficients(const unsigned char *bop, const float *dec, float (*mkk)[QT],
                                                  float (*mkq)[QT], int tid) {
  constexpr int NKK = QT * (QT - 1) / 2;
  constexpr int TASKS = QT * QT * 4;
  constexpr int ROUNDED = (TASKS + 31) / 32 * 32;  // whole warps take part in the shuffles
  for (int task = tid; task < ROUNDED; task += kVerifyThreads) {
    const bool live = task < TASKS;
    const int pr = live ? task >> 2 : 0, m = task & 3;
    const int kind = pr >= NKK ? 1 : 0;
    int rem = kind ? pr - NKK : pr, t = 0;
    while (rem >= (kind ? t + 1 : t)) {
      rem -= kind ? t + 1 : t;
      ++t;
    }
    const int s2 = rem;
    const int a = s2, b = kind ? QT + t : t;
    const unsigned char *slab = bop + m * B_SLAB;
    const unsigned char *ha = slab + a * 128, *la = slab + (NJ + a) * 128;
    const unsigned char *hb = slab + b * 128, *lb = slab + (NJ + b) * 128;
    const int sa = a & 7, sla = (NJ + a) & 7, sb = b & 7, slb = (NJ + b) & 7;
    float acc = 0.f;
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const int c = (i + 2 * m) & 7;
      const float4 xa = *reinterpret_cast<const float4 *>(ha + ((c ^ sa) << 4));
      const float4 ya = *reinterpret_cast<const float4 *>(la + ((c ^ sla) << 4));
      const float4 xb = *reinterpret_cast<const float4 *>(hb + ((c ^ sb) << 4));
      const float4 yb = *reinterpret_cast<const float4 *>(lb + ((c ^ slb) << 4));
      acc = fmaf(xa.x + ya.x, xb.x + yb.x, acc);
      acc = fmaf(xa.y + ya.y, xb.y + yb.y, acc);
      acc = fmaf(xa.z + ya.z, xb.z + yb.z, acc);
      acc = fmaf(xa.w + ya.w, xb.w + yb.w, acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (live && m == 0) {
      float d = 1.f;
      for (int r2 = s2 + 1; r2 <= t; ++r2) d *= dec[r2];
      if (kind == 0) {
        mkk[t][s2] = d * acc;
      } else {
        mkq[t][s2] = d * acc;
      }
    }
  }
}

template <int QT, typename Act>
__global__ void __launch_bounds__(kVerifyThreads, verify_tc_min_blocks<QT>())
    verify_tc_kernel(const __grid_constant__ CUtensorMap state_map, const VerifyParams p) {
  using Sh = VerifyTcShape<QT, Act>;
  using Small = typename Sh::Small;
  constexpr int DIM = Sh::DIM, NJ = Sh::NJ, NB = Sh::NB, EPL = DIM / 32;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char *tile = smem;
  unsigned char *bop = smem + Sh::TILE;
  Act(*vs)[DIM] = reinterpret_cast<Act(*)[DIM]>(smem + Sh::TILE + Sh::B_BYTES);
  Small &sm = *reinterpret_cast<Small *>(smem + Sh::TILE + Sh::B_BYTES + Sh::V_BYTES);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int64_t HV = p.value_heads;
  const int64_t row = blockIdx.x / HV;
  const int hv = static_cast<int>(blockIdx.x % HV);
  const int ratio = static_cast<int>(HV / p.heads);
  const int h = hv / ratio;
  const int Q = static_cast<int>(p.query_len);

  const int64_t bos = load_typed_index(p.qsl, row * p.qsl_stride, p.qsl_dtype);
  const int64_t eos = load_typed_index(p.qsl, (row + 1) * p.qsl_stride, p.qsl_dtype);
  const int64_t qlen = eos - bos;
  const int64_t slot = load_typed_index(p.indices, row * p.index_stride, p.index_dtype);
  int valid_mask = 0;
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    const int64_t tok = bos + t;
    if (t < Q && t < qlen && tok >= 0 && tok < p.tokens) valid_mask |= 1 << t;
  }
  Act *out = static_cast<Act *>(p.out);

  // ---- null / out-of-pool slot: zero output for the row's window ---------- //
  if (slot <= p.null_block || slot >= p.blocks) {
    for (int i = tid; i < QT * DIM; i += kVerifyThreads) {
      const int t = i / DIM, e = i % DIM;
      if ((valid_mask >> t) & 1) out[(bos + t) * p.out_ts + hv * DIM + e] = from_f32<Act>(0.f);
    }
    return;
  }

  // ---- tile load first, tensor memory next --------------------------------- //
  if (tid == 0) {
    ptx::prefetch_tensormap(&state_map);
    ptx::mbar_init(&sm.tile_bar, 1);
    ptx::mbar_init(&sm.mma_bar, 1);
    ptx::fence_mbar_init();
    ptx::mbar_arrive_expect_tx(&sm.tile_bar, Sh::TILE);
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int qt = 0; qt < 4; ++qt)
        ptx::tma_load_4d(tile + m * Sh::SLAB + qt * 32 * 128, &state_map, &sm.tile_bar, m * 32, qt * 32, hv,
                         static_cast<int32_t>(slot));
  }
  if (warp == 0) {
    __syncwarp();  // the allocation is warp-wide (.sync.aligned)
    ptx::tmem_alloc(&sm.tmem, Sh::TMEM_COLS);
    ptx::tmem_relinquish();
  }

  // ---- stage the window ------------------------------------------------------ //
  const bool normalize = (p.flags & GDN_RSSM_NORMALIZE_QK) != 0;
  const bool packed = (p.flags & GDN_RSSM_RECORD_PACKED) != 0;
  const bool rec_ok = row < p.record_rows;
  {
    // q/k rows: warp w owns vectors w, w + 8, ... (k_t for j < QT, q_t after);
    // lane l holds K elements 4l .. 4l + 3 = chunk l % 8 of slab l / 8
    constexpr int PER_WARP = (NJ + 7) / 8;
    float x[PER_WARP][EPL];
#pragma unroll
    for (int c = 0; c < PER_WARP; ++c) {
      const int j = warp + 8 * c;
      const int t = j % QT;
      const bool live = j < NJ && ((valid_mask >> t) & 1);
      const Act *src = static_cast<const Act *>(j >= QT ? p.q : p.k);
      const int64_t base = (bos + t) * (j >= QT ? p.q_ts : p.k_ts) + static_cast<int64_t>(h) * DIM + lane * EPL;
#pragma unroll
      for (int u = 0; u < EPL; ++u) x[c][u] = live ? to_f32<Act>(src[base + u]) : 0.f;
    }
    const Act *vin = static_cast<const Act *>(p.v);
    constexpr int VPER = (QT * DIM + kVerifyThreads - 1) / kVerifyThreads;
    Act vv[VPER];
#pragma unroll
    for (int c = 0; c < VPER; ++c) {
      const int i = tid + c * kVerifyThreads;
      const int t = i / DIM, e = i % DIM;
      vv[c] = (i < QT * DIM && ((valid_mask >> t) & 1)) ? vin[(bos + t) * p.v_ts + hv * DIM + e] : from_f32<Act>(0.f);
    }
    float dec = 1.f, bet = 0.f;
    if (tid < QT && ((valid_mask >> tid) & 1)) {
      dec = expf(p.g[(bos + tid) * p.g_ts + hv]);
      bet = load_float(p.beta, (bos + tid) * p.beta_ts + hv, p.beta_dtype);
    }
#pragma unroll
    for (int c = 0; c < VPER; ++c) {
      const int i = tid + c * kVerifyThreads;
      if (i < QT * DIM) vs[i / DIM][i % DIM] = vv[c];
    }
    if (tid < QT) {
      sm.dec[tid] = dec;
      sm.beta[tid] = bet;
      if (rec_ok && ((valid_mask >> tid) & 1)) p.decay[row * p.decay_rs + hv * p.decay_hs + tid * p.decay_ts] = dec;
    }
    // zero padding rows of the B operand (Q < 4)
    if constexpr (NB > 2 * NJ) {
      constexpr int PAD_CHUNKS = 4 * (NB - 2 * NJ) * 8;
      for (int i = tid; i < PAD_CHUNKS; i += kVerifyThreads) {
        const int m = i / ((NB - 2 * NJ) * 8), rem = i % ((NB - 2 * NJ) * 8);
        const int n = 2 * NJ + rem / 8, ch = rem % 8;
        *reinterpret_cast<uint4 *>(bop + m * Sh::B_SLAB + n * 128 + (ch << 4)) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int c = 0; c < PER_WARP; ++c) {
      const int j = warp + 8 * c;
      if (j >= NJ) continue;
      const int t = j % QT;
      if (normalize) {
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < EPL; ++u) ss = fmaf(x[c][u], x[c][u], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float mul = rsqrtf(ss + 1e-6f);
#pragma unroll
        for (int u = 0; u < EPL; ++u) x[c][u] *= mul;
      }
      if (j < QT) {
        // key record: packed -> every value head keeps its copy; typed -> once per key head
        if (rec_ok && ((valid_mask >> t) & 1) && (packed || hv % ratio == 0)) {
          const int64_t kh = packed ? hv : h;
          const int32_t kd = packed ? GDN_RSSM_F32 : p.key_dtype;
#pragma unroll
          for (int u = 0; u < EPL; ++u)
            store_key(p.key, row * p.key_rs + kh * p.key_hs + t * p.key_ts + lane * EPL + u, x[c][u], kd);
        }
      } else {
#pragma unroll
        for (int u = 0; u < EPL; ++u) x[c][u] *= p.scale;
      }
      float hi[EPL], lo[EPL];
#pragma unroll
      for (int u = 0; u < EPL; ++u) {
        hi[u] = tf32_hi(x[c][u]);
        lo[u] = x[c][u] - hi[u];
      }
      const int m = lane >> 3, ch = lane & 7, jl = NJ + j;
      *reinterpret_cast<float4 *>(bop + m * Sh::B_SLAB + j * 128 + ((ch ^ (j & 7)) << 4)) =
          make_float4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<float4 *>(bop + m * Sh::B_SLAB + jl * 128 + ((ch ^ (jl & 7)) << 4)) =
          make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
  }
  ptx::fence_proxy_async_smem();  // B operand -> tensor-core reads
  ptx::tc_fence_before_sync();
  __syncthreads();  // B, v, dec, beta staged; barriers initialised; tensor memory allocated
  ptx::tc_fence_after_sync();
  const uint32_t tmem = sm.tmem;

  // ---- Gram coefficients (x = hi + lo, read back from the B operand) --------- //
  gram_coefficients<QT, NJ, Sh::B_SLAB>(bop, sm.dec, sm.mkk, sm.mkq, tid);
  if (tid == 0) {
    float a = 1.f;
#pragma unroll
    for (int t = 0; t < QT; ++t) {
      a *= sm.dec[t];
      sm.A[t] = a;
    }
  }

  constexpr uint32_t IDESC = ptx::tf32_instr_desc<128, NB>();
  const uint32_t tile_addr = ptx::smem_addr(tile), b_addr = ptx::smem_addr(bop);
  bool ok = true;
  // ---- the tile has landed (every thread: its data is read below) ------------ //
  if (__syncthreads_or(!ptx::mbar_wait_bounded(&sm.tile_bar, 0, kWaitLimitNs))) {
    if (tid == 0) atomicExch(p.status, kStatusTmaTimeout);
    ptx::mbar_wait_bounded(&sm.tile_bar, 0, kWaitLimitNs);  // let an in-flight copy land before exiting
    ok = false;
  }
  // ---- pass 1: S (read as tf32) x [hi(X); lo(X)] ----------------------------- //
  if (ok) {
    if (tid == 0) {
      ptx::tc_fence_after_sync();
#pragma unroll
      for (int kk = 0; kk < DIM / 8; ++kk) {
        const uint32_t sub = (kk & 3) * 32;  // K sub-block (8 tf32) inside the 128-byte row
        const uint64_t a = ptx::sw128_kmajor_desc(tile_addr + (kk >> 2) * Sh::SLAB + sub);
        const uint64_t b = ptx::sw128_kmajor_desc(b_addr + (kk >> 2) * Sh::B_SLAB + sub);
        ptx::mma_tf32(tmem, a, b, IDESC, kk > 0);
      }
      ptx::mma_commit(&sm.mma_bar);
    }
    if (__syncthreads_or(!ptx::mbar_wait_bounded(&sm.mma_bar, 0, kWaitLimitNs))) {
      if (tid == 0) atomicExch(p.status, kStatusMmaTimeout);
      ptx::mbar_wait_bounded(&sm.mma_bar, 0, kWaitLimitNs);
      ok = false;
    }
  }
  // ---- rewrite the tile as lo(S), pass 2 ------------------------------------- //
  if (ok) {
    ptx::tc_fence_after_sync();
    float4 *t4 = reinterpret_cast<float4 *>(tile);
#pragma unroll 4
    for (int c = tid; c < Sh::TILE / 16; c += kVerifyThreads) {
      float4 v = t4[c];
      v.x -= tf32_hi(v.x);
      v.y -= tf32_hi(v.y);
      v.z -= tf32_hi(v.z);
      v.w -= tf32_hi(v.w);
      t4[c] = v;
    }
    ptx::fence_proxy_async_smem();  // lo(S) -> tensor-core reads
    ptx::tc_fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      ptx::tc_fence_after_sync();
#pragma unroll
      for (int kk = 0; kk < DIM / 8; ++kk) {
        const uint32_t sub = (kk & 3) * 32;
        const uint64_t a = ptx::sw128_kmajor_desc(tile_addr + (kk >> 2) * Sh::SLAB + sub);
        const uint64_t b = ptx::sw128_kmajor_desc(b_addr + (kk >> 2) * Sh::B_SLAB + sub);
        ptx::mma_tf32(tmem, a, b, IDESC, true);
      }
      ptx::mma_commit(&sm.mma_bar);
    }
    if (__syncthreads_or(!ptx::mbar_wait_bounded(&sm.mma_bar, 1, kWaitLimitNs))) {
      if (tid == 0) atomicExch(p.status, kStatusMmaTimeout);
      ptx::mbar_wait_bounded(&sm.mma_bar, 1, kWaitLimitNs);
      ok = false;
    }
  }
  // ---- per-row recurrence: lane = state row of this warp's 32-lane quadrant --- //
  if (ok) {
    ptx::tc_fence_after_sync();
    const int quad = warp & 3;
    float d[NB];
    ptx::tmem_ld_sync<NB>(tmem + (static_cast<uint32_t>(quad * 32) << 16), d);
    float pr[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) pr[j] = d[j] + d[NJ + j];
    const int r = quad * 32 + lane;
    const bool writer_corr = warp < 4;
    float cr[QT];
#pragma unroll
    for (int t = 0; t < QT; ++t) {
      cr[t] = 0.f;
      if (!((valid_mask >> t) & 1)) continue;
      float kv = sm.A[t] * pr[t];
#pragma unroll
      for (int s2 = 0; s2 < t; ++s2) kv = fmaf(sm.mkk[t][s2], cr[s2], kv);
      cr[t] = sm.beta[t] * (to_f32<Act>(vs[t][r]) - kv);
      const int64_t tok = bos + t;
      if (writer_corr) {
        if (rec_ok) p.corr[row * p.corr_rs + hv * p.corr_hs + t * p.corr_ts + r] = cr[t];
      } else {
        float o = sm.A[t] * pr[QT + t];
#pragma unroll
        for (int s2 = 0; s2 <= t; ++s2) o = fmaf(sm.mkq[t][s2], cr[s2], o);
        out[tok * p.out_ts + hv * DIM + r] = from_f32<Act>(o);
      }
    }
  }
  // ---- release tensor memory (every path after the allocation) ---------------- //
  ptx::tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc(tmem, Sh::TMEM_COLS);
  }
}

}  // namespace gdn_rssm
