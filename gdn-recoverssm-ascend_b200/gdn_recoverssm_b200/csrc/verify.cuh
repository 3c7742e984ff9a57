// Speculative verify kernel (sm_100a).
//
// Semantics follow the reference verify (kernels.py:491-697; AscendC
// verify.h:350-398): per (sequence row, value head) "unit", read the fp32
// checkpoint S[V,K] read-only, run the gated delta rule over the Q draft
// tokens, write the attention output per token and one record per token
// [corr(V), k_hat(K), decay].
//
// B200 design.  One CTA (256 threads) per unit, up to 3 resident per SM.
//  * The whole S tile is staged into shared memory by TMA (4-D tensor map over
//    the [blocks, HV, V, K] pool, 128-byte swizzle, boxes of 128 B x V rows),
//    so each thread can read "its" state row 16 B at a time without bank
//    conflicts while the tile is in flight for the other resident CTAs.
//  * The Q-step recurrence is evaluated in its chunked form: with
//    A_t = prod_{s<=t} d_s and D[t][s] = prod_{s<r<=t} d_r,
//        S'_t k_t = A_t (S_0 k_t) + sum_{s<t}  D[t][s] (k_s . k_t) c_s
//        S_t q_t  = A_t (S_0 q_t) + sum_{s<=t} D[t][s] (k_s . q_t) c_s
//        c_t      = beta_t (v_t - S'_t k_t)
//    so the only O(V K) work is ONE pass over S_0 computing 2Q dot products
//    per row (S_0 [k_1..k_Q, q_1..q_Q]); the per-token recurrence is O(Q^2)
//    scalar work per row.  No rank-1 update of the tile is ever materialised
//    and nothing is serialised behind a cross-lane reduction per token.
//  * Rows map to lanes (RPW rows per warp), the K extent is split KSPLIT ways
//    across lane groups and reduced with warp shuffles; the 2Q key/query
//    vectors live in shared memory and are read as warp-uniform broadcasts.
//
// Invalid tokens (t >= qlen or token index out of range) contribute decay 1,
// beta 0 and zero q/k: they change nothing and store nothing, exactly like the
// reference's masked `tl.where(valid, new_state, state)` (kernels.py:653).
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace gdn_rssm {

struct VerifyParams {
  const void *q, *k, *v;
  const float *g;
  const void *beta;
  float *corr;
  void *key;
  float *decay;
  void *out;
  const void *qsl, *indices;
  int32_t *status;  // device status word of this translation unit
  int64_t rows, tokens, heads, value_heads, query_len, blocks, record_rows, null_block;
  int64_t q_ts, k_ts, v_ts, g_ts, beta_ts;
  int64_t corr_rs, corr_hs, corr_ts;
  int64_t key_rs, key_hs, key_ts;
  int64_t decay_rs, decay_hs, decay_ts;
  int64_t out_ts, qsl_stride, index_stride;
  float scale;
  int32_t beta_dtype, key_dtype, qsl_dtype, index_dtype;
  uint32_t flags;
};

template <int DIM, int QT, typename St>
struct VerifyShape {
  static constexpr int kThreads = kVerifyThreads;
  static constexpr int KSPLIT = kThreads / DIM;         // lane groups splitting K
  static constexpr int RPW = 32 / KSPLIT;               // rows per warp
  static constexpr int KC = DIM / KSPLIT;               // K elements per lane group
  static constexpr int EPC = 16 / sizeof(St);           // state elements per 16-B chunk
  static constexpr int BOXW = 128 / sizeof(St);         // state elements per swizzled box row
  static constexpr int NBOX = DIM / BOXW;               // boxes per tile
  static constexpr int LDX = DIM + 4 * KSPLIT;          // padded X row (floats)
  static constexpr int TILE_BYTES = DIM * DIM * sizeof(St);
  static constexpr int X_BYTES = 2 * QT * LDX * 4;
  static constexpr int NPAIR = QT * QT;                 // Gram pairs (k.k s<t, k.q s<=t)
  static_assert(DIM % BOXW == 0, "state tile must be whole swizzle boxes");
  static_assert(KC % EPC == 0, "lane group K range must be whole chunks");
  static_assert(KSPLIT * RPW == 32, "lane layout");
};

template <int QT>
struct VerifySmall {
  uint64_t bar;
  float dec[QT];    // decay of token t (1 for invalid tokens)
  float beta[QT];   // beta of token t (0 for invalid tokens)
  float A[QT];      // prod_{s<=t} dec[s]
  float mkk[QT][QT];  // D[t][s] * (k_s . k_t), s < t
  float mkq[QT][QT];  // D[t][s] * (k_s . q_t), s <= t
  int32_t valid[QT];
  int32_t tok[QT];
};

template <int DIM, int QT, typename St>
constexpr int verify_smem_bytes() {
  using Sh = VerifyShape<DIM, QT, St>;
  return 1024 /* alignment slack */ + Sh::TILE_BYTES + Sh::X_BYTES + static_cast<int>(sizeof(VerifySmall<QT>));
}

__device__ __forceinline__ int64_t load_typed_index(const void *p, int64_t i, int32_t dtype) {
  return dtype == GDN_RSSM_I64 ? static_cast<const int64_t *>(p)[i]
                               : static_cast<int64_t>(static_cast<const int32_t *>(p)[i]);
}

__device__ __forceinline__ void store_key(void *p, int64_t i, float x, int32_t dtype) {
  switch (dtype) {
    case GDN_RSSM_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(x); break;
    case GDN_RSSM_F16: static_cast<__half *>(p)[i] = __float2half_rn(x); break;
    default: static_cast<float *>(p)[i] = x; break;
  }
}

// Three CTAs per SM keep ~3 state tiles in flight; the Q = 8 variant trades one
// resident CTA for registers (its 2Q accumulators would otherwise spill).
template <int QT>
constexpr int verify_min_blocks() {
  return QT >= 8 ? 2 : 3;
}

template <int DIM, int QT, typename Act, typename St>
__global__ void __launch_bounds__(kVerifyThreads, verify_min_blocks<QT>())
    verify_kernel(const __grid_constant__ CUtensorMap state_map, const VerifyParams p) {
  using Sh = VerifyShape<DIM, QT, St>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char *tile = smem;
  float *X = reinterpret_cast<float *>(smem + Sh::TILE_BYTES);
  VerifySmall<QT> &sm = *reinterpret_cast<VerifySmall<QT> *>(smem + Sh::TILE_BYTES + Sh::X_BYTES);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int64_t HV = p.value_heads;
  const int64_t row = blockIdx.x / HV;
  const int hv = static_cast<int>(blockIdx.x % HV);
  const int ratio = static_cast<int>(HV / p.heads);
  const int h = hv / ratio;

  const int64_t bos = load_typed_index(p.qsl, row * p.qsl_stride, p.qsl_dtype);
  const int64_t eos = load_typed_index(p.qsl, (row + 1) * p.qsl_stride, p.qsl_dtype);
  const int64_t qlen = eos - bos;
  const int64_t slot = load_typed_index(p.indices, row * p.index_stride, p.index_dtype);
  const int Q = static_cast<int>(p.query_len);

  // ---- null / out-of-pool slot: zero output for the row's window ---------- //
  if (slot <= p.null_block || slot >= p.blocks) {
    Act *out = static_cast<Act *>(p.out);
    for (int i = tid; i < QT * DIM; i += kVerifyThreads) {
      const int t = i / DIM, e = i % DIM;
      const int64_t tok = bos + t;
      if (t < Q && t < qlen && tok >= 0 && tok < p.tokens) out[tok * p.out_ts + hv * DIM + e] = from_f32<Act>(0.f);
    }
    return;
  }

  // ---- issue the TMA tile load first so it overlaps all the set-up -------- //
  if (tid == 0) {
    ptx::prefetch_tensormap(&state_map);
    ptx::mbar_init(&sm.bar, 1);
    ptx::fence_mbar_init();
    ptx::mbar_arrive_expect_tx(&sm.bar, Sh::TILE_BYTES);
#pragma unroll
    for (int b = 0; b < Sh::NBOX; ++b) {
      ptx::tma_load_4d(tile + b * DIM * 128, &state_map, &sm.bar, b * Sh::BOXW, 0, hv, static_cast<int32_t>(slot));
    }
  }
  // ---- per-token scalars ---------------------------------------------------- //
  if (tid < QT) {
    const int t = tid;
    const int64_t tok = bos + t;
    const bool valid = t < Q && t < qlen && tok >= 0 && tok < p.tokens;
    sm.valid[t] = valid;
    sm.tok[t] = valid ? static_cast<int32_t>(tok) : 0;
    sm.dec[t] = valid ? expf(p.g[tok * p.g_ts + hv]) : 1.f;
    sm.beta[t] = valid ? load_float(p.beta, tok * p.beta_ts + hv, p.beta_dtype) : 0.f;
  }
  __syncthreads();

  // ---- stage k_hat and q_tilde (fp32) into X, optional in-kernel L2 ------- //
  const bool normalize = (p.flags & GDN_RSSM_NORMALIZE_QK) != 0;
  for (int j = warp; j < 2 * QT; j += kVerifyThreads / 32) {
    const int t = j % QT;
    const bool is_q = j >= QT;
    float x[DIM / 32];
    const bool valid = sm.valid[t];
    const Act *src = static_cast<const Act *>(is_q ? p.q : p.k);
    const int64_t base = static_cast<int64_t>(sm.tok[t]) * (is_q ? p.q_ts : p.k_ts) + static_cast<int64_t>(h) * DIM;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < DIM / 32; ++i) {
      x[i] = valid ? to_f32<Act>(src[base + lane + 32 * i]) : 0.f;
      ss = fmaf(x[i], x[i], ss);
    }
    float mul = 1.f;
    if (normalize) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      mul = rsqrtf(ss + 1e-6f);
    }
#pragma unroll
    for (int i = 0; i < DIM / 32; ++i) {
      const int e = lane + 32 * i;
      float val = normalize ? x[i] * mul : x[i];
      if (is_q) val *= p.scale;
      X[j * Sh::LDX + (e / Sh::KC) * (Sh::KC + 4) + (e % Sh::KC)] = val;
    }
  }
  __syncthreads();

  // ---- Gram coefficients: one pair per warp iteration ---------------------- //
  for (int pr = warp; pr < Sh::NPAIR; pr += kVerifyThreads / 32) {
    // pairs [0, QT(QT-1)/2): k_s.k_t (s<t); then QT(QT+1)/2 pairs k_s.q_t (s<=t)
    int s, t, kind;
    {
      int idx = pr;
      kind = 0;
      const int nkk = QT * (QT - 1) / 2;
      if (idx >= nkk) {
        kind = 1;
        idx -= nkk;
      }
      // decode lower-triangular index
      t = 0;
      int lim = kind == 0 ? 0 : 1;  // number of s for t=0
      while (idx >= lim + t) {
        idx -= lim + t;
        ++t;
      }
      s = idx;
    }
    const float *a = X + s * Sh::LDX;
    const float *b = X + (kind == 0 ? t : QT + t) * Sh::LDX;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < DIM / 32; ++i) {
      const int e = lane + 32 * i;
      const int xi = (e / Sh::KC) * (Sh::KC + 4) + (e % Sh::KC);
      acc = fmaf(a[xi], b[xi], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      float dprod = 1.f;
      for (int r = s + 1; r <= t; ++r) dprod *= sm.dec[r];
      if (kind == 0) {
        sm.mkk[t][s] = dprod * acc;
      } else {
        sm.mkq[t][s] = dprod * acc;
      }
    }
  }
  if (tid == 0) {
    float a = 1.f;
#pragma unroll
    for (int t = 0; t < QT; ++t) {
      a *= sm.dec[t];
      sm.A[t] = a;
    }
  }

  // ---- records: key and decay (independent of the state) ------------------ //
  const bool rec_ok = row < p.record_rows;
  const bool packed = (p.flags & GDN_RSSM_RECORD_PACKED) != 0;
  if (rec_ok) {
    if (tid < QT && sm.valid[tid]) {
      p.decay[row * p.decay_rs + hv * p.decay_hs + tid * p.decay_ts] = sm.dec[tid];
    }
    if (packed || hv % ratio == 0) {
      const int64_t kh = packed ? hv : h;
      for (int i = tid; i < QT * DIM; i += kVerifyThreads) {
        const int t = i / DIM, e = i % DIM;
        if (!sm.valid[t]) continue;
        const float val = X[t * Sh::LDX + (e / Sh::KC) * (Sh::KC + 4) + (e % Sh::KC)];
        store_key(p.key, row * p.key_rs + kh * p.key_hs + t * p.key_ts + e, val, packed ? GDN_RSSM_F32 : p.key_dtype);
      }
    }
  }

  // ---- row ownership: r = warp*RPW + lane%RPW, K split ks = lane/RPW ------- //
  const int r = warp * Sh::RPW + (lane % Sh::RPW);
  const int ks = lane / Sh::RPW;
  __syncthreads();  // Gram coefficients visible

  // ---- wait for the tile ----------------------------------------------------- //
  if (!ptx::mbar_wait_bounded(&sm.bar, 0, 1000000000ull)) {
    if (tid == 0) atomicExch(p.status, kStatusTmaTimeout);
    ptx::mbar_wait_bounded(&sm.bar, 0, 1000000000ull);  // let an in-flight copy land before exiting
    return;
  }

  // ---- one pass over S_0: acc[j] = sum_k S[r][k] X[j][k] over this lane's K range //
  float acc[2 * QT];
#pragma unroll
  for (int j = 0; j < 2 * QT; ++j) acc[j] = 0.f;
  const unsigned char *trow = tile + r * 128;
  const float *xk = X + ks * (Sh::KC + 4);
#pragma unroll 4
  for (int cc = 0; cc < Sh::KC / Sh::EPC; ++cc) {
    const int k0 = ks * Sh::KC + cc * Sh::EPC;  // first element of this chunk
    const int box = k0 / Sh::BOXW;
    const int c = (k0 % Sh::BOXW) / Sh::EPC;
    const uint4 raw = *reinterpret_cast<const uint4 *>(trow + box * DIM * 128 + ((c ^ (r & 7)) << 4));
    float s[Sh::EPC];
    if constexpr (sizeof(St) == 4) {
      s[0] = __uint_as_float(raw.x);
      s[1] = __uint_as_float(raw.y);
      s[2] = __uint_as_float(raw.z);
      s[3] = __uint_as_float(raw.w);
    } else {
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s[2 * i] = __uint_as_float(w[i] << 16);
        s[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
    const float *xc = xk + cc * Sh::EPC;
#pragma unroll
    for (int j = 0; j < 2 * QT; ++j) {
#pragma unroll
      for (int e4 = 0; e4 < Sh::EPC; e4 += 4) {
        const float4 x4 = *reinterpret_cast<const float4 *>(xc + j * Sh::LDX + e4);
        acc[j] = fmaf(s[e4 + 0], x4.x, acc[j]);
        acc[j] = fmaf(s[e4 + 1], x4.y, acc[j]);
        acc[j] = fmaf(s[e4 + 2], x4.z, acc[j]);
        acc[j] = fmaf(s[e4 + 3], x4.w, acc[j]);
      }
    }
  }
  // reduce the KSPLIT partial sums (lanes l, l^RPW, l^2RPW, ...)
#pragma unroll
  for (int o = Sh::RPW; o < 32; o <<= 1) {
#pragma unroll
    for (int j = 0; j < 2 * QT; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  }
  if (ks != 0) return;

  // ---- per-row recurrence over the window ---------------------------------- //
  Act *out = static_cast<Act *>(p.out);
  const Act *vin = static_cast<const Act *>(p.v);
  float vv[QT];
#pragma unroll
  for (int t = 0; t < QT; ++t) vv[t] = sm.valid[t] ? to_f32<Act>(vin[static_cast<int64_t>(sm.tok[t]) * p.v_ts + hv * DIM + r]) : 0.f;
  float cr[QT];
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    cr[t] = 0.f;
    if (!sm.valid[t]) continue;
    float kv = sm.A[t] * acc[t];
#pragma unroll
    for (int s = 0; s < t; ++s) kv = fmaf(sm.mkk[t][s], cr[s], kv);
    cr[t] = sm.beta[t] * (vv[t] - kv);
    float o = sm.A[t] * acc[QT + t];
#pragma unroll
    for (int s = 0; s <= t; ++s) o = fmaf(sm.mkq[t][s], cr[s], o);
    const int64_t tok = sm.tok[t];
    out[tok * p.out_ts + hv * DIM + r] = from_f32<Act>(o);
    if (rec_ok) p.corr[row * p.corr_rs + hv * p.corr_hs + t * p.corr_ts + r] = cr[t];
  }
}

}  // namespace gdn_rssm
