// Speculative verify kernel (sm_100a), CUDA-core form: K = V in {32, 64}, or
// a bf16 state pool (K = V = 128 with an fp32 pool runs verify_tc.cuh).
//
// Semantics follow the reference verify (kernels.py:491-697; AscendC
// verify.h:350-398): per (sequence row, value head) "unit", read the fp32
// checkpoint S[V,K] read-only, run the gated delta rule over the Q draft
// tokens, write the attention output per token and one record per token
// [corr(V), k_hat(K), decay].
//
// Math.  The Q-step recurrence is evaluated in its chunked form.  With
// A_t = prod_{s<=t} d_s and D[t][s] = prod_{s<r<=t} d_r,
//     S'_t k_t = A_t (S_0 k_t) + sum_{s<t}  D[t][s] (k_s . k_t) c_s
//     S_t q_t  = A_t (S_0 q_t) + sum_{s<=t} D[t][s] (k_s . q_t) c_s
//     c_t      = beta_t (v_t - S'_t k_t),      o_t = S_t q_t
// so the only O(V K) work is one pass over S_0 computing 2Q dot products per
// state row; the per-token recurrence is O(Q^2) scalar work per row.
//
// B200 design: one CTA (256 threads, 8 warps) per unit, two or three resident
// per SM so that several 64 KiB tiles are in flight per SM.
//  * Thread 0 starts the TMA tile load of S_0 first (4-D tensor map over the
//    [blocks, HV, V, K] pool, 128-byte swizzle, one box per 128 bytes of K).
//  * While it flies, the warps stage the window: q/k/v/g/beta are loaded in
//    one memory round trip, q/k optionally L2-normalised, written to shared
//    memory as fp32 X rows (k_hat then q_tilde, in the tile's chunk order), the
//    key/decay records are written, and the Gram dot products k_s.k_t,
//    k_s.q_t plus the decay coefficients are computed (one pair per warp).
//  * One register-blocked pass over the swizzled tile: each thread owns
//    R = K/32 rows and 1/8 of K; the 8 K-groups of a quarter warp read one
//    contiguous 128-byte segment of the tile and of X (no bank conflicts) and
//    each X chunk feeds R rows.  A lane-group reduce-scatter gathers each row's
//    2Q sums, then the per-row recurrence writes the output and correction.
// Two CTA barriers in all, both before the tile is needed; the tile wait is
// bounded.
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
  const void *g;     // log-space decay g, or the raw gate input a (kGateInKernel)
  const void *beta;  // beta, or the raw input b (kGateInKernel)
  const float *A_log, *dt_bias;  // [HV] (kGateInKernel)
  float softplus_beta, softplus_threshold;
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
  int32_t gate_dtype, beta_dtype, key_dtype, qsl_dtype, index_dtype;
  uint32_t flags;
};

// Internal flag (set by gdn_rssm_verify_gated): the g / beta slots hold the
// raw gate inputs a / b, and the kernel computes the gates.
constexpr uint32_t kGateInKernel = 1u << 8;

// Decay exp(g) and beta of value head hv from the two values loaded from the
// g and beta slots.  Gated: g = -exp(A_log) * softplus(a + dt_bias) with
// softplus(x) = log1p(exp(sb x)) / sb below the threshold and x above it,
// beta = sigmoid(b).  a_log / dt_bias are the head's A_log and dt_bias
// (read only when gated).
__device__ __forceinline__ void gate_math(const VerifyParams &p, float a_log, float dt_bias, float a, float b,
                                          float &dec, float &bet) {
  const float x = a + dt_bias;
  const float bx = p.softplus_beta * x;
  const float sp = bx <= p.softplus_threshold ? log1pf(expf(bx)) / p.softplus_beta : x;
  dec = expf(-expf(a_log) * sp);
  bet = 1.f / (1.f + expf(-b));
}

__device__ __forceinline__ void token_gates(const VerifyParams &p, float a_log, float dt_bias, float graw,
                                            float braw, float &dec, float &bet) {
  if (p.flags & kGateInKernel) {
    gate_math(p, a_log, dt_bias, graw, braw, dec, bet);
  } else {
    dec = expf(graw);
    bet = braw;
  }
}

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

// Matvec form: 1 = packed f32x2 FMAs over (even, odd) K pairs, 0 = scalar FMAs.
#ifndef GDN_RSSM_VERIFY_PACKED_FMA
#define GDN_RSSM_VERIFY_PACKED_FMA 0
#endif

template <int DIM, int QT, typename Act, typename St>
struct VerifyShape {
  static constexpr int NJ = 2 * QT;              // dot products per state row
  static constexpr int EPC = 16 / sizeof(St);    // state elements per 16-byte chunk
  static constexpr int BOXW = 128 / sizeof(St);  // state elements per swizzled box row
  static constexpr int NBOX = DIM / BOXW;        // boxes (= chunks per K-group) per row
  static constexpr int R = DIM / 32;             // rows per consumer thread
  static constexpr int EPL = DIM / 32;           // K elements per prep lane
  static constexpr int NP = QT * QT;             // Gram pairs (k.k s<t, then k.q s<=t)
  static constexpr int V = R * NJ;               // partial sums per consumer thread
  static constexpr int TILE = DIM * DIM * sizeof(St);
  static constexpr int NQ = DIM / 32;          // 32-row quarters of the tile, one mbarrier each
  struct Small {
    uint64_t bar[NQ];
    float A[QT];
    float beta[QT];
    float dec[QT];
    float mkk[QT][QT];  // D[t][s] * (k_s . k_t), s < t
    float mkq[QT][QT];  // D[t][s] * (k_s . q_t), s <= t
  };
  static constexpr int X_BYTES = NJ * DIM * 4;
  static constexpr int V_BYTES = (QT * DIM * static_cast<int>(sizeof(Act)) + 15) / 16 * 16;
  static constexpr int SMEM = 1024 /* alignment slack */ + TILE + X_BYTES + V_BYTES + static_cast<int>(sizeof(Small));
  static_assert(DIM % BOXW == 0, "state tile must be whole swizzle boxes");
  static_assert(R >= 1 && R <= 4, "rows per thread");
};

template <int DIM, int QT, typename Act, typename St>
constexpr int verify_smem_bytes() {
  return VerifyShape<DIM, QT, Act, St>::SMEM;
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

// Position of K element e inside an X row: the tile's 16-byte chunk order, so
// that the 8 K-groups of a quarter warp read 128 contiguous bytes of X
// (identity for fp32 tiles).
template <int BOXW, int EPC>
__device__ __forceinline__ int x_pos(int e) {
  const int m = e / BOXW, kg = (e % BOXW) / EPC, w = e % EPC;
  return m * BOXW + (w / 4) * 32 + kg * 4 + (w % 4);
}

// Packed pair FMA (fma.rn.f32x2, sm_100): acc.lo += s.lo * x.lo and
// acc.hi += s.hi * x.hi, each rounded like fmaf.
__device__ __forceinline__ unsigned long long ffma2(unsigned long long s, unsigned long long x,
                                                    unsigned long long acc) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(s), "l"(x), "l"(acc));
  return d;
}

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}

// Sums NV per-lane values over the lanes that differ in the bits HI, HI/2,
// ..., 1 of the lane index.  While more than one value is left, a level keeps
// half of them (lanes with the bit set keep the upper half) and adds the
// partner's copy; once one value is left the remaining levels all-reduce it.
// With NV >= 2^levels, the lane whose selected bits read b holds the sums of
// indices [b * NV / 2^levels, (b + 1) * NV / 2^levels).
template <int NV, int HI>
__device__ __forceinline__ void reduce_scatter(float *a, int lane) {
  if constexpr (HI >= 1) {
    if constexpr (NV >= 2) {
      constexpr int half = NV / 2;
      const bool upper = (lane & HI) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? a[i] : a[i + half];
        const float keep = upper ? a[i + half] : a[i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, HI);
      }
      reduce_scatter<half, HI / 2>(a, lane);
    } else {
      a[0] += __shfl_xor_sync(0xffffffffu, a[0], HI);
      reduce_scatter<1, HI / 2>(a, lane);
    }
  }
}

// Resident CTAs per SM: three while the window is short, two at Q = 8 (its 2Q
// accumulators per row need the registers and the larger X the shared memory).
template <int QT>
constexpr int verify_min_blocks() {
  return (QT >= 8 || GDN_RSSM_VERIFY_PACKED_FMA) ? 2 : 3;
}

template <int DIM, int QT, typename Act, typename St>
__global__ void __launch_bounds__(kVerifyThreads, verify_min_blocks<QT>())
    verify_kernel(const __grid_constant__ CUtensorMap state_map, const VerifyParams p) {
  ptx::launch_dependents();  // a commit plan behind it may launch; it waits for this grid
  using Sh = VerifyShape<DIM, QT, Act, St>;
  using Small = typename Sh::Small;
  constexpr int NJ = Sh::NJ, EPC = Sh::EPC, BOXW = Sh::BOXW, R = Sh::R, EPL = Sh::EPL, V = Sh::V;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char *tile = smem;
  float(*X)[DIM] = reinterpret_cast<float(*)[DIM]>(smem + Sh::TILE);
  Act(*vs)[DIM] = reinterpret_cast<Act(*)[DIM]>(smem + Sh::TILE + Sh::X_BYTES);
  Small &sm = *reinterpret_cast<Small *>(smem + Sh::TILE + Sh::X_BYTES + Sh::V_BYTES);

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

  // ---- start the tile load first so it overlaps all of the set-up --------- //
  if (tid == 0) {
    ptx::prefetch_tensormap(&state_map);
#pragma unroll
    for (int qt = 0; qt < Sh::NQ; ++qt) ptx::mbar_init(&sm.bar[qt], 1);
    ptx::fence_mbar_init();
    // quarter by quarter, so the first rows can be folded while the rest fly
#pragma unroll
    for (int qt = 0; qt < Sh::NQ; ++qt) {
      ptx::mbar_arrive_expect_tx(&sm.bar[qt], Sh::NBOX * 32 * 128);
#pragma unroll
      for (int m = 0; m < Sh::NBOX; ++m) {
        ptx::tma_load_4d(tile + m * DIM * 128 + qt * 32 * 128, &state_map, &sm.bar[qt], m * BOXW, qt * 32, hv,
                         static_cast<int32_t>(slot));
      }
    }
  }

  // ---- stage the window ------------------------------------------------------ //
  const bool normalize = (p.flags & GDN_RSSM_NORMALIZE_QK) != 0;
  const bool packed = (p.flags & GDN_RSSM_RECORD_PACKED) != 0;
  const bool rec_ok = row < p.record_rows;
  {
    // q/k rows: warp w owns vectors w, w + 8, ... (k_t for j < QT, q_t after)
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
    // v rows (raw activation values) and per-token scalars
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
      const bool gated = (p.flags & kGateInKernel) != 0;
      token_gates(p, gated ? p.A_log[hv] : 0.f, gated ? p.dt_bias[hv] : 0.f,
                  load_float(p.g, (bos + tid) * p.g_ts + hv, p.gate_dtype),
                  load_float(p.beta, (bos + tid) * p.beta_ts + hv, p.beta_dtype), dec, bet);
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
#pragma unroll
      for (int u = 0; u < EPL; ++u) X[j][x_pos<BOXW, EPC>(lane * EPL + u)] = x[c][u];
    }
  }
  __syncthreads();  // X, v, dec, beta staged; barrier initialised

  // ---- Gram coefficients: one pair per warp iteration ---------------------- //
  {
    constexpr int NKK = QT * (QT - 1) / 2;
    for (int pr = warp; pr < Sh::NP; pr += 8) {
      const int kind = pr >= NKK ? 1 : 0;
      int rem = kind ? pr - NKK : pr, t = 0;
      while (rem >= (kind ? t + 1 : t)) {
        rem -= kind ? t + 1 : t;
        ++t;
      }
      const int s2 = rem;
      const float *a = X[s2];
      const float *b = X[kind ? QT + t : t];
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < EPL; ++u) acc = fmaf(a[lane + 32 * u], b[lane + 32 * u], acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        float d = 1.f;
        for (int r2 = s2 + 1; r2 <= t; ++r2) d *= sm.dec[r2];
        if (kind == 0) {
          sm.mkk[t][s2] = d * acc;
        } else {
          sm.mkq[t][s2] = d * acc;
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
  }
  __syncthreads();  // coefficients visible

  // ---- wait for this warp's 32-row quarter of the tile ---------------------- //
  {
    const int qt = (warp * 4 * R) / 32;
    if (!ptx::mbar_wait_bounded(&sm.bar[qt], 0, kWaitLimitNs)) {
      if (lane == 0) atomicExch(p.status, kStatusTmaTimeout);
      ptx::mbar_wait_bounded(&sm.bar[qt], 0, kWaitLimitNs);  // let an in-flight copy land before exiting
      return;
    }
  }

  // ---- one pass over S_0: thread = R rows x 1/8 of K --------------------------- //
  const int kg = lane & 7;                  // K-group: chunk kg of every box
  const int r0 = (warp * 4 + (lane >> 3)) * R;  // first row of this thread
  float acc[V];
#if GDN_RSSM_VERIFY_PACKED_FMA
  // accumulators hold (even-k, odd-k) partial sums as packed f32 pairs
  unsigned long long acc2[R][NJ];
#pragma unroll
  for (int a = 0; a < R; ++a)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc2[a][j] = 0ull;
#pragma unroll
  for (int m = 0; m < Sh::NBOX; ++m) {
    unsigned long long sp[R][EPC / 2];
#pragma unroll
    for (int a = 0; a < R; ++a) {
      const int r = r0 + a;
      const uint4 raw = *reinterpret_cast<const uint4 *>(tile + m * DIM * 128 + r * 128 + ((kg ^ (r & 7)) << 4));
      if constexpr (sizeof(St) == 4) {
        sp[a][0] = (static_cast<unsigned long long>(raw.y) << 32) | raw.x;
        sp[a][1] = (static_cast<unsigned long long>(raw.w) << 32) | raw.z;
      } else {
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) sp[a][u] = pack2(__uint_as_float(w4[u] << 16), __uint_as_float(w4[u] & 0xffff0000u));
      }
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) {
        const ulonglong2 xx = *reinterpret_cast<const ulonglong2 *>(&X[j][m * BOXW + e4 * 32 + kg * 4]);
#pragma unroll
        for (int a = 0; a < R; ++a) {
          acc2[a][j] = ffma2(sp[a][e4 * 2 + 0], xx.x, acc2[a][j]);
          acc2[a][j] = ffma2(sp[a][e4 * 2 + 1], xx.y, acc2[a][j]);
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < R; ++a)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      acc[a * NJ + j] = __uint_as_float(static_cast<uint32_t>(acc2[a][j])) +
                        __uint_as_float(static_cast<uint32_t>(acc2[a][j] >> 32));
#else
#pragma unroll
  for (int a = 0; a < V; ++a) acc[a] = 0.f;
#pragma unroll
  for (int m = 0; m < Sh::NBOX; ++m) {
    float sv[R][EPC];
#pragma unroll
    for (int a = 0; a < R; ++a) {
      const int r = r0 + a;
      const uint4 raw = *reinterpret_cast<const uint4 *>(tile + m * DIM * 128 + r * 128 + ((kg ^ (r & 7)) << 4));
      if constexpr (sizeof(St) == 4) {
        sv[a][0] = __uint_as_float(raw.x);
        sv[a][1] = __uint_as_float(raw.y);
        sv[a][2] = __uint_as_float(raw.z);
        sv[a][3] = __uint_as_float(raw.w);
      } else {
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sv[a][2 * u] = __uint_as_float(w4[u] << 16);
          sv[a][2 * u + 1] = __uint_as_float(w4[u] & 0xffff0000u);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) {
        const float4 x4 = *reinterpret_cast<const float4 *>(&X[j][m * BOXW + e4 * 32 + kg * 4]);
#pragma unroll
        for (int a = 0; a < R; ++a) {
          float &ac = acc[a * NJ + j];
          ac = fmaf(sv[a][e4 * 4 + 0], x4.x, ac);
          ac = fmaf(sv[a][e4 * 4 + 1], x4.y, ac);
          ac = fmaf(sv[a][e4 * 4 + 2], x4.z, ac);
          ac = fmaf(sv[a][e4 * 4 + 3], x4.w, ac);
        }
      }
    }
  }
#endif
  // ---- reduce the 8 K-groups and gather each row's 2Q sums ----------------- //
  constexpr bool SCATTER = V >= 8;              // else a plain all-reduce
  constexpr int C = SCATTER ? V / 8 : V;        // values held after the scatter
  constexpr int LPR = SCATTER ? NJ / C : 1;     // lanes sharing one row (= 8 / R)
  float pr[NJ];
  int my_row;
  bool writer_out, writer_corr;
  if constexpr (SCATTER) {
    reduce_scatter<V, 4>(acc, lane);
    // lane kg now holds flat indices [kg*C, kg*C + C): row kg*C/NJ, j from (kg*C)%NJ
    my_row = (kg * C) / NJ;
    if constexpr (LPR == 2) {
      // even lanes hold the row's k-dots (j < Q), odd lanes its q-dots: swap halves
      const bool even = (kg & 1) == 0;
#pragma unroll
      for (int j = 0; j < C; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, acc[j], 1);
        pr[j] = even ? acc[j] : other;
        pr[C + j] = even ? other : acc[j];
      }
    } else {
      const int jbase = (kg * C) % NJ;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        float v = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c)
          if (j == jbase + c) v = acc[c];
        pr[j] = v;
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) {
#pragma unroll
        for (int j = 0; j < NJ; ++j) pr[j] += __shfl_xor_sync(0xffffffffu, pr[j], o);
      }
    }
    writer_out = (kg % LPR) == LPR - 1;
    writer_corr = (kg % LPR) == 0;
  } else {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
#pragma unroll
      for (int a = 0; a < V; ++a) acc[a] += __shfl_xor_sync(0xffffffffu, acc[a], o);
    }
    my_row = kg < R ? kg : 0;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      float v = 0.f;
#pragma unroll
      for (int a = 0; a < R; ++a)
        if (a == my_row) v = acc[a * NJ + j];
      pr[j] = v;
    }
    writer_out = writer_corr = kg < R;
  }
  // ---- per-row recurrence over the window ------------------------------------ //
  const int r = r0 + my_row;
  float cr[QT];
#pragma unroll
  for (int t = 0; t < QT; ++t) {
    cr[t] = 0.f;
    if (!((valid_mask >> t) & 1)) continue;
    float kv = sm.A[t] * pr[t];
#pragma unroll
    for (int s2 = 0; s2 < t; ++s2) kv = fmaf(sm.mkk[t][s2], cr[s2], kv);
    cr[t] = sm.beta[t] * (to_f32<Act>(vs[t][r]) - kv);
    float o = sm.A[t] * pr[QT + t];
#pragma unroll
    for (int s2 = 0; s2 <= t; ++s2) o = fmaf(sm.mkq[t][s2], cr[s2], o);
    const int64_t tok = bos + t;
    if (writer_out) out[tok * p.out_ts + hv * DIM + r] = from_f32<Act>(o);
    if (writer_corr && rec_ok) p.corr[row * p.corr_rs + hv * p.corr_hs + t * p.corr_ts + r] = cr[t];
  }
}

}  // namespace gdn_rssm
