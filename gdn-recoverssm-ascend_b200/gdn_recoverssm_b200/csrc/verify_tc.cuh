// Tensor-core verify kernel for K = V = 128 with an fp32 state pool (sm_100a).
//
// Same semantics and the same chunked form of the Q-step recurrence as
// verify_kernel (verify.cuh): the only O(V K) work is P = S_0 X^T, the 2Q dot
// products of every state row with the window's k_hat / q_tilde vectors.  Here
// that product runs on the 5th-generation tensor cores (tcgen05.mma,
// kind::tf32, M = 128 state rows, accumulators in tensor memory).
//
// fp32 accuracy from tf32 / bf16 operands (split products): every operand x
// is written as x = hi(x) + lo(x) with hi(x) = x with its low 13 mantissa
// bits cleared (exactly a tf32 value) and lo(x) = x - hi(x) (exact in fp32).
//   pass 1 (16 x kind::tf32, A = the TMA-loaded tile, which the tensor core
//          reads as tf32 by dropping the same 13 bits, i.e. hi(S); B = the
//          rows [hi(X); lo(X)] padded to a multiple of 16) gives hi(S) hi(X)
//          and hi(S) lo(X) side by side in tensor memory;
//   pass 2 (8 x kind::f16, A = bf16(lo(S)) written by the threads into tensor
//          memory, B = bf16(X)) adds lo(S) X in its own columns.
// Column j + column 2Q + j of pass 1 plus column j of pass 2 is the row's j-th
// dot product; the dropped terms are below 2^-19 relative.  With exact
// operands (lo(X) = 0) pass 1 holds hi(S) X alone and pass 2 accumulates onto
// those columns, so column j is the dot product.
//
// Grid: up to three CTAs (256 threads) per SM (two at Q = 8), each walking the
// units blockIdx.x, blockIdx.x + gridDim.x, ...; per unit:
//   all:      stage [hi(X); lo(X)], decay / beta and the decay and key
//             records (the unit's q/k/v/g/beta were loaded into registers
//             during the previous unit -- at Q = 8 with exact operands its
//             q/k/v rows into shared memory by cp.async); wait for the tile;
//   thread 0: pass 1, no commit yet;
//   all:      meanwhile bf16(lo(S)) -> tensor memory (one row per lane),
//             bf16(X) -> the pass-2 operand; warps 4-7 the Gram partial
//             sums; the loads of the next unit's activations, and one
//             thread's cp.async of the row metadata of the unit after it into
//             shared memory; with the fused gating prologue, warp 1 computes
//             decay / beta from the raw inputs here;
//   thread 0: pass 2 right behind pass 1, one commit for both;
//   warps 4+: Gram coefficients (warp 0, which issues the MMAs, takes no
//             part in the Gram); the metadata thread decodes its copy (token
//             mask, slot, key head) for everyone to read after the barrier;
//             after the commit, thread 0 starts the NEXT
//             unit's tile (4-D tensor map, 128-byte swizzle -- the layout
//             the MMA's K-major descriptor reads directly -- one 128-row box
//             per K slab) into the freed buffer, and every warp loads its 32
//             rows' sums from tensor memory (one row per lane) and runs the
//             recurrence (all window tokens, no mask test: a masked token's
//             correction is a signed zero) -- warps 0-3 write the correction
//             records, warps 4-7 the outputs, stores masked -- while that
//             load is in flight.
// Three CTA barriers per unit; the per-unit scalars are double-buffered by
// unit parity.  Every wait is bounded (1 s) and reported through the status
// word; tensor memory is released on every path after it was allocated.
#pragma once

#include <type_traits>

#include "verify.cuh"

namespace gdn_rssm {

// (row, value head) of a CTA's units, advanced by gridDim.x units without a
// 64-bit division per step.
struct TcCursor {
  int32_t row;
  int32_t hv;
  __device__ __forceinline__ void advance(int32_t dq, int32_t dr, int32_t HV) {
    row += dq;
    hv += dr;
    if (hv >= HV) {
      hv -= HV;
      row += 1;
    }
  }
};

// A unit's row metadata, reduced to 32-bit fields when it is loaded (the host
// keeps rows, tokens and blocks below 2^31): the token mask holds the window's
// masking (t < Q, t < qlen, 0 <= bos + t < tokens), so bos only addresses valid
// tokens and always fits; slot is -1 for a null or out-of-pool page.  Small
// fields matter here: every register the walk keeps across units counts
// against the 80 that three resident CTAs leave per thread.
struct TcUnitMeta {
  int32_t bos, slot;
  int32_t vk;       // token mask (bits 0-7) | the key head the value head reads << 8
  int32_t row, hv;  // the unit
  __device__ __forceinline__ int vmask() const { return vk & 0xff; }
  __device__ __forceinline__ int kh() const { return vk >> 8; }
};

// EXACT: the window's vectors are exact tf32 values (bf16 / fp16 inputs used as
// they are, no in-kernel normalisation, q unscaled), so lo(X) = 0 and the
// pass-1 operand holds X alone; the output is scaled after the dot products.
template <int QT, typename Act, bool EXACT>
struct VerifyTcShape {
  static constexpr int DIM = 128;
  static constexpr int NJ = 2 * QT;                    // dot products per state row
  static constexpr int XROWS = EXACT ? NJ : 2 * NJ;    // pass-1 B rows with data: X, or hi(X) and lo(X)
  static constexpr int NB = (XROWS + 15) / 16 * 16;    // ... padded with zero rows to the MMA's N
  static constexpr int TMEM_COLS = 128;
  static constexpr uint32_t D_COL = 0;                 // pass-1 accumulator: NB columns
  static constexpr uint32_t D2_COL = 32;               // pass-2 accumulator: 16 columns (split operands)
  static constexpr int NLD = NJ <= 8 ? 8 : 16;         // accumulator columns read back (exact operands)
  static constexpr uint32_t A_LO = 64;                 // bf16 lo(S): 64 columns of packed pairs
  static constexpr int NB2 = 16;                       // pass-2 N (minimum for M = 128)
  static constexpr int G2 = (NJ + 7) / 8;              // 8-row groups of bf16(X) that hold data
  static constexpr int SLAB = DIM * 128;               // one 32-column K slab of the tile (bytes)
  static constexpr int TILE = DIM * DIM * 4;
  static constexpr int B2_SLAB = G2 * 1024;            // one 64-element K slab of the pass-2 operand
  static constexpr int B2_BYTES = 2 * B2_SLAB;
  static constexpr int B_SLAB = NB * 128;
  static constexpr int B_BYTES = 4 * B_SLAB;
  // Q = 8 (two CTAs per SM leave shared memory to spare): X in fp32, row j at
  // j * 512 bytes, for the Gram on every warp (gram_all_warps)
  static constexpr bool GRAM_ALL = QT >= 8;
  static constexpr int X32_BYTES = GRAM_ALL ? NJ * DIM * 4 : 0;
  // Q = 8 with exact (2-byte) operands: the next unit's q / k / v rows come
  // into shared memory by cp.async (two buffers, by unit parity) instead of
  // registers -- the 8-token walk is at the 128 registers two CTAs leave.
  // The host selects this form only for 16-byte aligned activation rows.
  static constexpr bool SIN = EXACT && QT >= 8;
  static constexpr int IN_X = NJ * DIM * static_cast<int>(sizeof(Act));  // one unit's [k; q] rows
  static constexpr int IN_V = QT * DIM * static_cast<int>(sizeof(Act));  // one unit's v rows
  static constexpr int IN_BYTES = SIN ? 2 * (IN_X + IN_V) : 0;
  struct Window {  // per-unit scalars
    float A[QT];
    float beta[QT];
    float dec[QT];
    float mkk[QT][QT];  // D[t][s] * (k_s . k_t), s < t
    float mkq[QT][QT];  // D[t][s] * (k_s . q_t), s <= t
  };
  struct Small {
    uint64_t tile_bar;
    uint64_t mma_bar;
    // bos, eos, slot of the unit two ahead, as copied (cp.async), by the
    // parity of the walk step that copied them, and the same decoded by the
    // copying thread once its copy has landed (read by everyone after the
    // next CTA barrier): a slow warp still reading step i's entry never races
    // the copy that step i + 1 starts before any barrier
    uint64_t meta_raw[2][3];
    TcUnitMeta meta[2];
    TcCursor cur2;  // (row, value head) of the unit two ahead (Q <= 4): that thread's alone
    uint32_t tmem;
    float gpart[4][QT * QT];  // Gram partial sums per K slab
    Window win[2];
  };
  // tile | pass-2 operand | pass-1 operand | fp32 X (Q = 8) | scalars; the
  // dynamic shared memory base is 1024-byte aligned (checked at run time), as
  // the 128-byte swizzle atoms require
  static constexpr int SMEM = TILE + B2_BYTES + B_BYTES + X32_BYTES + IN_BYTES + static_cast<int>(sizeof(Small));
  static_assert(NB <= static_cast<int>(D2_COL) && (NB == 16 || NB == 32), "accumulator columns");
  static_assert(!EXACT || !std::is_same<Act, float>::value, "fp32 activations are not exact tf32 values");
  static_assert(NJ <= NB2, "pass-2 operand rows");
  static_assert(!GRAM_ALL || QT * QT * 4 == kVerifyThreads, "gram_all_warps: four threads per Gram pair");
  static_assert(B_SLAB % 1024 == 0 && B2_SLAB % 1024 == 0, "operand slabs must stay 1024-byte aligned");
};

// Resident CTAs per SM: three up to Q = 4 (74 KB of shared memory each), two
// at Q = 8.
template <int QT>
constexpr int verify_tc_min_blocks() {
  return QT >= 8 ? 2 : 3;
}

// Shared memory of one SM (228 KB) and what the runtime reserves per CTA.
constexpr int kSmemPerSm = 233472;
constexpr int kSmemReservedPerCta = 1024;

template <int QT, typename Act, bool EXACT>
constexpr int verify_tc_smem_bytes() {
  static_assert(verify_tc_min_blocks<QT>() * (VerifyTcShape<QT, Act, EXACT>::SMEM + kSmemReservedPerCta) <=
                    kSmemPerSm,
                "the verify CTAs of one SM must fit its shared memory");
  return VerifyTcShape<QT, Act, EXACT>::SMEM;
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

// Gram coefficients of the window, in two steps.
//
// gram_partials: called by four warps; warp g covers K slab g of the B operand
// ([hi(X); lo(X)], rows 128 bytes apart in 4 K slabs of B_SLAB bytes, 16-byte
// chunk c of row n at chunk c ^ (n % 8)) and lane l its element 32 g + l.
// Every lane forms x_j = hi + lo (exact) for the 2Q vectors -- one
// conflict-free read of the operand in all -- and all Q^2 pair products, in
// the order: k_s . k_t for t = 1..Q-1, s < t, then k_s . q_t for t = 0..Q-1,
// s <= t.  A reduce-scatter over the warp leaves each pair's slab sum on known
// lanes, which store part[g][pair].
template <int QT, int NJ, int B_SLAB, bool EXACT>
__device__ __forceinline__ void gram_partials(const unsigned char *bop, float (*part)[QT * QT], int g, int lane) {
  constexpr int NP = QT * QT;
  const unsigned char *slab = bop + g * B_SLAB;
  const int chunk = lane >> 2, word = (lane & 3) * 4;
  float x[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const float hi = *reinterpret_cast<const float *>(slab + j * 128 + ((chunk ^ (j & 7)) << 4) + word);
    if constexpr (EXACT) {
      x[j] = hi;
    } else {
      const int jl = NJ + j;
      x[j] = hi + *reinterpret_cast<const float *>(slab + jl * 128 + ((chunk ^ (jl & 7)) << 4) + word);
    }
  }
  float acc[NP];
  int p = 0;
#pragma unroll
  for (int t = 1; t < QT; ++t)
#pragma unroll
    for (int s2 = 0; s2 < t; ++s2) acc[p++] = x[s2] * x[t];
#pragma unroll
  for (int t = 0; t < QT; ++t)
#pragma unroll
    for (int s2 = 0; s2 <= t; ++s2) acc[p++] = x[s2] * x[QT + t];
  reduce_scatter<NP, 16>(acc, lane);
  if constexpr (NP >= 32) {
    constexpr int PER = NP / 32;  // lane holds pairs lane * PER .. + PER - 1
#pragma unroll
    for (int i = 0; i < PER; ++i) part[g][lane * PER + i] = acc[i];
  } else {
    constexpr int SPAN = 32 / NP;  // lanes sharing one pair's sum
    if (lane % SPAN == 0) part[g][lane / SPAN] = acc[0];
  }
}

// gram_all_warps (Q = 8: Q^2 = 64 pairs x 4 K quarters = 256 threads): thread
// 4 pr + sq sums pair pr's products over K elements 32 sq .. 32 sq + 31 from
// the fp32 copy of X (rows `pair` = a | b << 8, 512 bytes apart), two lane
// shuffles add the four quarters, and lane sq = 0 stores part[0][pr].  The
// eight lanes of a quarter-warp start at eight different 16-byte chunks (the
// chunk order is rotated by 2 sq + pr % 2), so the 128-bit reads are free of
// bank conflicts.  No reduce-scatter: at Q = 8 the one in gram_partials is
// ~4x the instructions, all on warps 4-7.
template <int QT>
__device__ __forceinline__ void gram_all_warps(const float *x32, float (*part)[QT * QT], int pair, int tid) {
  const int pr = tid >> 2, sq = tid & 3;
  const float4 *xa = reinterpret_cast<const float4 *>(x32 + (pair & 0xff) * 128 + sq * 32);
  const float4 *xb = reinterpret_cast<const float4 *>(x32 + (pair >> 8) * 128 + sq * 32);
  const int rot = 2 * sq + (pr & 1);
  float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int cc = (c + rot) & 7;
    const float4 a = xa[cc], b = xb[cc];
    acc0 = fmaf(a.x, b.x, acc0);
    acc1 = fmaf(a.y, b.y, acc1);
    acc0 = fmaf(a.z, b.z, acc0);
    acc1 = fmaf(a.w, b.w, acc1);
  }
  float acc = acc0 + acc1;
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  if (sq == 0) part[0][pr] = acc;
}

// The X rows (a, b) of Gram pair pr, packed a | b << 8, in gram_partials'
// order: k_s . k_t for t = 1..Q-1, s < t, then k_s . q_t for t = 0..Q-1, s <= t.
template <int QT>
__device__ __forceinline__ int gram_pair_rows(int pr) {
  constexpr int NKK = QT * (QT - 1) / 2;
  const int kind = pr >= NKK ? 1 : 0;
  int rem = kind ? pr - NKK : pr, t = kind ? 0 : 1;
  while (rem >= (kind ? t + 1 : t)) {
    rem -= kind ? t + 1 : t;
    ++t;
  }
  return rem | ((kind ? QT + t : t) << 8);
}

// gram_finalize: thread `pr` (< Q^2) sums pair pr over the four slabs (or
// takes the whole sum from slab 0, SUMMED) and scales it by the decay product
// D[t][s] = prod_{s<r<=t} dec[r]:
//     mkk[t][s] = D[t][s] (k_s . k_t)  for s < t,
//     mkq[t][s] = D[t][s] (k_s . q_t)  for s <= t.
template <int QT, bool SUMMED>
__device__ __forceinline__ void gram_finalize(const float (*part)[QT * QT], const float *dec, float (*mkk)[QT],
                                              float (*mkq)[QT], int pr) {
  constexpr int NKK = QT * (QT - 1) / 2;
  const float sum = SUMMED ? part[0][pr] : (part[0][pr] + part[1][pr]) + (part[2][pr] + part[3][pr]);
  const int kind = pr >= NKK ? 1 : 0;
  int rem = kind ? pr - NKK : pr, t = kind ? 0 : 1;
  while (rem >= (kind ? t + 1 : t)) {
    rem -= kind ? t + 1 : t;
    ++t;
  }
  float d = 1.f;
  for (int r2 = rem + 1; r2 <= t; ++r2) d *= dec[r2];
  if (kind == 0) {
    mkk[t][rem] = d * sum;
  } else {
    mkq[t][rem] = d * sum;
  }
}



__device__ __forceinline__ TcUnitMeta tc_unit_meta(int64_t bos, int64_t eos, int64_t slot, int32_t row, int32_t hv,
                                                   int32_t kh, int QT, int64_t Q, int64_t tokens, int64_t null_block,
                                                   int64_t blocks) {
  int mask = 0;
  for (int t = 0; t < QT; ++t) {
    const int64_t tok = bos + t;
    if (t < Q && t < eos - bos && tok >= 0 && tok < tokens) mask |= 1 << t;
  }
  const bool live = slot > null_block && slot < blocks;
  return TcUnitMeta{mask ? static_cast<int32_t>(bos) : 0, live ? static_cast<int32_t>(slot) : -1, mask | (kh << 8), row,
                    hv};
}

// GATED: the fused gating prologue (raw a, b in the g / beta slots).
// EXACT: see VerifyTcShape (bf16 / fp16 activations without in-kernel
// normalisation).
template <int QT, typename Act, bool GATED, bool EXACT>
__global__ void __launch_bounds__(kVerifyThreads, verify_tc_min_blocks<QT>())
    verify_tc_kernel(const __grid_constant__ CUtensorMap state_map, const VerifyParams p) {
  ptx::launch_dependents();  // a commit plan behind it may launch; it waits for this grid
  using Sh = VerifyTcShape<QT, Act, EXACT>;
  using Small = typename Sh::Small;
  using Window = typename Sh::Window;
  constexpr int DIM = Sh::DIM, NJ = Sh::NJ, NB = Sh::NB, EPL = DIM / 32;
  constexpr int PER_WARP = (NJ + 7) / 8;  // q/k vectors staged per warp
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if ((ptx::smem_addr(smem_raw) & 1023u) != 0) {  // swizzle atoms need 1024-byte alignment
    if (threadIdx.x == 0) atomicExch(p.status, kStatusMisaligned);
    return;
  }
  unsigned char *tile = smem_raw;
  unsigned char *b2op = smem_raw + Sh::TILE;  // pass-2 operand: bf16(X)
  unsigned char *bop = b2op + Sh::B2_BYTES;    // pass-1 operand: [hi(X); lo(X)]
  float *x32 = reinterpret_cast<float *>(bop + Sh::B_BYTES);  // fp32 X (Q = 8)
  unsigned char *in_buf = bop + Sh::B_BYTES + Sh::X32_BYTES;  // staged activations (SIN), 2 buffers
  Small &sm = *reinterpret_cast<Small *>(in_buf + Sh::IN_BYTES);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3;
  const int r = qd * 32 + lane;  // state row of this thread in the recurrence
  const int64_t HV = p.value_heads;
  const int64_t units = p.rows * HV;
  const int64_t G = gridDim.x;
  const int ratio = static_cast<int>(HV / p.heads);
  const bool normalize = !EXACT && (p.flags & GDN_RSSM_NORMALIZE_QK) != 0;  // exact operands: never
  const bool packed = (p.flags & GDN_RSSM_RECORD_PACKED) != 0;
  Act *out = static_cast<Act *>(p.out);

  auto load_meta = [&](const TcCursor &c, bool in_range) {
    if (!in_range) return TcUnitMeta{0, -1, 0, 0, 0};
    const int64_t bos = load_typed_index(p.qsl, static_cast<int64_t>(c.row) * p.qsl_stride, p.qsl_dtype);
    const int64_t eos = load_typed_index(p.qsl, static_cast<int64_t>(c.row + 1) * p.qsl_stride, p.qsl_dtype);
    const int64_t slot = load_typed_index(p.indices, static_cast<int64_t>(c.row) * p.index_stride, p.index_dtype);
    return tc_unit_meta(bos, eos, slot, c.row, c.hv, c.hv / ratio, QT, p.query_len, p.tokens, p.null_block,
                        p.blocks);
  };
  auto is_live = [&](const TcUnitMeta &m) { return m.slot >= 0; };
  // The unit two ahead: one thread starts asynchronous copies of its row's raw
  // qsl / slot entries into shared memory (no registers held, no stall) and
  // decodes them, once they have landed, for everyone to read after the next
  // CTA barrier.
  constexpr int kMetaThread = 64;
  auto load_meta_async = [&](uint64_t *raw, const TcCursor &c, bool in_range) {  // thread kMetaThread
    if (!in_range) {
      raw[0] = 0;
      raw[1] = 0;
      raw[2] = ~0ull;  // decodes to slot -1 for either index dtype
      return;
    }
    const int qb = p.qsl_dtype == GDN_RSSM_I64 ? 8 : 4, ib = p.index_dtype == GDN_RSSM_I64 ? 8 : 4;
    const char *qsl = static_cast<const char *>(p.qsl);
    const char *idx = static_cast<const char *>(p.indices);
    ptx::cp_async_small(&raw[0], qsl + static_cast<int64_t>(c.row) * p.qsl_stride * qb, qb);
    ptx::cp_async_small(&raw[1], qsl + static_cast<int64_t>(c.row + 1) * p.qsl_stride * qb, qb);
    ptx::cp_async_small(&raw[2], idx + static_cast<int64_t>(c.row) * p.index_stride * ib, ib);
    ptx::cp_async_commit();
  };
  auto decode_meta = [&](const uint64_t *raw, const TcCursor &c) {  // thread kMetaThread
    auto val = [](uint64_t b, int32_t dt) {
      return dt == GDN_RSSM_I64 ? static_cast<int64_t>(b)
                                : static_cast<int64_t>(static_cast<int32_t>(static_cast<uint32_t>(b)));
    };
    return tc_unit_meta(val(raw[0], p.qsl_dtype), val(raw[1], p.qsl_dtype), val(raw[2], p.index_dtype), c.row, c.hv,
                        c.hv / ratio, QT, p.query_len, p.tokens, p.null_block, p.blocks);
  };
  struct Inputs {  // one unit's activations in registers
    Act x[PER_WARP][EPL];  // q/k: vector warp + 8c, K elements 4 lane .. 4 lane + 3
    Act v[QT];             // v[t][r]
    // g / beta of token t on thread GT + t (t < QT); gated: raw a / b there,
    // and the head's A_log / dt_bias on thread GT + QT
    float g, beta;
  };
  // plain: warp 0 turns g into the decay while staging; gated: warp 1 runs
  // the gating prologue in the pass-1 window, where it has slack
  constexpr int GT = GATED ? 32 : 0;
  // Starts the loads of one unit's activations (nothing for null units); with
  // SIN the q / k / v rows go to shared-memory buffer `b` by cp.async (masked
  // tokens zero-filled) and only g / beta to registers.
  auto load_inputs = [&](Inputs &in, const TcUnitMeta &m, int b) {
    const int vmask = is_live(m) ? m.vmask() : 0;
    const int hv = m.hv;
    const int h = m.kh();
    if constexpr (Sh::SIN) {
      constexpr int CPV = DIM * static_cast<int>(sizeof(Act)) / 16;  // 16-byte chunks per row
      unsigned char *xb = in_buf + b * (Sh::IN_X + Sh::IN_V);
      {
        const int j = tid / CPV, c = tid % CPV;  // NJ x CPV == 256 chunks: one per thread
        const int t = j % QT;
        const bool live = (vmask >> t) & 1;
        const Act *src = static_cast<const Act *>(j >= QT ? p.q : p.k) +
                         (static_cast<int64_t>(m.bos) + t) * (j >= QT ? p.q_ts : p.k_ts) + h * DIM + c * 8;
        ptx::cp_async16_zfill(xb + j * DIM * sizeof(Act) + c * 16, live ? src : p.q, live);
      }
      if (tid < QT * CPV) {
        const int t = tid / CPV, c = tid % CPV;
        const bool live = (vmask >> t) & 1;
        const Act *src = static_cast<const Act *>(p.v) + (static_cast<int64_t>(m.bos) + t) * p.v_ts + hv * DIM + c * 8;
        ptx::cp_async16_zfill(xb + Sh::IN_X + t * DIM * sizeof(Act) + c * 16, live ? src : p.v, live);
      }
      ptx::cp_async_commit();
    } else {
#pragma unroll
    for (int cc = 0; cc < PER_WARP; ++cc) {
      const int j = warp + 8 * cc;
      const int t = j % QT;
      const bool live = j < NJ && ((vmask >> t) & 1);
      const Act *src = static_cast<const Act *>(j >= QT ? p.q : p.k);
      const int64_t base =
          (static_cast<int64_t>(m.bos) + t) * (j >= QT ? p.q_ts : p.k_ts) + static_cast<int64_t>(h) * DIM + lane * EPL;
#pragma unroll
      for (int e = 0; e < EPL; ++e) in.x[cc][e] = live ? src[base + e] : from_f32<Act>(0.f);
    }
    const Act *vrow = static_cast<const Act *>(p.v) + static_cast<int64_t>(m.bos) * p.v_ts + hv * DIM + r;
#pragma unroll
    for (int t = 0; t < QT; ++t) in.v[t] = ((vmask >> t) & 1) ? vrow[t * p.v_ts] : from_f32<Act>(0.f);
    }
    in.g = 0.f;
    in.beta = 0.f;
    const int gt = tid - GT;
    if (gt >= 0 && gt < QT && ((vmask >> gt) & 1)) {
      const int64_t tok = static_cast<int64_t>(m.bos) + gt;
      in.g = load_float(p.g, tok * p.g_ts + hv, p.gate_dtype);
      in.beta = load_float(p.beta, tok * p.beta_ts + hv, p.beta_dtype);
    } else if (GATED && gt == QT && vmask != 0) {
      in.g = p.A_log[hv];  // handed to the token lanes by a shuffle
      in.beta = p.dt_bias[hv];
    }
  };
  auto issue_tile = [&](const TcUnitMeta &m) {  // thread 0
    if (p.flags & GDN_RSSM_VERIFY_TEST_NO_TILE) return;  // failure-detection test: the tile wait runs out
    ptx::mbar_arrive_expect_tx(&sm.tile_bar, Sh::TILE);
#pragma unroll
    for (int mm = 0; mm < 4; ++mm)  // one 128-row box per 32-column K slab
      ptx::tma_load_4d(tile + mm * Sh::SLAB, &state_map, &sm.tile_bar, mm * 32, 0, m.hv, m.slot);
  };

  // ---- walk: metadata of units i and i + 1 in registers; the cursor of unit
  // i + 2 in shared memory, kept by the thread that copies and decodes its
  // metadata ---------------------------------------------------------------- //
  const int32_t HV32 = static_cast<int32_t>(HV);
  const int32_t dq = static_cast<int32_t>(G / HV), dr = static_cast<int32_t>(G % HV);
  TcUnitMeta m0, m1;
  // the cursor two ahead: in shared memory up to Q = 4, where every register
  // counts against the 80 of three resident CTAs; in registers at Q = 8
  TcCursor c2reg{0, 0};
  TcCursor &c2 = QT >= 8 ? c2reg : sm.cur2;
  {
    TcCursor c{static_cast<int32_t>(blockIdx.x / HV32), static_cast<int32_t>(blockIdx.x % HV32)};
    m0 = load_meta(c, true);
    c.advance(dq, dr, HV32);
    m1 = load_meta(c, blockIdx.x + G < units);
    c.advance(dq, dr, HV32);
    if (QT >= 8 || tid == kMetaThread) c2 = c;  // read after the first CTA barrier
  }

  if (tid == 0) {
    ptx::prefetch_tensormap(&state_map);
    ptx::mbar_init(&sm.tile_bar, 1);
    ptx::mbar_init(&sm.mma_bar, 1);
    ptx::fence_mbar_init();
    if (is_live(m0)) issue_tile(m0);
  }
  if (warp == 0) {
    __syncwarp();  // the allocation is warp-wide (.sync.aligned)
    ptx::tmem_alloc(&sm.tmem, Sh::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  // operand rows no unit writes: the zero padding of the pass-1 operand up to
  // the MMA's N, and the rows of the last pass-2 data group past the window
  // (they reach accumulator columns that are never read; zeroed once here)
  if constexpr (NB > Sh::XROWS) {
    constexpr int PAD = (NB - Sh::XROWS) * 8;  // 16-byte chunks per slab
    for (int e = tid; e < 4 * PAD; e += kVerifyThreads) {
      const int mm = e / PAD, rem = e % PAD;
      *reinterpret_cast<uint4 *>(bop + mm * Sh::B_SLAB + (Sh::XROWS + rem / 8) * 128 + ((rem % 8) << 4)) =
          make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if constexpr (8 * Sh::G2 > NJ) {
    constexpr int PAD = (8 * Sh::G2 - NJ) * 8;
    for (int e = tid; e < 2 * PAD; e += kVerifyThreads) {
      const int m = e / PAD, rem = e % PAD;
      *reinterpret_cast<uint4 *>(b2op + m * Sh::B2_SLAB + (NJ + rem / 8) * 128 + ((rem % 8) << 4)) =
          make_uint4(0u, 0u, 0u, 0u);
    }
  }
  const int gpair = Sh::GRAM_ALL ? gram_pair_rows<QT>(tid >> 2) : 0;  // this thread's Gram pair (Q = 8)
  Inputs ic;
  load_inputs(ic, m0, 0);
  if constexpr (Sh::SIN) ptx::cp_async_wait_all();  // unit 0's rows staged before the barrier
  ptx::tc_fence_before_sync();
  __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem = sm.tmem;
  constexpr uint32_t IDESC = ptx::tf32_instr_desc<128, NB>();
  const uint32_t tile_addr = ptx::smem_addr(tile), b_addr = ptx::smem_addr(bop), b2_addr = ptx::smem_addr(b2op);
  uint32_t tile_par = 0, mma_par = 0;
  bool ok = true;

  for (int64_t u = blockIdx.x, i = 0; u < units && ok; u += G, ++i) {
    Inputs in;  // one unit ahead
    auto prefetch = [&]() {
      if (tid == kMetaThread) load_meta_async(sm.meta_raw[i & 1], c2, u + 2 * G < units);  // two units ahead
      load_inputs(in, m1, static_cast<int>((i + 1) & 1));
    };
    const int64_t row = m0.row;
    const int hv = m0.hv;
    const int h = m0.kh();
    const int vmask = m0.vmask();
    const bool rec_ok = row < p.record_rows;
    Window &w = sm.win[i & 1];

    if (!is_live(m0)) {
      // ---- null / out-of-pool slot: zero output, nothing loaded ------------ //
      // staged rows: the previous unit's recurrence may still read the v rows
      // of the buffer this prefetch refills -- a CTA barrier first
      if constexpr (Sh::SIN) __syncthreads();
      prefetch();
      for (int e = tid; e < QT * DIM; e += kVerifyThreads) {
        const int t = e / DIM;
        if ((vmask >> t) & 1)
          out[(static_cast<int64_t>(m0.bos) + t) * p.out_ts + hv * DIM + (e % DIM)] = from_f32<Act>(0.f);
      }
      // the next unit's tile (this unit started none)
      if (tid == 0 && u + G < units && is_live(m1)) issue_tile(m1);
      if (tid == kMetaThread) {
        ptx::cp_async_wait_all();
        sm.meta[i & 1] = decode_meta(sm.meta_raw[i & 1], c2);
      }
      if constexpr (Sh::SIN) ptx::cp_async_wait_all();  // the next unit's rows staged
      __syncthreads();  // the previous unit's recurrence is done with its window buffer; metadata decoded
    } else {
      // ---- stage the window --------------------------------------------------- //
      // decay and beta of the window -> shared memory (read after the next CTA
      // barrier) and the decay records
      auto stage_gates = [&](float a_log, float dt_bias) {
        const int t = tid - GT;
        const bool live = (vmask >> t) & 1;
        float dec = 1.f, bet = 0.f;
        if (live) {
          if constexpr (GATED) {
            gate_math(p, a_log, dt_bias, ic.g, ic.beta, dec, bet);
          } else {
            dec = expf(ic.g);
            bet = ic.beta;
          }
        }
        w.dec[t] = dec;
        w.beta[t] = bet;
        if (rec_ok && live) p.decay[row * p.decay_rs + hv * p.decay_hs + t * p.decay_ts] = dec;
      };
      if constexpr (!GATED) {
        if (tid < QT) stage_gates(0.f, 0.f);
      }
      float xs[PER_WARP][EPL];  // this warp's staged vectors, kept for the pass-2 operand
#pragma unroll
      for (int c = 0; c < PER_WARP; ++c) {
        const int j = warp + 8 * c;
        if (j >= NJ) continue;
        const int t = j % QT;
        float *x = xs[c];
        if constexpr (Sh::SIN) {  // this vector's 4 elements of the staged rows: one 8-byte read
          const uint2 raw = *reinterpret_cast<const uint2 *>(in_buf + (i & 1) * (Sh::IN_X + Sh::IN_V) +
                                                             (j * DIM + lane * EPL) * sizeof(Act));
          const Act *e4 = reinterpret_cast<const Act *>(&raw);
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] = to_f32<Act>(e4[e]);
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] = to_f32<Act>(ic.x[c][e]);
        }
        if (normalize) {
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float mul = rsqrtf(ss + 1e-6f);
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] *= mul;
        }
        if (j < QT) {
          // key record: packed -> every value head keeps its copy; typed -> once per key head
          if (rec_ok && ((vmask >> t) & 1) && (packed || h * ratio == hv)) {
            const int64_t at = row * p.key_rs + (packed ? hv : h) * p.key_hs + t * p.key_ts + lane * EPL;
            const int32_t kd = packed ? GDN_RSSM_F32 : p.key_dtype;  // one dtype switch per vector slice
            if (kd == GDN_RSSM_F32) {
              float *kp = static_cast<float *>(p.key) + at;
#pragma unroll
              for (int e = 0; e < EPL; ++e) kp[e] = x[e];
            } else {
#pragma unroll
              for (int e = 0; e < EPL; ++e) store_key(p.key, at + e, x[e], kd);
            }
          }
        } else if constexpr (!EXACT) {  // exact operands keep q unscaled: the output is scaled instead
#pragma unroll
          for (int e = 0; e < EPL; ++e) x[e] *= p.scale;
        }
        if constexpr (Sh::GRAM_ALL)
          *reinterpret_cast<float4 *>(x32 + j * DIM + lane * EPL) = make_float4(x[0], x[1], x[2], x[3]);
        const int mm = lane >> 3, ch = lane & 7;
        if constexpr (EXACT) {
          *reinterpret_cast<float4 *>(bop + mm * Sh::B_SLAB + j * 128 + ((ch ^ (j & 7)) << 4)) =
              make_float4(x[0], x[1], x[2], x[3]);
        } else {
          float hi[EPL], lo[EPL];
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            hi[e] = tf32_hi(x[e]);
            lo[e] = x[e] - hi[e];
          }
          const int jl = NJ + j;
          *reinterpret_cast<float4 *>(bop + mm * Sh::B_SLAB + j * 128 + ((ch ^ (j & 7)) << 4)) =
              make_float4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<float4 *>(bop + mm * Sh::B_SLAB + jl * 128 + ((ch ^ (jl & 7)) << 4)) =
              make_float4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
      ptx::fence_proxy_async_smem();  // B operand -> tensor-core reads
      // ---- B, dec, beta staged by every thread; the tile has landed ---------- //
      if (__syncthreads_or(!ptx::mbar_wait_bounded(&sm.tile_bar, tile_par, kWaitLimitNs))) {
        if (tid == 0) atomicExch(p.status, kStatusTmaTimeout);
        ptx::mbar_wait_bounded(&sm.tile_bar, tile_par, kWaitLimitNs);  // let an in-flight copy land
        ok = false;
        break;
      }
      tile_par ^= 1u;
      // ---- pass 1: S (read as tf32) x [hi(X); lo(X)] -------------------------- //
      if (tid == 0) {
        ptx::tc_fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < DIM / 8; ++kk) {
          const uint32_t sub = (kk & 3) * 32;  // K sub-block (8 tf32) inside the 128-byte row
          const uint64_t a = ptx::sw128_kmajor_desc(tile_addr + (kk >> 2) * Sh::SLAB + sub);
          const uint64_t b = ptx::sw128_kmajor_desc(b_addr + (kk >> 2) * Sh::B_SLAB + sub);
          ptx::mma_tf32(tmem + Sh::D_COL, a, b, IDESC, kk > 0);
        }
      }
      // ---- while pass 1 runs: bf16 lo(S) -> tensor memory ---------------------- //
      // warp w: rows 32 (w % 4) .. + 31 (one per lane), K elements 64 (w / 4) .. + 63
      {
        const int kh = warp >> 2;
        const unsigned char *row_base = tile + r * 128;
#pragma unroll
        for (int mm = 0; mm < 2; ++mm) {  // one 32-element K slab (16 packed columns) at a time
          const int m = 2 * kh + mm;
          uint32_t packed_lo[16];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 x = *reinterpret_cast<const float4 *>(row_base + m * Sh::SLAB + ((c ^ (r & 7)) << 4));
            const __nv_bfloat162 lo01 = __floats2bfloat162_rn(x.x - tf32_hi(x.x), x.y - tf32_hi(x.y));
            const __nv_bfloat162 lo23 = __floats2bfloat162_rn(x.z - tf32_hi(x.z), x.w - tf32_hi(x.w));
            packed_lo[2 * c] = *reinterpret_cast<const uint32_t *>(&lo01);
            packed_lo[2 * c + 1] = *reinterpret_cast<const uint32_t *>(&lo23);
          }
          __syncwarp();  // tcgen05.st is warp-wide (.sync.aligned)
          ptx::tmem_st16_u(tmem + (static_cast<uint32_t>(qd * 32) << 16) + Sh::A_LO + 32u * kh + 16u * mm, packed_lo);
        }
        ptx::tmem_wait_st();
      }
      if constexpr (GATED) {
        if (warp == 1) {
          const float a_log = __shfl_sync(0xffffffffu, ic.g, QT);  // the head's constants, from lane QT
          const float dt_bias = __shfl_sync(0xffffffffu, ic.beta, QT);
          if (lane < QT) stage_gates(a_log, dt_bias);
        }
      }
      // ---- ... the pass-2 operand bf16(X): G2 8-row groups per 64-element slab ---- //
#pragma unroll
      for (int c = 0; c < PER_WARP; ++c) {
        const int j = warp + 8 * c;
        if (j >= NJ) continue;
        const __nv_bfloat162 b01 = __floats2bfloat162_rn(xs[c][0], xs[c][1]);
        const __nv_bfloat162 b23 = __floats2bfloat162_rn(xs[c][2], xs[c][3]);
        // lane l holds K elements 4l .. 4l + 3: slab l / 16, chunk (l % 16) / 2, half l % 2
        const int m = lane >> 4, ch = (lane & 15) >> 1;
        *reinterpret_cast<uint2 *>(b2op + m * Sh::B2_SLAB + j * 128 + ((ch ^ (j & 7)) << 4) + (lane & 1) * 8) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&b01), *reinterpret_cast<const uint32_t *>(&b23));
      }
      // ---- ... the Gram partial sums and the next units' loads ---------------- //
      if constexpr (Sh::GRAM_ALL) {
        gram_all_warps<QT>(x32, sm.gpart, gpair, tid);
      } else {
        if (warp >= 4) gram_partials<QT, NJ, Sh::B_SLAB, EXACT>(bop, sm.gpart, warp - 4, lane);
      }
      prefetch();
      ptx::fence_proxy_async_smem();  // pass-2 operand -> tensor-core reads
      ptx::tc_fence_before_sync();
      __syncthreads();  // lo(S) in tensor memory, bf16(X) staged, Gram partials written
      // ---- pass 2 right behind pass 1: bf16 lo(S) x bf16(X) into its own columns -- //
      // N = 16: rows past the G2 data groups are read from the following bytes of
      // shared memory (the next slab or the pass-1 operand) and only reach
      // accumulator columns that are never read.
      if (tid == 0) {
        ptx::tc_fence_after_sync();
        constexpr uint32_t IDESC2 = ptx::bf16_instr_desc<128, Sh::NB2>();
#pragma unroll
        for (int kk = 0; kk < DIM / 16; ++kk) {
          const uint64_t b = ptx::sw128_kmajor_desc(b2_addr + (kk >> 2) * Sh::B2_SLAB + (kk & 3) * 32);
          // exact operands: onto pass 1's sums (in issue order); split: own columns
          if constexpr (EXACT)
            ptx::mma_bf16_ts(tmem + Sh::D_COL, tmem + Sh::A_LO + kk * 8, b, IDESC2, true);
          else
            ptx::mma_bf16_ts(tmem + Sh::D2_COL, tmem + Sh::A_LO + kk * 8, b, IDESC2, kk > 0);
        }
        ptx::mma_commit(&sm.mma_bar);
      }
      // ---- Gram coefficients and decay products (off warp 0, which issues) ---- //
      if (tid >= 128 && tid < 128 + QT * QT) gram_finalize<QT, Sh::GRAM_ALL>(sm.gpart, w.dec, w.mkk, w.mkq, tid - 128);
      if (tid == 224) {
        float a = 1.f;
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          a *= w.dec[t];
          w.A[t] = a;
        }
      }
      if (tid == kMetaThread) {  // the copies started a phase ago: decoded once, for everyone
        ptx::cp_async_wait_all();
        sm.meta[i & 1] = decode_meta(sm.meta_raw[i & 1], c2);
      }
      if constexpr (Sh::SIN) ptx::cp_async_wait_all();  // the next unit's rows, staged a phase ago
      if (__syncthreads_or(!ptx::mbar_wait_bounded(&sm.mma_bar, mma_par, kWaitLimitNs))) {
        if (tid == 0) atomicExch(p.status, kStatusMmaTimeout);
        ptx::mbar_wait_bounded(&sm.mma_bar, mma_par, kWaitLimitNs);
        ok = false;
        break;
      }
      mma_par ^= 1u;
      // ---- both passes done, the tile is free: start the next unit's load ---- //
      if (tid == 0 && u + G < units && is_live(m1)) issue_tile(m1);
      // ---- per-row recurrence: lane = state row of the warp's lane quadrant --- //
      ptx::tc_fence_after_sync();
      float d[NB], d2[16];
      __syncwarp();  // tcgen05.ld is warp-wide (.sync.aligned)
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(qd * 32) << 16);
      if constexpr (EXACT) {
        ptx::tmem_ld_sync<Sh::NLD>(lane_base + Sh::D_COL, d);  // the data columns only
      } else {
        ptx::tmem_ld_sync<NB>(lane_base + Sh::D_COL, d);
        ptx::tmem_ld_sync<16>(lane_base + Sh::D2_COL, d2);
      }
      ptx::tc_fence_before_sync();
      // The chain runs over every token without a mask test: a masked token
      // has beta = 0 and zero k / v rows (so zero Gram terms), its
      // correction comes out as a signed zero and adds nothing to the later
      // tokens -- the live tokens' arithmetic is unchanged.  Only the stores
      // test the mask.
      float cr[QT];
#pragma unroll
      for (int t = 0; t < QT; ++t) {
        float kv = w.A[t] * (EXACT ? d[t] : (d[t] + d[NJ + t]) + d2[t]);
#pragma unroll
        for (int s2 = 0; s2 < t; ++s2) kv = fmaf(w.mkk[t][s2], cr[s2], kv);
        float vt;
        if constexpr (Sh::SIN)
          vt = to_f32<Act>(reinterpret_cast<const Act *>(in_buf + (i & 1) * (Sh::IN_X + Sh::IN_V) + Sh::IN_X)[t * DIM + r]);
        else
          vt = to_f32<Act>(ic.v[t]);
        cr[t] = w.beta[t] * (vt - kv);
      }
      if (warp < 4) {  // correction records
        if (rec_ok) {
          float *cp = p.corr + row * p.corr_rs + hv * p.corr_hs + r;
#pragma unroll
          for (int t = 0; t < QT; ++t)
            if ((vmask >> t) & 1) cp[t * p.corr_ts] = cr[t];
        }
      } else {  // outputs
        Act *op = out + static_cast<int64_t>(m0.bos) * p.out_ts + hv * DIM + r;
#pragma unroll
        for (int t = 0; t < QT; ++t) {
          if (!((vmask >> t) & 1)) continue;
          float o = w.A[t] * (EXACT ? d[QT + t] : (d[QT + t] + d[NJ + QT + t]) + d2[QT + t]);
#pragma unroll
          for (int s2 = 0; s2 <= t; ++s2) o = fmaf(w.mkq[t][s2], cr[s2], o);
          if constexpr (EXACT) o *= p.scale;
          op[t * p.out_ts] = from_f32<Act>(o);
        }
      }
    }
    ic = in;
    m0 = m1;
    m1 = sm.meta[i & 1];  // decoded before the last CTA barrier
    if (QT >= 8 || tid == kMetaThread) c2.advance(dq, dr, HV32);
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
