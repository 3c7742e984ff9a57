// Commit-plan, align-publication and conv-compaction kernels (integer /
// byte work, bit-exact with the reference).
//
//  * commit_plan_kernel  <- _prepare_commit_plan_kernel (kernels.py:936-1072)
//  * grouped_plan_kernel <- _grouped_plan_kernel (grouped_commit.py:31-222)
//  * publish_align_kernel <- _publish_grouped_align_kernel (grouped_commit.py:531-560)
//  * compact_conv_kernel <- _grouped_compact_conv_state_kernel
//    (grouped_commit.py:225-322) / _compact_conv_state_kernel
//    (kernels.py:1075-1169)
//
// One thread per plan row (the reference launches one single-warp program per
// row).  Every table read is bounds-checked against the lengths the host
// passes: a row whose request index falls outside `sampled`, the block table
// or `num_computed` becomes an invalid (no-op) row instead of an out-of-bounds
// read.
#pragma once

#include "params.cuh"
#include "ptx.cuh"

namespace gdn_rssm {

// Longest conv history compacted (kernel width - 1; the Gated DeltaNet family
// uses width 4, history 3).
constexpr int kMaxConvHistory = 8;
constexpr int kConvThreads = 256;
constexpr int kConvChannelsPerCta = 1024;  // largest chunk
constexpr int kConvSmemLimit = 48 * 1024;  // staging of the contiguous path: 3 chunks
constexpr uint64_t kConvWaitLimitNs = 1000000000ull;  // 1 s


// 32-bit two's-complement arithmetic of the per-context plan: the reference
// kernel loads the accepted and computed counts as int32 and does the align
// arithmetic in int32 (kernels.py:978-1035), so sums past 2^31 wrap there and
// must wrap here too.  Done on uint32 to keep the wrap defined in C++.
__device__ __forceinline__ int32_t add_wrap32(int32_t a, int32_t b) {
  return static_cast<int32_t>(static_cast<uint32_t>(a) + static_cast<uint32_t>(b));
}
__device__ __forceinline__ int32_t mul_wrap32(int32_t a, int32_t b) {
  return static_cast<int32_t>(static_cast<uint32_t>(a) * static_cast<uint32_t>(b));
}

// One plan row: what the conv compaction and the fold of that row do, in the
// form the plan arrays store it (invalid rows: length 0, null pages).
struct RowPlan {
  int64_t source;  // the page folded from (grouped plans store it masked)
  int64_t request;
  int32_t length, final_page, boundary, boundary_len, valid, col;
};

// Per-context plan of row r (_prepare_commit_plan_kernel, kernels.py:936-1072).
__device__ __forceinline__ RowPlan context_row_plan(const CommitPlanParams &p, int64_t r) {
  const int64_t nul = p.null_block;
  const int64_t source = load_index(p.state, r);
  const int64_t req = p.request.data ? load_index(p.request, r) : r;
  bool row_ok = true;
  const int32_t acc = static_cast<int32_t>(load_index_checked(p.accepted, req, row_ok));
  const int64_t bos = load_index(p.qsl, r), eos = load_index(p.qsl, r + 1);
  const int32_t qlen = static_cast<int32_t>(eos - bos);
  int32_t n = acc > 0 ? acc : 0;
  n = n < qlen ? n : qlen;
  n = n < p.Q ? n : static_cast<int32_t>(p.Q);
  int64_t fin = source, boundary = nul;
  int32_t blen = 0, colv = 0, c = 0;
  const bool align = p.table.data != nullptr;
  if (align) {
    // a request without a computed count or a block-table row makes the row
    // invalid and its align arithmetic start from zero (the stored column too)
    bool have = true;
    c = static_cast<int32_t>(load_index_checked(p.computed, req, have));
    if (!have || req < 0 || req >= p.table.rows) {
      row_ok = false;
      c = 0;
    }
    const int32_t W = static_cast<int32_t>(p.table.cols), B = static_cast<int32_t>(p.block_size);  // B >= 1
    const int32_t end = add_wrap32(c, n);
    const int32_t last = add_wrap32(end, -1);
    colv = (last > 0 ? last : 0) / B;
    colv = colv < W - 1 ? colv : W - 1;
    fin = row_ok ? load_table(p.table, req, colv) : nul;
    // c >= 0 on every row whose outputs are kept, where / is floor division
    const int32_t nxt = mul_wrap32(add_wrap32(c / B, 1), B);
    const bool crosses = end >= nxt;
    blen = add_wrap32(nxt, -c);
    const int32_t bcol = nxt / B - 1;
    boundary = (row_ok && crosses && bcol >= 0 && bcol < W) ? load_table(p.table, req, bcol) : nul;
  }
  const bool geometry = bos >= 0 && bos <= eos && qlen <= p.Q;
  bool valid = row_ok && source > nul && source < p.num_blocks && fin > nul && fin < p.num_blocks && geometry && n > 0 &&
               n <= qlen;
  if (align) {
    valid = valid && c >= 0;
    if (!(boundary > nul && boundary < p.num_blocks)) blen = 0;
  }
  RowPlan out;
  out.source = source;
  out.request = req;
  out.length = valid ? n : 0;
  out.final_page = static_cast<int32_t>(valid ? fin : nul);
  out.boundary = static_cast<int32_t>(valid ? boundary : nul);
  out.boundary_len = valid ? blen : 0;
  out.valid = valid ? 1 : 0;
  out.col = colv;
  return out;
}

__device__ __forceinline__ void store_context_plan(const CommitPlanParams &p, int64_t r, const RowPlan &pl) {
  p.lens[r] = pl.length;
  p.finals[r] = pl.final_page;
  p.boundaries[r] = pl.boundary;
  p.boundary_lens[r] = pl.boundary_len;
  p.valid[r] = pl.valid;
  p.col[r] = pl.col;
}

__global__ void commit_plan_kernel(const CommitPlanParams p) {
  // launched as a programmatic dependent of the kernel before it (the sampler
  // in serving, verify in a bench step): wait for it before reading its
  // results, then let the fold start launching (it waits for this grid)
  ptx::wait_prerequisite_grid();
  ptx::launch_dependents();
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (r >= p.rows) return;
  store_context_plan(p, r, context_row_plan(p, r));
}

// Grouped plan of (group gi, row) (_grouped_plan_kernel, grouped_commit.py:31-222):
// the source is stored masked, and a group-local invalid boundary becomes
// null before the bucket-wide pool bound of the fold could make it valid.
__device__ __forceinline__ RowPlan group_row_plan(const GroupedPlanParams &p, int gi, int64_t row) {
  const int64_t nul = p.null_block;
  const gdn_rssm_plan_group &g = p.groups[gi];
  const int64_t req = load_index(g.request_indices, row);
  const int64_t source = load_index(g.state_indices, row);
  const int64_t bos = load_index(g.query_start_loc, row), eos = load_index(g.query_start_loc, row + 1);
  const int64_t qlen = eos - bos;
  bool row_ok = true;
  const int64_t acc = static_cast<int32_t>(load_index_checked(p.sampled, req, row_ok));
  int64_t n = acc > 0 ? acc : 0;
  n = n < qlen ? n : qlen;
  n = n < p.Q ? n : p.Q;
  int64_t fin = source, boundary = nul, blen = 0, colv = 0;
  bool computed_ok = true;
  if (p.align) {
    bool have = true;  // as in context_row_plan: no computed count or table row -> invalid, from zero
    int64_t c = load_index_checked(g.num_computed, req, have);
    if (!have || req < 0 || req >= g.block_table.rows) {
      row_ok = false;
      c = 0;
    }
    computed_ok = c >= 0;
    const int64_t B = g.block_size, W = g.block_table.cols;
    const int64_t pos = c + n;
    colv = floordiv(pos - 1 > 0 ? pos - 1 : 0, B);
    colv = colv < W - 1 ? colv : W - 1;
    fin = row_ok ? load_table(g.block_table, req, colv) : nul;
    const int64_t nxt = (floordiv(c, B) + 1) * B;
    const bool crossed = pos >= nxt;
    blen = static_cast<int32_t>(nxt - c);
    const int64_t bcol = floordiv(nxt, B) - 1;
    boundary = (row_ok && crossed && computed_ok && bcol >= 0 && bcol < W) ? load_table(g.block_table, req, bcol) : nul;
  }
  const bool geometry = bos >= 0 && bos <= eos && qlen <= p.Q;
  const bool valid = row_ok && geometry && source > nul && source < g.num_blocks && fin > nul && fin < g.num_blocks &&
                     n > 0 && n <= qlen && computed_ok;
  if (!(boundary > nul && boundary < g.num_blocks)) {
    blen = 0;
    boundary = nul;
  }
  RowPlan out;
  out.source = valid ? source : nul;
  out.request = req;
  out.length = valid ? static_cast<int32_t>(n) : 0;
  out.final_page = static_cast<int32_t>(valid ? fin : nul);
  out.boundary = static_cast<int32_t>(valid ? boundary : nul);
  out.boundary_len = valid ? static_cast<int32_t>(blen) : 0;
  out.valid = valid ? 1 : 0;
  out.col = static_cast<int32_t>(colv);
  return out;
}

__device__ __forceinline__ void store_group_plan(const GroupedPlanParams &p, int gi, int64_t row, const RowPlan &pl) {
  const int64_t off = gi * p.capacity + row;
  p.source[off] = static_cast<int32_t>(pl.source);
  p.length[off] = pl.length;
  p.finals[off] = pl.final_page;
  p.boundaries[off] = pl.boundary;
  p.boundary_lens[off] = pl.boundary_len;
  p.valid[off] = pl.valid;
  p.col[off] = pl.col;
}

// Every group's plan of one row, stored, then (align + publish) the row's
// publication: when all groups are valid and agree on column and request,
// persistent_cols[slot] = col and persistent_accepted[slot] = 1 with
// slot = idx_mapping[request] (grouped_commit.py:214-222).
__device__ __forceinline__ void grouped_plan_row(const GroupedPlanParams &p, int64_t row) {
  bool all_valid = true;
  int64_t shared_col = -1, shared_req = -1;
  for (int gi = 0; gi < p.num_groups; ++gi) {
    const RowPlan pl = group_row_plan(p, gi, row);
    store_group_plan(p, gi, row, pl);
    if (gi == 0) {
      shared_col = pl.col;
      shared_req = pl.request;
    } else {
      all_valid = all_valid && pl.col == shared_col && pl.request == shared_req;
    }
    all_valid = all_valid && pl.valid;
  }
  if (p.align && p.publish) {
    bool ok = true;
    const int64_t slot = load_index_checked(p.idx_mapping, shared_req, ok, -1);
    if (all_valid && ok && slot >= 0 && slot < p.cols_out.length && slot < p.accepted_out.length) {
      store_index(p.cols_out, slot, shared_col);
      store_index(p.accepted_out, slot, 1);
    }
  }
}

__global__ void grouped_plan_kernel(const GroupedPlanParams p) {
  ptx::wait_prerequisite_grid();  // as in commit_plan_kernel
  ptx::launch_dependents();
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (row >= p.rows) return;
  grouped_plan_row(p, row);
}


__global__ void publish_align_kernel(const PublishParams p) {
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (row >= p.rows) return;
  const int32_t *first_cols = reinterpret_cast<const int32_t *>(p.descriptors[1]);
  const int32_t shared = first_cols[row];
  bool ok = true;
  for (int b = 0; b < p.num_buckets; ++b) {
    const int64_t *d = p.descriptors + 4 * b;
    const int32_t *valid = reinterpret_cast<const int32_t *>(d[0]);
    const int32_t *col = reinterpret_cast<const int32_t *>(d[1]);
    const int64_t cap = d[2];
    const int64_t groups = d[3];
    for (int64_t gi = 0; gi < groups; ++gi) {
      const int64_t off = gi * cap + row;
      ok = ok && valid[off] != 0 && col[off] == shared;
    }
  }
  const int64_t req = load_index(p.request, row);
  bool in_range = true;
  const int64_t slot = load_index_checked(p.idx_mapping, req, in_range, -1);
  if (ok && in_range && slot >= 0 && slot < p.cols_out.length && slot < p.accepted_out.length) {
    store_index(p.cols_out, slot, shared);
    store_index(p.accepted_out, slot, 1);
  }
}


// One CTA per (layer, row); threads stride over the [conv_dim, history] window.
// Both windows are read into registers before either is stored (the final or
// the boundary page may alias the source page).
// dst[h] = src[from + h] for h < hist (element stride ts), ascending: safe in
// place (dst == src) because every read (from + h >= h) is at or ahead of
// the writes already done.
template <typename E>
__device__ __forceinline__ void shift_window(E *dst, const E *src, int64_t from, int hist, int64_t ts) {
#pragma unroll 1
  for (int h = 0; h < hist; ++h) dst[h * ts] = src[(from + h) * ts];
}

// The history windows of one channel: boundary snapshot (when do_b) and final
// window, both taken from the source rows as they were before either store.
// A target that aliases the source is written last (ascending, in place); a
// boundary on the final page is overwritten by the final window, so it is not
// written at all.
template <typename E>
__device__ __forceinline__ void compact_channel(E *fin_row, E *bnd_row, const E *src_row, int32_t n, int32_t blen,
                                                bool do_b, bool bnd_is_src, bool bnd_is_fin, int hist, int64_t ts) {
  if (do_b && bnd_is_src && !bnd_is_fin) {
    shift_window(fin_row, src_row, n - 1, hist, ts);
    shift_window(bnd_row, src_row, blen - 1, hist, ts);
  } else {
    if (do_b && !bnd_is_fin) shift_window(bnd_row, src_row, blen - 1, hist, ts);
    shift_window(fin_row, src_row, n - 1, hist, ts);
  }
}

template <typename E>
__global__ void __launch_bounds__(kConvThreads, 4) compact_conv_kernel(const ConvParams p) {
  ptx::wait_prerequisite_grid();  // launched as a dependent of the plan: its results first
  ptx::launch_dependents();       // the fold may start launching (it waits for this grid)
  const int64_t row = blockIdx.x % p.rows;
  const int64_t layer = blockIdx.x / p.rows;
  const int64_t prow = static_cast<int64_t>(p.layer_groups[layer]) * p.capacity + row;
  if (prow < 0 || prow >= p.plan_len) return;
  bool ok = true;
  const int64_t src = load_index_checked(p.source, prow, ok);
  const int32_t n = p.lengths[prow];
  const int64_t fin = p.finals[prow];
  // n < 1 or a window reaching past the conv state would read outside the
  // page: such a row is skipped (the plan never produces one).
  if (!ok || src <= p.null_block || src >= p.num_blocks || n < 1 || n - 1 + p.history > p.window ||
      fin <= p.null_block || fin >= p.num_blocks)
    return;
  const int64_t bidx = p.boundaries[prow];
  const int32_t blen = p.boundary_lens[prow];
  const bool do_b = p.align && bidx > p.null_block && bidx < p.num_blocks && blen >= 1 && blen - 1 + p.history <= p.window;
  E *base = reinterpret_cast<E *>(p.addrs[layer]);
  const int64_t bs = p.block_strides[layer], ds = p.dim_strides[layer], ts = p.token_strides[layer];
  const E *srcp = base + src * bs;
  E *finp = base + fin * bs;
  E *bndp = base + (do_b ? bidx : 0) * bs;
  const int hist = static_cast<int>(p.history);  // <= kMaxConvHistory (checked on the host)
  const int64_t d0 = static_cast<int64_t>(blockIdx.y) * p.chunk;
  const int64_t nch = p.conv_dim - d0 < p.chunk ? p.conv_dim - d0 : p.chunk;
  if (nch <= 0) return;
  const bool bnd_is_src = do_b && bidx == src;
  const bool bnd_is_fin = do_b && bidx == fin;  // the final window overwrites it: not stored separately
  const int64_t W = p.window;
  const uint32_t bytes = static_cast<uint32_t>(nch * W * static_cast<int64_t>(sizeof(E)));
  const bool aligned = ((reinterpret_cast<uintptr_t>(srcp + d0 * W) | reinterpret_cast<uintptr_t>(finp + d0 * W) |
                         reinterpret_cast<uintptr_t>(bndp + d0 * W) | bytes) & 15) == 0;
  if (p.vec && ts == 1 && ds == W && aligned) {
    // Contiguous windows: the chunk's rows of each distinct page (source,
    // final, boundary) come into shared memory with one bulk copy each, the
    // history windows move there, and the final / boundary chunks go back
    // with one bulk store each -- full-sector traffic and a few instructions
    // per CTA.  A page that is the source (in place, or a boundary aliasing
    // the source) is read once.  Every read lands before any store.
    extern __shared__ __align__(16) unsigned char conv_smem[];
    __shared__ uint64_t bar;
    E *sA = reinterpret_cast<E *>(conv_smem);
    E *sB = sA + static_cast<int64_t>(p.chunk) * W;
    E *sC = sB + static_cast<int64_t>(p.chunk) * W;
    const bool fin_is_src = fin == src;
    E *t_fin = fin_is_src ? sA : sB;
    E *t_bnd = bnd_is_src ? sA : sC;
    const int tid = threadIdx.x;
    if (tid == 0) {
      const uint32_t loads = 1 + (fin_is_src ? 0 : 1) + (do_b && !bnd_is_src && !bnd_is_fin ? 1 : 0);
      ptx::mbar_init(&bar, 1);
      ptx::fence_mbar_init();
      ptx::mbar_arrive_expect_tx(&bar, loads * bytes);
      ptx::bulk_load(sA, srcp + d0 * W, bytes, &bar);
      if (!fin_is_src) ptx::bulk_load(sB, finp + d0 * W, bytes, &bar);
      if (do_b && !bnd_is_src && !bnd_is_fin) ptx::bulk_load(sC, bndp + d0 * W, bytes, &bar);
    }
    __syncthreads();  // barrier initialised
    if (!ptx::mbar_wait_bounded(&bar, 0, kConvWaitLimitNs)) {
      if (tid == 0) atomicExch(p.status, kStatusTmaTimeout);
      ptx::mbar_wait_bounded(&bar, 0, kConvWaitLimitNs);  // let an in-flight copy land before exiting
      return;
    }
    const int w = static_cast<int>(W), nc = static_cast<int>(nch);
    for (int c = tid; c < nc; c += kConvThreads)
      compact_channel(t_fin + c * w, t_bnd + c * w, sA + c * w, n, blen, do_b, bnd_is_src, bnd_is_fin, hist, 1);
    ptx::fence_proxy_async_smem();  // the composed rows -> the bulk stores' reads
    __syncthreads();
    if (tid == 0) {
      if (do_b && !bnd_is_fin) ptx::bulk_store(bndp + d0 * W, t_bnd, bytes);
      ptx::bulk_store(finp + d0 * W, t_fin, bytes);
      ptx::bulk_commit();
      ptx::bulk_wait_read();  // shared memory stays valid until the stores have read it
    }
    return;
  }
  // General strides: one thread per channel; no two threads touch the same
  // channel, so an in-place row (final or boundary == source) needs no barrier.
#pragma unroll 1
  for (int64_t d = d0 + threadIdx.x; d < d0 + nch; d += blockDim.x)
    compact_channel(finp + d * ds, bndp + d * ds, srcp + d * ds, n, blen, do_b, bnd_is_src, bnd_is_fin, hist, ts);
}

}  // namespace gdn_rssm
