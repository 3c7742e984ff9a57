// Thin inline-PTX wrappers for the sm_100a machinery used here: shared-memory
// mbarriers, TMA (cp.async.bulk.tensor) and bulk tile loads into this CTA's
// own shared memory, and the tcgen05 tensor-core / tensor-memory operations.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace gdn_rssm {
namespace ptx {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Asynchronous global -> shared copy of 4 or 8 bytes (cp.async, L1-cached);
// both addresses aligned to the size.  Complete with cp_async_wait_all() in
// the issuing thread, then a barrier, before others read the destination.
__device__ __forceinline__ void cp_async_small(void *smem_dst, const void *gsrc, int bytes) {
  if (bytes == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
  }
}
// 16-byte global -> shared copy, cached in L2 only (cp.async.cg); both
// addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
}
// As cp_async16, but copies nothing and zero-fills the 16 bytes when !full.
__device__ __forceinline__ void cp_async16_zfill(void *smem_dst, const void *gsrc, bool full) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem_dst)), "l"(gsrc),
               "r"(full ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Programmatic dependent launch: a primary kernel lets the next kernel in the
// stream start launching; that kernel waits for the primary's completion (and
// its memory) before reading what it wrote.  Both are no-ops without such a
// launch pairing.
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_prerequisite_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Makes the barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// As mbar_try_wait, but the thread may sleep (up to `hint_ns`) until the
// phase completes instead of returning at once.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Wait for phase `parity` of `bar` for at most `limit_ns`; false on timeout.
// A waiting thread sleeps in the barrier (woken when the phase completes)
// rather than spinning, so it takes no issue slots from working warps.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait_sleep(bar, parity, 100000u)) {
    if (global_timer_ns() - start > limit_ns) return false;
  }
  return true;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled TMA load global -> shared, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t c0,
                                            int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace ptx
}  // namespace gdn_rssm

namespace gdn_rssm {
namespace ptx {

// Untiled bulk copy shared -> global (16-byte aligned addresses, size a
// multiple of 16), tracked by this thread's bulk async-group; make generic
// shared-memory writes visible to it first (fence_proxy_async_smem).
__device__ __forceinline__ void bulk_store(void *dst, const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store of this thread has read its shared
// memory (the buffers may then be reused or the CTA may exit).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completion signalled on `bar`.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace ptx
}  // namespace gdn_rssm

// ---- tcgen05: 5th-generation tensor cores with tensor-memory accumulators --
namespace gdn_rssm {
namespace ptx {

// Warp-wide: allocate `ncols` (power of two >= 32) tensor-memory columns and
// write their base address to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
}

// Warp-wide: this CTA allocates no more tensor memory.
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Warp-wide (the allocating warp): free the columns.
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Order tcgen05 operations around a thread synchronisation.
__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor-core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand stored in 128-byte
// swizzle atoms (8 rows x 128 bytes, 1024-byte aligned, rows 128 bytes apart,
// 16-byte chunk c of row r at chunk c ^ (r % 8)).  `addr` may point 32, 64 or
// 96 bytes into the first row to select a K sub-block.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3fffu);  // start address, 16-byte units
  d |= static_cast<uint64_t>(1) << 16;                // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;        // stride byte offset: next 8-row group
  d |= static_cast<uint64_t>(1) << 46;                // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                // 128-byte swizzle
  return d;
}

// Instruction descriptor: D (f32) += A (tf32, K-major, M rows) x B^T (tf32,
// K-major, N rows).
template <int M, int N>
__host__ __device__ constexpr uint32_t tf32_instr_desc() {
  static_assert(M == 128 && N % 16 == 0 && N >= 16 && N <= 256, "tf32 MMA shape");
  return (1u << 4)                                 // accumulator f32
         | (2u << 7)                               // A tf32
         | (2u << 10)                              // B tf32
         | (static_cast<uint32_t>(N >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);  // M / 16
}

// One thread: D[tmem] (+)= A x B^T, K = 8 (32 bytes of each operand row).
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

// Instruction descriptor: D (f32) += A (bf16, K-major, M rows) x B^T (bf16,
// K-major, N rows), K = 16 per instruction.
template <int M, int N>
__host__ __device__ constexpr uint32_t bf16_instr_desc() {
  static_assert(M == 128 && N % 16 == 0 && N >= 16 && N <= 256, "bf16 MMA shape");
  return (1u << 4)                                 // accumulator f32
         | (1u << 7)                               // A bf16
         | (1u << 10)                              // B bf16
         | (static_cast<uint32_t>(N >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);  // M / 16
}

// One thread: D[tmem] (+)= A[tmem] x B^T, A = 128 lanes x 8 columns of packed
// bf16 pairs (K = 16, element 2c in the low half of column c) in tensor
// memory, B in shared memory.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05 operation this thread issued so
// far has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Warp-wide: lane i reads NCOL (16 or 32) consecutive 32-bit columns of
// tensor-memory lane (lane base of `taddr`) + i.  The wait for the load is in
// the same asm statement, so no use of the outputs can be scheduled before
// the data has arrived.
template <int NCOL>
__device__ __forceinline__ void tmem_ld_sync(uint32_t taddr, float *v) {
  static_assert(NCOL == 8 || NCOL == 16 || NCOL == 32, "tcgen05.ld width");
  uint32_t r[NCOL];
  if constexpr (NCOL == 8) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
  } else if constexpr (NCOL == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
  }
#pragma unroll
  for (int i = 0; i < NCOL; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp-wide: lane i writes 16 consecutive 32-bit columns (raw words) of
// tensor-memory lane (lane base of `taddr`) + i.  Complete with
// tmem_wait_st() before the columns are read by an MMA.
__device__ __forceinline__ void tmem_st16_u(uint32_t taddr, const uint32_t *v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
               : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace ptx
}  // namespace gdn_rssm
