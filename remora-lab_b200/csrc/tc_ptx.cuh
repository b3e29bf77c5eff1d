// tc_ptx.cuh — thin inline-PTX wrappers for the sm_100a tensor-core path:
// mbarriers, cp.async, TMEM allocation, tcgen05.mma / commit / ld, and the
// shared-memory and instruction descriptors of kind::f16 MMAs.
//
// Operand layout used everywhere: K-major, 128-byte swizzle.  A tile of R rows
// by 64 f16 (128 B per row) is one "atom column": rows are 128 B apart inside
// groups of 8 rows, groups are 1024 B apart (the descriptor's stride byte
// offset), and the 16-byte piece j of row r sits at piece position j ^ (r % 8).
// Atom columns start on 1024-byte boundaries.  Moving the descriptor's start
// address by 32 B steps to the next K=16 slice inside the atom column.
#pragma once

#include <stdint.h>

namespace har {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of the same condition (never suspends the thread).
__device__ __forceinline__ uint32_t mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok;
}
// The same test at shared address bar + OFF (bytes).
template <int OFF>
__device__ __forceinline__ uint32_t mbar_test_wait_at(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1+%3], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(OFF)
      : "memory");
  return ok;
}
// Bounded wait: false after `limit` polls (the caller records an error word).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// The same with a short sleep between polls (32 ns doubling up to cap_ns),
// for waiters that can afford the delay: a spinning warp takes issue slots
// from the warps that do the work.  At most limit polls, ~limit * cap_ns.
__device__ __forceinline__ bool mbar_wait_lazy(uint64_t *bar, uint32_t parity, uint32_t limit,
                                               uint32_t cap_ns) {
  uint32_t ns = 32;
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(ns);
    if (ns < cap_ns) ns <<= 1;
  }
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// ---- TMA (tiled tensor loads, no multicast) ------------------------------------
// 2-D box at coordinates (x innermost, y) of the tensor map into shared memory;
// completion is counted in bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Untiled bulk copy of `bytes` contiguous bytes global -> this CTA's shared
// memory, completing `bytes` of transaction on `bar`.  Both addresses 16-byte
// aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- cp.async (16 B, zero-filled when src_bytes == 0) ------------------------
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// waits until at most N of this thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMEM ---------------------------------------------------------------------
// Warp-wide: allocates `ncols` (power of two >= 32) columns; the TMEM address is
// written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- descriptors ----------------------------------------------------------------
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B
// apart; bits: start>>4 [0,14), LBO>>4 [16,30) (unused here), SBO>>4 [32,46),
// version 1 [46,48), base offset 0, layout type 2 (SWIZZLE_128B) [61,64).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Shared-memory matrix descriptor: K-major, no swizzle.  Core matrices are
// 8 rows x 16 bytes (rows 16 B apart); lbo = byte distance between core
// matrices adjacent in K, sbo = between core matrices adjacent in M/N
// (layout type 0, SWIZZLE_NONE).
__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// Instruction descriptor of kind::f16: A and B f16, D f32, both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// ---- MMA --------------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Warp-collective: 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T: A (M=128 rows = TMEM lanes, K along
// columns, two f16 per 32-bit column) read from tensor memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-collective stores of 32 (x32) or 16 (x16) consecutive 32-bit columns
// into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Warp-wide forms: the whole (converged) warp executes them and the lane
// picked once by elect_one() (`lead` != 0) issues.  Keeping the issuing loop
// warp-uniform lets the operands stay in uniform registers; a loop run by a
// single thread, or an elect.sync per MMA, issues several times more slowly.
__device__ __forceinline__ uint32_t elect_one() {
  uint32_t p;
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, e;\n\t}"
      : "=r"(p));
  return p;
}
__device__ __forceinline__ void mma_f16_ts_w(uint32_t lead, uint32_t d_tmem, uint32_t a_tmem,
                                             uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "setp.ne.b32 e, %5, 0;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(lead)
      : "memory");
}
// Warp-wide form of one MMA with both operands in shared memory,
// D[tmem] += A[desc] * B[desc]^T, issued by the elected lane.
__device__ __forceinline__ void mma_f16_ss_w(uint32_t lead, uint32_t d_tmem, uint64_t adesc,
                                             uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "setp.ne.b32 e, %4, 0;\n\t"
      "setp.eq.b32 p, %4, %4;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(lead)
      : "memory");
}

// The MMAs of one 64-value K-step (4 x K=16) for NA = 1 or 2 matrices, from
// one asm block: matrix m accumulates at column d + m*bw and reads its weights
// from TMEM columns a + m*32 + kk*8; B advances 32 bytes (2 descriptor units)
// per K=16 slice.  The first slice overwrites when acc0 == 0.
template <int NA>
__device__ __forceinline__ void mma_kstep_ts(uint32_t lead, uint32_t d, uint32_t bw, uint32_t a,
                                             uint64_t b, uint32_t idesc, uint32_t acc0) {
  if (NA == 2) {
    asm volatile(
        "{\n\t.reg .pred e, p, t;\n\t.reg .b32 d1, a1, a2, a3, a4, a5, a6, a7;\n\t"
        ".reg .b64 b1, b2, b3;\n\t"
        "setp.ne.b32 e, %0, 0;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "setp.eq.b32 t, %0, %0;\n\t"
        "add.u32 d1, %1, %2;\n\t"
        "add.u32 a1, %3, 32;\n\t"
        "add.u32 a2, %3, 8;\n\t"
        "add.u32 a3, %3, 40;\n\t"
        "add.u32 a4, %3, 16;\n\t"
        "add.u32 a5, %3, 48;\n\t"
        "add.u32 a6, %3, 24;\n\t"
        "add.u32 a7, %3, 56;\n\t"
        "add.u64 b1, %4, 2;\n\t"
        "add.u64 b2, %4, 4;\n\t"
        "add.u64 b3, %4, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%3], %4, %5, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [a1], %4, %5, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [a2], b1, %5, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [a3], b1, %5, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [a4], b2, %5, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [a5], b2, %5, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [a6], b3, %5, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [d1], [a7], b3, %5, t;\n\t}" ::"r"(lead),
        "r"(d), "r"(bw), "r"(a), "l"(b), "r"(idesc), "r"(acc0)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred e, p, t;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
        "setp.ne.b32 e, %0, 0;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.eq.b32 t, %0, %0;\n\t"
        "add.u32 a1, %2, 8;\n\t"
        "add.u32 a2, %2, 16;\n\t"
        "add.u32 a3, %2, 24;\n\t"
        "add.u64 b1, %3, 2;\n\t"
        "add.u64 b2, %3, 4;\n\t"
        "add.u64 b3, %3, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %3, %4, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [a1], b1, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [a2], b2, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [a3], b3, %4, t;\n\t}" ::"r"(lead),
        "r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc0)
        : "memory");
    (void)bw;
  }
}

// mma_kstep_ts with every column offset an immediate (TMEM addresses take
// [reg+imm]): matrix m accumulates at column d + m*BW and reads weight
// columns a + m*32 + 8*kk for K=16 slice kk; B advances 2 descriptor units
// per slice.  Fewer instructions between two K-steps' MMAs keep the tensor
// pipe fed: a single issuing warp runs them back to back.
template <int NA, int BW>
__device__ __forceinline__ void mma_kstep_ts_imm(uint32_t lead, uint32_t d, uint32_t a, uint64_t b,
                                                 uint32_t idesc, uint32_t acc0) {
  if (NA == 2) {
    asm volatile(
        "{\n\t.reg .pred e, p, t;\n\t.reg .b64 b1, b2, b3;\n\t"
        "setp.ne.b32 e, %0, 0;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.eq.b32 t, %0, %0;\n\t"
        "add.u64 b1, %3, 2;\n\t"
        "add.u64 b2, %3, 4;\n\t"
        "add.u64 b3, %3, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %3, %4, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1+%6], [%2+32], %3, %4, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2+8], b1, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1+%6], [%2+40], b1, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2+16], b2, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1+%6], [%2+48], b2, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2+24], b3, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1+%6], [%2+56], b3, %4, t;\n\t}" ::"r"(lead),
        "r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc0), "n"(BW)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred e, p, t;\n\t.reg .b64 b1, b2, b3;\n\t"
        "setp.ne.b32 e, %0, 0;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.eq.b32 t, %0, %0;\n\t"
        "add.u64 b1, %3, 2;\n\t"
        "add.u64 b2, %3, 4;\n\t"
        "add.u64 b3, %3, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %3, %4, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2+8], b1, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2+16], b2, %4, t;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%2+24], b3, %4, t;\n\t}" ::"r"(lead),
        "r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc0), "n"(BW)
        : "memory");
  }
}

// Commit to the mbarrier at shared address bar + OFF (bytes).
template <int OFF>
__device__ __forceinline__ void mma_commit_at(uint32_t lead, uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %1, 0;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0+%2];\n\t}" ::"r"(bar),
      "r"(lead), "n"(OFF)
      : "memory");
}

__device__ __forceinline__ void mma_commit_w(uint32_t lead, uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "setp.ne.b32 e, %1, 0;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(lead)
      : "memory");
}

// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Warp-collective: this thread's TMEM lane, 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Warp-collective: this thread's TMEM lane, 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte offset of 16-byte piece j (0..7) of row r inside a 128B-swizzled atom column.
__device__ __forceinline__ uint32_t sw128_off(int r, int j) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

}  // namespace tc
}  // namespace har
