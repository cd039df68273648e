// tcgen05 (5th-generation tensor core) helpers for sm_100a: UMMA shared-memory
// and instruction descriptors, MMA issue (operands in shared memory, or A in
// tensor memory), commits to mbarriers, tensor-memory allocation and
// warp-collective TMEM loads/stores.
//
// Shared-memory operands use the 128-byte-swizzle canonical layouts that TMA
// boxes of 64 bf16 x R rows produce (1024-byte aligned):
//  * K-major (A = Q, B = K in S = Q K^T): rows of 128 B, 8-row groups 1024 B
//    apart (SBO = 1024); one MMA K-step of 16 elements advances the start
//    address by 32 B inside the swizzle atom; the next 64-element column block
//    is a separate box.
//  * MN-major (B = V in O = P V): 64 contiguous N elements per 128-B row, rows
//    are K (tokens), 8-row groups 1024 B apart (SBO), the next 64-element N
//    block LBO bytes away.
#pragma once

#include "common.cuh"

namespace mb {

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: bf16 A and B, f32 accumulator.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Warp-wide forms: all 32 lanes execute them (converged) and elect.sync picks
// the one lane that issues. Running the MMA warp's whole control flow with all
// lanes keeps descriptors and TMEM addresses warp-uniform, which issues
// markedly faster than a loop confined to `if (lane == 0)`.
__device__ __forceinline__ void umma_ss_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// One warp-wide asm block per group of MMAs: a single elect.sync, then the
// K-steps with their descriptor offsets as immediates, so the issuing warp
// spends a few instructions per MMA (its SM sub-partition is shared with
// element-wise warps, and a long issue sequence starves the tensor pipe).
//
// D = A B^T over 128 (HD = 128: K-steps at 32-byte offsets inside each of two
// 64-element boxes 16 KB apart) or 64 (one box) elements; A and B K-major
// SW128 descriptors; the first K-step overwrites D.
__device__ __forceinline__ void umma_ss_k128_warp(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, t, f;\n\t.reg .b64 a, b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 f, %3, %3;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, f;\n\t"
      "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 1024;\n\tadd.s64 b, %2, 1024;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 1026;\n\tadd.s64 b, %2, 1026;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 1028;\n\tadd.s64 b, %2, 1028;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 1030;\n\tadd.s64 b, %2, 1030;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}"
      ::"r"(d), "l"(da), "l"(db), "r"(idesc));
}

__device__ __forceinline__ void umma_ss_k64_warp(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, t, f;\n\t.reg .b64 a, b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 f, %3, %3;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, f;\n\t"
      "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}"
      ::"r"(d), "l"(da), "l"(db), "r"(idesc));
}

// D (+)= A B over 128 tokens: A bf16 in TMEM, 16 tokens per K-step packed in
// 8 columns, the K-steps of token block kk at column 64 * (kk / 4) + 8 * (kk % 4)
// (two 64-token halves, each packed into its first 32 columns); B MN-major
// SW128 (16 token rows = 2048 bytes per K-step). `accumulate` applies to the
// first K-step only.
__device__ __forceinline__ void umma_ts_t128_warp(uint32_t d, uint32_t a, uint64_t db, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, t, p;\n\t.reg .b32 ta;\n\t.reg .b64 b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "add.u32 ta, %1, 8;\n\tadd.s64 b, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 16;\n\tadd.s64 b, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 24;\n\tadd.s64 b, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 64;\n\tadd.s64 b, %2, 512;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 72;\n\tadd.s64 b, %2, 640;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 80;\n\tadd.s64 b, %2, 768;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 88;\n\tadd.s64 b, %2, 896;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t}"
      ::"r"(d), "r"(a), "l"(db), "r"(idesc), "r"(accumulate));
}

// Shared-memory descriptor of a non-swizzled canonical layout: 8 x 16-byte
// core matrices of 128 contiguous bytes. For an MN-major operand, LBO is the
// byte distance between core matrices adjacent in K (8 rows further) and SBO
// between core matrices adjacent in M/N (8 elements further).
__device__ __forceinline__ uint64_t umma_desc_noswz(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100; swizzle field 0 = none
  return d;
}

// D (+)= A B over 128 K rows, both operands MN-major in shared memory: A
// non-swizzled with K-adjacent core matrices 128 bytes apart (a K-step of 16
// rows advances it by 256 bytes), B SW128 (16 rows = 2048 bytes per K-step).
// `accumulate` applies to the first K-step only.
__device__ __forceinline__ void umma_ss_mn_t128_warp(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, t, p;\n\t.reg .b64 a, b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "add.s64 a, %1, 16;\n\tadd.s64 b, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 32;\n\tadd.s64 b, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 48;\n\tadd.s64 b, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 64;\n\tadd.s64 b, %2, 512;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 80;\n\tadd.s64 b, %2, 640;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 96;\n\tadd.s64 b, %2, 768;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 112;\n\tadd.s64 b, %2, 896;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}"
      ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

// As umma_ts_t128_warp, with A written by four 32-token quarters, each packed
// into the first 16 columns of its own 32: K-step kk at column
// 32 * (kk / 2) + 8 * (kk % 2).
__device__ __forceinline__ void umma_ts_t128_quarters_warp(uint32_t d, uint32_t a, uint64_t db, uint32_t idesc,
                                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, t, p;\n\t.reg .b32 ta;\n\t.reg .b64 b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "add.u32 ta, %1, 8;\n\tadd.s64 b, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 32;\n\tadd.s64 b, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 40;\n\tadd.s64 b, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 64;\n\tadd.s64 b, %2, 512;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 72;\n\tadd.s64 b, %2, 640;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 96;\n\tadd.s64 b, %2, 768;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 104;\n\tadd.s64 b, %2, 896;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t}"
      ::"r"(d), "r"(a), "l"(db), "r"(idesc), "r"(accumulate));
}

// Half of umma_ts_t128_quarters_warp: the four K-steps of two 32-token
// quarters (A columns 0, 8, 32, 40 from `a`; B rows 0-63 from `db`). The
// second half is the same call with a + 64, db + 512 and accumulate = 1.
__device__ __forceinline__ void umma_ts_t64_quarters_warp(uint32_t d, uint32_t a, uint64_t db, uint32_t idesc,
                                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, t, p;\n\t.reg .b32 ta;\n\t.reg .b64 b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "add.u32 ta, %1, 8;\n\tadd.s64 b, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 32;\n\tadd.s64 b, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 40;\n\tadd.s64 b, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t}"
      ::"r"(d), "r"(a), "l"(db), "r"(idesc), "r"(accumulate));
}

// As umma_ts_t128_warp, with the 128 tokens of A packed contiguously: K-step
// kk at column 8 * kk.
__device__ __forceinline__ void umma_ts_t128_linear_warp(uint32_t d, uint32_t a, uint64_t db, uint32_t idesc,
                                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, t, p;\n\t.reg .b32 ta;\n\t.reg .b64 b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "add.u32 ta, %1, 8;\n\tadd.s64 b, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 16;\n\tadd.s64 b, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 24;\n\tadd.s64 b, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 32;\n\tadd.s64 b, %2, 512;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 40;\n\tadd.s64 b, %2, 640;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 48;\n\tadd.s64 b, %2, 768;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t"
      "add.u32 ta, %1, 56;\n\tadd.s64 b, %2, 896;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], b, %3, t;\n\t}"
      ::"r"(d), "r"(a), "l"(db), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Every MMA the calling warp issued completes before its CTA frees TMEM and
// exits: one commit of all of them to `bar` (a barrier of count 1 used for
// nothing else) and a wait on its first phase, bounded by kDrainCycles. An
// issued MMA always completes (its operands were complete when it was
// issued), so this holds on a timed-out pipeline too.
__device__ __forceinline__ void umma_drain_warp(uint64_t* bar) {
  umma_commit_warp(bar);
  mbar_drain(bar, 0);
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Whole-warp TMEM allocation; the base address lands in *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 16 consecutive 32-bit columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 3-D tiled TMA load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 2^x on the SFU (ex2.approx: about 2 ulp, flushes denormals; x = -inf gives 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, to take part of the exponentials off the SFU when it is
// the bottleneck. Range reduction: adding 1.5 * 2^23 rounds x to the nearest
// integer n (kept in the low mantissa bits), f = x - n lies in [-0.5, 0.5];
// 2^f is a cubic (1 + c1 f + c2 f^2 + c3 f^3, least-squares fit of the
// relative error, reweighted to near-minimax: max relative error 1.0e-4,
// below the bf16 rounding the results get), and n is added to the exponent
// field. x is clamped at -126 (the result is then ~1e-38, not 0).
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  float p = fmaf(0.0550089821f, f, 0.242210975f);
  p = fmaf(p, f, 0.693282916f);
  p = fmaf(p, f, 1.f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Three-input f32 maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Three-input f32 minimum.
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed fp32 pairs (one instruction for two lanes of arithmetic on sm_100):
// (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1) and (d0, d1) = (a0, a1) + (b0, b1),
// each rounded to nearest like fmaf / a + b.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// exp2_fma on a pair, its range reduction and cubic in packed fp32 pairs:
// the same arithmetic (and results) as two exp2_fma calls in fewer
// instructions.
__device__ __forceinline__ void exp2_fma2(float& y0, float& y1, float x0, float x1) {
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float t0, t1, n0, n1, f0, f1, q0, q1;
  fadd2(t0, t1, x0, x1, 12582912.f, 12582912.f);
  fadd2(n0, n1, t0, t1, -12582912.f, -12582912.f);
  ffma2(f0, f1, n0, n1, -1.f, -1.f, x0, x1);  // x - n, exact
  ffma2(q0, q1, 0.0550089821f, 0.0550089821f, f0, f1, 0.242210975f, 0.242210975f);
  ffma2(q0, q1, q0, q1, f0, f1, 0.693282916f, 0.693282916f);
  ffma2(q0, q1, q0, q1, f0, f1, 1.f, 1.f);
  y0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// Warpgroup register re-balancing (all four warps of a warpgroup execute it).
// The block's register budget is fixed at launch; a kernel's decreases and
// increases must sum to no more than that budget.
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Warp-uniform bounded wait: false (in every lane) if any lane timed out.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int code) {
  const bool ok = mbar_wait(bar, parity, code);
  return __all_sync(0xffffffffu, ok);
}

}  // namespace mb
