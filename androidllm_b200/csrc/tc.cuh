// tcgen05 (5th-generation tensor core) primitives for sm_100a: tensor-memory
// allocation, register <-> tensor-memory moves, the MMA with its A operand in
// tensor memory and B in shared memory, completion tracking on mbarriers, and
// the descriptors those instructions take.
//
// Layouts (kind::f16, cta_group::1, M = 128):
//   * A in tensor memory: row i in lane i; column c holds k = 2c (low half)
//     and 2c + 1 (high half); one k16 step spans 8 columns.
//   * B in shared memory, K-major, no swizzle: "core matrices" of 8 rows x 16
//     bytes stored row after row (128 B); the leading byte offset (LBO) steps
//     between the two 8-element K halves of a k16 step, the stride byte
//     offset (SBO) between groups of 8 rows (N).
//   * D (fp32) in tensor memory: row i in lane i, column n.
// A warp may only reach the 32 lanes 32 * (warp_id % 4) ... + 31.
#pragma once
#include "common.cuh"

namespace alm {

// Instruction descriptor of tcgen05.mma kind::f16: f32 accumulator, f16 A and
// B, both K-major, shape M x N (M = 64 / 128, N a multiple of 16 up to 256).
__host__ __device__ constexpr uint32_t tc_idesc_f16(int m, int n) {
  return (1u << 4)                                      // D format: f32
         | (0u << 7) | (0u << 10)                       // A, B: f16
         | (static_cast<uint32_t>(n >> 3) << 17)        // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);       // M / 16
}

// Shared-memory matrix descriptor, K-major without swizzle.
ALM_DEV uint64_t tc_sdesc(uint32_t smem_byte_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;   // descriptor version of sm_100
  return d;
}

// Tensor-memory address of (lane, column).
ALM_DEV uint32_t tc_addr(uint32_t base, int lane, int col) {
  return base + (static_cast<uint32_t>(lane) << 16) + static_cast<uint32_t>(col);
}

// Allocation: one full warp; the base address is written to shared memory.
ALM_DEV void tc_alloc(uint32_t* dst_smem, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
ALM_DEV void tc_dealloc(uint32_t base, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

ALM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ALM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
ALM_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
ALM_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive columns of the warp's 32 lanes from registers.
ALM_DEV void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 16 consecutive columns of the warp's 32 lanes into registers (fp32 bits).
ALM_DEV void tc_ld16(uint32_t taddr, uint32_t (&d)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]), "=r"(d[8]),
        "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
      : "r"(taddr)
      : "memory");
}

// D (+)= A (tensor memory) x B (shared memory descriptor); one thread.
ALM_DEV void tc_mma_ts(uint32_t d_taddr, uint32_t a_taddr, uint64_t b_desc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_taddr),
      "r"(a_taddr), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0)
      : "memory");
}

// Arrive (once) on an mbarrier when every tcgen05 operation this thread has
// issued so far has completed.
ALM_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

ALM_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

}  // namespace alm
