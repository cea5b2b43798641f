// 5th-generation tensor-core MMA (tcgen05.mma, kind::f16, one CTA) with both operands in
// shared memory and the fp32 accumulator in tensor memory.
//
// Operand tiles are K-major with the 128-byte swizzle (the layout the TMA tile maps write):
// rows of 64 16-bit values (128 bytes), groups of 8 rows 1024 bytes apart, tile base
// 1024-byte aligned. One instruction consumes K = 16 (32 bytes of each row); the next K
// step starts 32 bytes further into the swizzled row.
#pragma once

#include <stdint.h>

namespace ttt {

// Shared-memory matrix descriptor: start address >> 4 (bits 0-13), leading byte offset
// (bits 16-29, 16-byte units; 1 for swizzled K-major), stride byte offset between 8-row
// groups (bits 32-45: 1024 B), descriptor version 1 (bits 46-47), base offset 0, layout
// type 2 = 128-byte swizzle (bits 61-63).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor for kind::f16 with fp32 accumulation, both operands K-major:
// D format f32 (bits 4-5 = 1), A and B format (bits 7-9, 10-12: 0 f16, 1 bf16), N >> 3
// (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t umma_idesc_f32(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A * B^T for one K = 16 step; issued by a single thread.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrive on the mbarrier once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

}  // namespace ttt
