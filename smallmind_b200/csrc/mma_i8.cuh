// Integer tensor-core fragment MMA (legacy mma.sync path, sm_80+ instruction set).
#pragma once
#include <cstdint>

namespace sm {

// D = A B, m16n8k32, A u8 (row), B s8 (col), zero accumulator input
__device__ __forceinline__ void mma_u8s8(int& d0, int& d1, int& d2, int& d3, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  const int z = 0;
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}

}  // namespace sm
