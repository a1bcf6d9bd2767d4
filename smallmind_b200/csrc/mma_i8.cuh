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

// 2^e for -126 < e < 128, built from the exponent field
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// Exponent e with am < 2^e (for a normal am > 0: the frexp exponent), clamped so
// that 2^(+-(22 - e)) stay normal floats; 0 for am == 0.
__device__ __forceinline__ int block_exp(float am) {
  return am > 0.f ? max(((__float_as_int(am) >> 23) & 0xFF) - 126, -100) : 0;
}

// Balanced base-256 digits of four integers |x| < 2^22, x = hi 2^16 + b 2^8 + c
// with b, c in [-128, 127]: x + 0x808080 holds c + 128, b + 128 and hi + 128 as its
// three low bytes, so the digits are those bytes with the sign bit flipped.  Word
// whi / wb / wc holds the digit of x0..x3 in bytes 0..3.
__device__ __forceinline__ void digits4(int x0, int x1, int x2, int x3, uint32_t& whi, uint32_t& wb,
                                        uint32_t& wc) {
  const uint32_t y0 = (uint32_t)(x0 + 0x808080), y1 = (uint32_t)(x1 + 0x808080);
  const uint32_t y2 = (uint32_t)(x2 + 0x808080), y3 = (uint32_t)(x3 + 0x808080);
  const uint32_t l01 = __byte_perm(y0, y1, 0x5140), l23 = __byte_perm(y2, y3, 0x5140);  // bytes 0, 1
  const uint32_t h01 = __byte_perm(y0, y1, 0x7362), h23 = __byte_perm(y2, y3, 0x7362);  // bytes 2, 3
  wc = __byte_perm(l01, l23, 0x5410) ^ 0x80808080u;
  wb = __byte_perm(l01, l23, 0x7632) ^ 0x80808080u;
  whi = __byte_perm(h01, h23, 0x5410) ^ 0x80808080u;
}

}  // namespace sm
