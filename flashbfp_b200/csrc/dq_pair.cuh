// dq_pair.cuh — OABF block to bf16 pairs with integer bit operations, shared by the tcgen05
// kernels (one row per lane; results are exact).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace fbfp {

// One 16-weight block -> 8 bf16 pairs of natural elements (2j, 2j+1), each element exactly
// s*m*2^e (the format's 1/15 is applied by the caller): v = +-(128 + m) * 2^e (sign bit 15/31,
// exponent field e + 134 = eb, nibble in bits 0-3/16-19) and c = +-128 * 2^e are built with bit
// operations; v - c is exact in bf16. w0/w1 hold elements 0-7/8-15 (element i in nibble i % 8),
// s16 bit i is the sign of element i.
__device__ __forceinline__ void dq_block(uint32_t w0, uint32_t w1, uint32_t s16, uint32_t eb,
                                         uint32_t* out) {
  const uint32_t SM = 0x80008000u, NM = 0x000F000Fu;
  const uint32_t y = s16 | (s16 << 15);          // sign bit b lands on 15 and 31 after << (15 - b)
  const uint32_t K = eb * 0x00800080u;
  const uint32_t t0 = w0 >> 4, t1 = w1 >> 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sel = (uint32_t)j | ((uint32_t)(4 + j) << 8);   // byte j of w, byte j of w>>4
    const uint32_t c0 = ((y << (15 - 2 * j)) & SM) | K;
    const uint32_t c1 = ((y << (7 - 2 * j)) & SM) | K;
    const uint32_t v0 = (__byte_perm(w0, t0, sel) & NM) | c0;
    const uint32_t v1 = (__byte_perm(w1, t1, sel) & NM) | c1;
    __nv_bfloat162 r0 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v0),
                                *reinterpret_cast<const __nv_bfloat162*>(&c0));
    __nv_bfloat162 r1 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v1),
                                *reinterpret_cast<const __nv_bfloat162*>(&c1));
    out[j] = *reinterpret_cast<uint32_t*>(&r0);
    out[4 + j] = *reinterpret_cast<uint32_t*>(&r1);
  }
}

// Write bf16 bits `b` into element `el` (0..63) of the 32 pair registers of a 4-block substage.
// The switch compiles to a jump table, which keeps the array in registers.
__device__ __forceinline__ void patch_pair(uint32_t (&w)[32], int el, uint32_t b) {
  const uint32_t keep = (el & 1) ? 0x0000FFFFu : 0xFFFF0000u;
  const uint32_t put = (el & 1) ? (b << 16) : b;
  switch (el >> 1) {
#define FBFP_PATCH_CASE(r) case r: w[r] = (w[r] & keep) | put; break;
    FBFP_PATCH_CASE(0) FBFP_PATCH_CASE(1) FBFP_PATCH_CASE(2) FBFP_PATCH_CASE(3)
    FBFP_PATCH_CASE(4) FBFP_PATCH_CASE(5) FBFP_PATCH_CASE(6) FBFP_PATCH_CASE(7)
    FBFP_PATCH_CASE(8) FBFP_PATCH_CASE(9) FBFP_PATCH_CASE(10) FBFP_PATCH_CASE(11)
    FBFP_PATCH_CASE(12) FBFP_PATCH_CASE(13) FBFP_PATCH_CASE(14) FBFP_PATCH_CASE(15)
    FBFP_PATCH_CASE(16) FBFP_PATCH_CASE(17) FBFP_PATCH_CASE(18) FBFP_PATCH_CASE(19)
    FBFP_PATCH_CASE(20) FBFP_PATCH_CASE(21) FBFP_PATCH_CASE(22) FBFP_PATCH_CASE(23)
    FBFP_PATCH_CASE(24) FBFP_PATCH_CASE(25) FBFP_PATCH_CASE(26) FBFP_PATCH_CASE(27)
    FBFP_PATCH_CASE(28) FBFP_PATCH_CASE(29) FBFP_PATCH_CASE(30) FBFP_PATCH_CASE(31)
#undef FBFP_PATCH_CASE
    default: break;
  }
}

}  // namespace fbfp
