// Noise for stochastic rounding: Philox4x32-10 draws as Triton's tl.rand makes them,
// shared by the MoE backward (backward.cu) and the single-matrix backward
// (linear_bwd.cu, quant.cu).
#pragma once

#include "common.cuh"

namespace mcl4 {

// Word 0 of Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers:
// as easy as 1, 2, 3", SC'11) for counter (c0, 0, 0, 0) and key (k0, k1): the
// draw of Triton's tl.randint(seed, offset) for a 32-bit offset.
// Each round takes both halves of its two 32x32-bit products from one wide multiply.
__device__ __forceinline__ uint32_t philox_word0(uint32_t c0, uint32_t k0, uint32_t k1) {
  uint32_t c1 = 0u, c2 = 0u, c3 = 0u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t pa = uint64_t(0xD2511F53u) * uint64_t(c0);
    const uint64_t pb = uint64_t(0xCD9E8D57u) * uint64_t(c2);
    c0 = uint32_t(pb >> 32) ^ c1 ^ k0;
    c2 = uint32_t(pa >> 32) ^ c3 ^ k1;
    c1 = uint32_t(pb);
    c3 = uint32_t(pa);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

// Triton's uint_to_uniform_float for 32-bit words: int32 x, x < 0 ? -x - 1 : x,
// times 4.6566127342e-10 in float32.
__device__ __forceinline__ float uniform_from_word(uint32_t w) {
  const int32_t x = int32_t((w & 0x80000000u) ? ~w : w);
  return __fmul_rn(__int2float_rn(x), 4.6566127342e-10f);
}

// Uniform draw for noise offset `off` under seed (k0 = low word, k1 = high word).
__device__ __forceinline__ float sr_uniform(uint32_t off, uint32_t k0, uint32_t k1) {
  return uniform_from_word(philox_word0(off, k0, k1));
}

// E2M1 code of a normalised value with stochastic rounding
// (src/mcl4_coe/nvfp4.py:186-194, stochastic branch): m = min(|v|, 6);
// u = 2m | m+2 | m/2+4; code = min(trunc(u + U), 7) | signbit(v) << 3.
__device__ __forceinline__ uint32_t e2m1_code_sr(float v, float uni) {
  const float m = fminf(fabsf(v), 6.0f);
  float u;
  if (m <= 2.0f) u = __fmul_rn(m, 2.0f);
  else if (m <= 4.0f) u = __fadd_rn(m, 2.0f);
  else u = __fadd_rn(__fmul_rn(m, 0.5f), 4.0f);
  const uint32_t code = min(static_cast<uint32_t>(__fadd_rn(u, uni)), 7u);
  return code | ((__float_as_uint(v) >> 31) << 3);
}

}  // namespace mcl4
