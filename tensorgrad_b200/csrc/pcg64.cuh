// NumPy's PCG64 generator on the device: the 128-bit LCG x <- x * M + inc (mod 2^128) with
// the XSL-RR output permutation rotr64(hi ^ lo, hi >> 58) of each new state (O'Neill 2014),
// and its n-step jump x -> A_n x + C_n by squaring (Brown 1994). Shared by the dropout
// kernels (dropout.cu, attention_dropout.cu).
#pragma once

#include "common.cuh"

namespace tg {
namespace pcg {

typedef unsigned __int128 u128;

constexpr uint64_t kMulHi = 0x2360ED051FC65DA4ull, kMulLo = 0x4385DF649FCCF645ull;

__host__ __device__ __forceinline__ u128 make128(uint64_t hi, uint64_t lo) {
  return ((u128)hi << 64) | (u128)lo;
}

// The LCG's n-step map: x_{k+n} = a x_k + c (mod 2^128).
struct Affine {
  u128 a, c;
};

__host__ __device__ inline Affine lcg_jump(u128 inc, uint64_t n) {
  u128 acc_a = 1, acc_c = 0, cur_a = make128(kMulHi, kMulLo), cur_c = inc;
  while (n) {
    if (n & 1) {
      acc_a *= cur_a;
      acc_c = acc_c * cur_a + cur_c;
    }
    cur_c = (cur_a + 1) * cur_c;
    cur_a *= cur_a;
    n >>= 1;
  }
  return {acc_a, acc_c};
}

__device__ __forceinline__ uint64_t xsl_rr(u128 x) {
  const uint64_t hi = (uint64_t)(x >> 64), lo = (uint64_t)x;
  const uint64_t v = hi ^ lo;
  const unsigned r = (unsigned)(hi >> 58);
  return (v >> r) | (v << ((64 - r) & 63));
}

// The 64-bit output `index` (0-based) of the stream that starts at state s0 (before its first
// draw).
__device__ __forceinline__ uint64_t output_at(u128 s0, u128 inc, uint64_t index) {
  const Affine j = lcg_jump(inc, index + 1);
  return xsl_rr(j.a * s0 + j.c);
}

}  // namespace pcg
}  // namespace tg
