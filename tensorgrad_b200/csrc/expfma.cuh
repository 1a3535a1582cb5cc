// exp(x) on the FMA and integer pipes, for softmax numerators (x <= a few units above 0).
//
// The fused attention kernels need one exponential per score; the hardware's approximate
// exponential runs on the XU pipe, which the counters show as the busiest unit of those
// kernels, so part of the exponentials is computed here instead, in plain fp32 arithmetic:
//
//   * range reduction in the manner of Cody and Waite (W. J. Cody, W. Waite, "Software Manual
//     for the Elementary Functions", 1980): n = round(x log2(e)), found by adding and
//     subtracting 1.5 * 2^23 (the sum rounds to an integer in fp32, so no conversion
//     instruction is needed), then r = x - n ln2 evaluated exactly with ln2 split into a
//     16-bit head (n * head is exact for |n| < 2^8) and a tail, r in [-ln2/2, ln2/2];
//   * e^r by a degree-6 polynomial fitted for this file to e^r on that interval (iteratively
//     reweighted least squares on Chebyshev nodes towards the minimax relative error:
//     1.9e-9 in exact arithmetic, about 8e-8 evaluated in fp32 by Horner's rule with FMAs);
//   * 2^n added into the exponent bits with integer arithmetic.
//
// Inputs below -87.3 (e^x < 2^-126) give 0, which is what a softmax numerator of that size
// contributes at fp32 precision; -inf gives +0; NaN gives NaN. Inputs are expected below +88.
#pragma once

namespace tg {

__device__ __forceinline__ float exp_fma(float x) {
  const float t = fmaxf(x * 1.44269504f, -127.f);  // about x log2(e); only n depends on it
  const float s = t + 12582912.f;                  // 1.5 * 2^23: s = n + 1.5 * 2^23
  const float n = s - 12582912.f;
  float r = fmaf(n, -0.693145752f, x);             // ln2 head (0x3F317200): exact product
  r = fmaf(n, -1.42860677e-6f, r);                 // ln2 tail
  float p = 1.38294231e-3f;
  p = fmaf(p, r, 8.37477110e-3f);
  p = fmaf(p, r, 4.16683592e-2f);
  p = fmaf(p, r, 1.66664213e-1f);
  p = fmaf(p, r, 4.99999911e-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = __float_as_int(s) - 0x4B400000;  // n as an integer
  const float v = __int_as_float(__float_as_int(p) + (ni << 23));
  return x < -87.3f ? 0.f : (x == x ? v : x);  // NaN stays NaN (its bits plus 2^n would not)
}

}  // namespace tg
