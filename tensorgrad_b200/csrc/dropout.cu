// Inverted dropout with the reference's keep-mask generated on the device (_random.py:53-70,
// ops/layers.py:235-259, ops/attention.py:59-68).
//
// The reference draws its masks from NumPy's default generator, PCG64: a 128-bit linear
// congruential generator x <- x * M + inc (mod 2^128) whose 64-bit output for each step is
// the XSL-RR permutation of the new state, rotr64(hi ^ lo, hi >> 58) (O'Neill, "PCG: A Family
// of Simple Fast Space-Efficient Statistically Good Algorithms for Random Number Generation",
// 2014). `keep_mask` takes ceil(n / 4) raw 64-bit outputs, views them as 16-bit words
// (little-endian: element 4w + j is bits [16 j, 16 j + 16) of output w) and keeps an element
// when its word is >= threshold = round(p * 65536). Kept elements are multiplied by
// 65536 / (65536 - threshold) in the tensor's dtype, dropped ones by 0.
//
// Here every thread computes its outputs directly from the generator state the host passes
// in (the state before the call's first draw): the LCG's n-step map x -> A_n x + C_n is
// formed by squaring (Brown, "Random Number Generation with Arbitrary Strides", Trans. Am.
// Nucl. Soc. 1994), so a thread jumps once to its first 64-bit output and then strides by
// the grid's thread count with one precomputed affine step per output. The mask is never
// stored: the VJP regenerates it from the same state. Same state in, same mask out as the
// reference, bit for bit; the host advances its generator past the n / 4 outputs consumed.
#include <algorithm>

#include "common.cuh"
#include "pcg64.cuh"

namespace tg {
namespace {

using pcg::Affine;
using pcg::lcg_jump;
using pcg::make128;
using pcg::u128;
using pcg::xsl_rr;

struct PcgArgs {
  uint64_t s_hi, s_lo, inc_hi, inc_lo;  // state before the first draw, increment
  uint64_t stride_a_hi, stride_a_lo, stride_c_hi, stride_c_lo;  // map over `threads` steps
  int64_t word0;     // output index of element 0 (the element offset / 4 of a view)
  int64_t threads;   // grid size in threads
  uint32_t threshold;
};

// y[i] = x[i] * (keep(e0 + i) ? scale : 0) for the n elements of x, e0 = 4 * word0 + lane0.
template <typename T>
__global__ void __launch_bounds__(256)
dropout_pcg_kernel(int64_t n, int lane0, const T* __restrict__ x, T* __restrict__ y, T scale,
                   PcgArgs a) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // Outputs (64-bit words) covering elements [0, n) of this view: word k holds elements
  // 4 k - lane0 .. 4 k - lane0 + 3.
  const int64_t words = (n + lane0 + 3) / 4;
  if (tid >= words) return;
  const u128 inc = make128(a.inc_hi, a.inc_lo);
  // State after output (word0 + tid) has been drawn: jump (word0 + tid + 1) steps.
  const Affine j = lcg_jump(inc, (uint64_t)(a.word0 + tid + 1));
  u128 x_state = j.a * make128(a.s_hi, a.s_lo) + j.c;
  const u128 sa = make128(a.stride_a_hi, a.stride_a_lo), sc = make128(a.stride_c_hi, a.stride_c_lo);
  for (int64_t w = tid; w < words; w += a.threads) {
    const uint64_t r = xsl_rr(x_state);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t i = 4 * w + q - lane0;
      if (i >= 0 && i < n) {
        const uint32_t word16 = (uint32_t)(r >> (16 * q)) & 0xFFFFu;
        y[i] = x[i] * (word16 >= a.threshold ? scale : T(0));
      }
    }
    x_state = sa * x_state + sc;
  }
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" int tg_dropout_pcg64(int dtype, int64_t n, const void* x, void* y,
                                const uint64_t* pcg_state, int64_t first_element,
                                uint32_t threshold, double scale, void* stream) {
  TG_CHECK_ARG(n >= 0 && first_element >= 0 && pcg_state != nullptr && threshold <= 65536,
               "dropout_pcg64: bad arguments");
  if (n == 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  PcgArgs a{};
  a.s_hi = pcg_state[0]; a.s_lo = pcg_state[1];
  a.inc_hi = pcg_state[2]; a.inc_lo = pcg_state[3];
  a.word0 = first_element / 4;
  const int lane0 = (int)(first_element % 4);
  a.threshold = threshold;
  const int64_t words = (n + lane0 + 3) / 4;
  const int64_t want = (words + 7) / 8;  // about 8 outputs per thread
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>((want + 255) / 256, 1), 148 * 8);
  a.threads = (int64_t)blocks * 256;
  const Affine st = lcg_jump(make128(a.inc_hi, a.inc_lo), (uint64_t)a.threads);
  a.stride_a_hi = (uint64_t)(st.a >> 64); a.stride_a_lo = (uint64_t)st.a;
  a.stride_c_hi = (uint64_t)(st.c >> 64); a.stride_c_lo = (uint64_t)st.c;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    dropout_pcg_kernel<T><<<blocks, 256, 0, s>>>(n, lane0, (const T*)x, (T*)y, (T)scale, a);
    return check_launch("dropout_pcg64");
  });
}
