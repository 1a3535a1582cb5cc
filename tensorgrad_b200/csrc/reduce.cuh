// Reduction helpers shared between translation units.
#pragma once
#include "common.cuh"

namespace tg {

constexpr int kMaxDims = 8;

struct ReduceDims {
  int n_keep, n_red;
  int64_t keep_size[kMaxDims], keep_stride[kMaxDims];
  int64_t red_size[kMaxDims], red_stride[kMaxDims];
  int64_t out_count, red_count;
};

// Row-chunk count of the two-pass column sum (fixes its scratch size).
int64_t colsum_chunks(int64_t rows, int64_t cols);

// out[c] = (accumulate ? out[c] : 0) + sum_r x[r * cols + c]; scratch of
// colsum_chunks(rows, cols) * cols elements.
template <typename T>
int colsum(const T* x, T* out, int64_t rows, int64_t cols, int accumulate, void* scratch,
           cudaStream_t stream);

}  // namespace tg
