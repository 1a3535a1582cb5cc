// GEMM argument block shared by the SIMT and tensor-core kernels.
#pragma once
#include "common.cuh"

namespace tg {

template <typename T>
struct GemmArgs {
  int64_t m, n, k;
  const T* a;
  int64_t lda, stride_a;
  const T* b;
  int64_t ldb, stride_b;
  T* c;
  int64_t ldc, stride_c;
  const T* bias;
  T alpha, beta;
  int trans_a, trans_b;
  int64_t batch;
};

template <typename T>
int gemm_simt(const GemmArgs<T>& p, cudaStream_t stream);

// tcgen05 3xTF32 path. Returns TG_ERR_UNSUPPORTED (without launching) when the operands'
// strides or base addresses do not meet the TMA's 16-byte rules, so the caller can fall back.
int gemm_tc_f32(const GemmArgs<float>& p, cudaStream_t stream);

}  // namespace tg
