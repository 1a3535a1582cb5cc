// GEMM argument block shared by the SIMT and tensor-core kernels.
#pragma once
#include "common.cuh"

namespace tg {

// Per-output-tile reduction ranges for the causal attention products (tensor-core path; the
// tile is 128 output rows starting at m0):
//   GEMM_K_UP_TO_ROW  -- reduce over k < m0 + 128 (operand zero beyond the diagonal tile)
//   GEMM_K_FROM_ROW   -- reduce over k >= m0 rounded down to 32 (operand zero before it)
//   GEMM_K_SKIP_UPPER -- full reduction, but tiles whose first column n0 > m0 + 127 are
//                        skipped (never written)
enum GemmKMode { GEMM_K_FULL = 0, GEMM_K_UP_TO_ROW = 1, GEMM_K_FROM_ROW = 2, GEMM_K_SKIP_UPPER = 3 };

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
  int kmode = GEMM_K_FULL;
  int precision = 0;  // 0: fp32-accurate (3xTF32 on the tensor cores); 1: plain TF32
};

template <typename T>
int gemm_simt(const GemmArgs<T>& p, cudaStream_t stream);

// tcgen05 3xTF32 path. Returns TG_ERR_UNSUPPORTED (without launching) when the operands'
// strides or base addresses do not meet the TMA's 16-byte rules, so the caller can fall back.
int gemm_tc_f32(const GemmArgs<float>& p, cudaStream_t stream);

}  // namespace tg
