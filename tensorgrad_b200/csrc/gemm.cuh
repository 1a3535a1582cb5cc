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
enum GemmEpilogue { GEMM_EPI_STORE = 0, GEMM_EPI_SOFTMAX_DS = 1, GEMM_EPI_SOFTMAX_P = 2 };

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
  // Convolution addressing (0 = plain row-major operands):
  //   a_fold > 0: the reduction index of a K-major A (trans_a == 0) folds as
  //               k = q * a_fold + r -> element (m, k) at a + q * stride_a + m * lda + r,
  //               so k may run over images of an NCHW tensor (A itself is then not batched).
  //   c_hw > 0  : C(m, n) of batch entry bz at c + bz * stride_ch + (m / c_hw) * stride_c +
  //               n * ldc + (m % c_hw): the GEMM row is image * hw + pixel and the column a
  //               channel, written as NCHW (column-major tiles; heads must be 1).
  int64_t a_fold = 0;
  int64_t c_hw = 0;
  // Batch entries split as (outer, head) with bz = outer * heads + head; each operand is
  // addressed at outer * stride_x + head * stride_xh (attention over (B, H, T, D) views with
  // arbitrary strides, e.g. the packed QKV projection). heads == 1: plain batch strides.
  int64_t heads = 1;
  int64_t stride_ah = 0, stride_bh = 0, stride_ch = 0;
  // Epilogue (tensor-core path), for the attention backward besides GEMM_EPI_STORE:
  //   GEMM_EPI_SOFTMAX_P : C = P = exp(alpha * acc - rv0[row]) with rv0 = lse per output row
  //                        (index bz * m + row), zero above the diagonal when kmode is
  //                        GEMM_K_SKIP_UPPER (the scores S = alpha Q K^T are never stored);
  //   GEMM_EPI_SOFTMAX_DS: C = dS = P (acc - rv1[row]) alpha with P read from `aux` (same
  //                        layout as C) and rv1 = delta per output row.
  int epi = 0;
  const T* rv0 = nullptr;
  const T* rv1 = nullptr;
  T* aux = nullptr;
  // Split-K partials (tensor-core path, batch 1): with a workspace of workspace_bytes the
  // reduction may be split over more CTAs, each writing an fp32 partial, summed in split
  // order by a second kernel (deterministic). nullptr: no split.
  float* workspace = nullptr;
  size_t workspace_bytes = 0;
};

// Address of C(m, n) of batch entry bz under the layouts above.
template <typename T>
__host__ __device__ __forceinline__ int64_t gemm_c_offset(const GemmArgs<T>& p, int64_t bz,
                                                          int64_t m, int64_t n) {
  if (p.c_hw > 0) return bz * p.stride_ch + (m / p.c_hw) * p.stride_c + n * p.ldc + (m % p.c_hw);
  return (bz / p.heads) * p.stride_c + (bz % p.heads) * p.stride_ch + m * p.ldc + n;
}

template <typename T>
int gemm_simt(const GemmArgs<T>& p, cudaStream_t stream);
// Reductions of at most 8 (memory-bound outer products) on the CUDA cores.
template <typename T>
bool gemm_smallk_applies(const GemmArgs<T>& p);
template <typename T>
int gemm_smallk(const GemmArgs<T>& p, cudaStream_t stream);

// The library's GEMM: the tensor-core kernel for fp32 where the TMA can address the
// operands, the SIMT kernel otherwise (and for fp64); live-profiled like tg_gemm.
template <typename T>
int gemm_run(const GemmArgs<T>& p, cudaStream_t stream);

// The tensor-core kernel alone (no SIMT fallback), live-profiled like gemm_run.
int gemm_tc_profiled(const GemmArgs<float>& p, cudaStream_t stream);

// tcgen05 3xTF32 path. Returns TG_ERR_UNSUPPORTED (without launching) when the operands'
// strides or base addresses do not meet the TMA's 16-byte rules, so the caller can fall back.
int gemm_tc_f32(const GemmArgs<float>& p, cudaStream_t stream);

}  // namespace tg
