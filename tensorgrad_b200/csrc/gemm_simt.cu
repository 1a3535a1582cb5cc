// CUDA-core (SIMT) GEMM: C = alpha * op(A) op(B) + beta * C (+ bias), fp32 and fp64.
//
// The accuracy reference for the tensor-core path and the kernel for shapes whose strides
// the TMA cannot describe (rows not 16-byte aligned) and for the float64 build mode. Classic
// register-blocked tiling: a BM x BN tile per 256-thread block, TM x TN outputs per thread,
// BK-deep slices of A and B staged in shared memory. Accumulation is in the element type,
// in ascending k order.
#include "common.cuh"
#include "gemm.cuh"

namespace tg {
namespace {

template <typename T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmArgs<T> p) {
  __shared__ T As[BK][BM + 4];
  __shared__ T Bs[BK][BN + 4];
  const int64_t bz = blockIdx.z;
  const int64_t bo = bz / p.heads, bh = bz % p.heads;
  const T* __restrict__ A = p.a + (p.a_fold > 0 ? 0 : bo * p.stride_a + bh * p.stride_ah);
  const T* __restrict__ B = p.b + bo * p.stride_b + bh * p.stride_bh;
  T* __restrict__ C = p.c;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);

  T acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = T(0);

  for (int64_t k0 = 0; k0 < p.k; k0 += BK) {
    // A slice: BM x BK elements; element e -> (row, kk). For trans_a = 0 the kk index runs
    // fastest so that neighbouring threads read neighbouring addresses.
#pragma unroll
    for (int e = tid; e < BM * BK; e += 256) {
      int r, kk;
      if (p.trans_a) { kk = e / BM; r = e % BM; } else { r = e / BK; kk = e % BK; }
      const int64_t gi = m0 + r, gk = k0 + kk;
      T v = T(0);
      if (gi < p.m && gk < p.k) {
        if (p.a_fold > 0) v = A[(gk / p.a_fold) * p.stride_a + gi * p.lda + gk % p.a_fold];
        else v = p.trans_a ? A[gk * p.lda + gi] : A[gi * p.lda + gk];
      }
      As[kk][r] = v;
    }
#pragma unroll
    for (int e = tid; e < BN * BK; e += 256) {
      int c, kk;
      if (p.trans_b) { c = e / BK; kk = e % BK; } else { kk = e / BN; c = e % BN; }
      const int64_t gj = n0 + c, gk = k0 + kk;
      T v = T(0);
      if (gj < p.n && gk < p.k) v = p.trans_b ? B[gj * p.ldb + gk] : B[gk * p.ldb + gj];
      Bs[kk][c] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      T ra[TM], rb[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) ra[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) rb[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fma(ra[i], rb[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t gi = m0 + ty * TM + i;
    if (gi >= p.m) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t gj = n0 + tx * TN + j;
      if (gj >= p.n) continue;
      const int64_t off = gemm_c_offset(p, bz, gi, gj);
      T v = p.alpha * acc[i][j];
      if (p.beta != T(0)) v += p.beta * C[off];
      if (p.bias) v += p.bias[gj];
      C[off] = v;
    }
  }
}

}  // namespace

template <typename T>
int gemm_simt(const GemmArgs<T>& p, cudaStream_t stream) {
  if (p.m == 0 || p.n == 0) return TG_OK;
  if (sizeof(T) == 4) {
    constexpr int BM = 128, BN = 128, BK = 8;
    dim3 grid((unsigned)((p.n + BN - 1) / BN), (unsigned)((p.m + BM - 1) / BM), (unsigned)p.batch);
    gemm_simt_kernel<T, BM, BN, BK, 8, 8><<<grid, 256, 0, stream>>>(p);
  } else {
    constexpr int BM = 64, BN = 64, BK = 8;
    dim3 grid((unsigned)((p.n + BN - 1) / BN), (unsigned)((p.m + BM - 1) / BM), (unsigned)p.batch);
    gemm_simt_kernel<T, BM, BN, BK, 4, 4><<<grid, 256, 0, stream>>>(p);
  }
  return check_launch("gemm_simt");
}

template int gemm_simt<float>(const GemmArgs<float>&, cudaStream_t);
template int gemm_simt<double>(const GemmArgs<double>&, cudaStream_t);

}  // namespace tg
