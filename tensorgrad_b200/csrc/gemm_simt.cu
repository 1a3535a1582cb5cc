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

// Products whose reduction is at most kSmallK long (an LSTM/GRU input projection from 2
// inputs: 51200 x 2048 outputs from k = 2): the output dominates the bytes, so each thread
// writes 4 consecutive columns of one row, from the row's k values (a warp shares its row)
// and B's k x 4 block (L1 hits: B is k x n), with fp32/fp64 FMAs in k order.
constexpr int kSmallK = 8;

template <typename T>
__global__ void __launch_bounds__(256) gemm_smallk_kernel(GemmArgs<T> p, bool vec) {
  const int64_t nq = (p.n + 3) / 4;
  const int64_t total = p.m * nq;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / nq;
    const int64_t c0 = (i - row * nq) * 4;
    T a[kSmallK];
#pragma unroll
    for (int k = 0; k < kSmallK; ++k)
      a[k] = k < p.k ? (p.trans_a ? p.a[k * p.lda + row] : p.a[row * p.lda + k]) : T(0);
    T acc[4] = {T(0), T(0), T(0), T(0)};
#pragma unroll
    for (int k = 0; k < kSmallK; ++k) {
      if (k >= p.k) break;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t col = c0 + j < p.n ? c0 + j : p.n - 1;
        const T bkj = p.trans_b ? p.b[col * p.ldb + k] : p.b[k * p.ldb + col];
        acc[j] = fma(a[k], bkj, acc[j]);
      }
    }
    T* crow = p.c + row * p.ldc;
    T v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = c0 + j;
      v[j] = p.alpha * acc[j];
      if (col < p.n) {
        if (p.beta != T(0)) v[j] += p.beta * crow[col];
        if (p.bias) v[j] += p.bias[col];
      }
    }
    if constexpr (sizeof(T) == 4) {
      if (vec && c0 + 4 <= p.n) {
        *reinterpret_cast<float4*>(crow + c0) = make_float4(v[0], v[1], v[2], v[3]);
        continue;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (c0 + j < p.n) crow[c0 + j] = v[j];
  }
}

}  // namespace

template <typename T>
bool gemm_smallk_applies(const GemmArgs<T>& p) {
  return p.k >= 1 && p.k <= kSmallK && p.batch == 1 && p.heads == 1 && p.c_hw == 0 &&
         p.a_fold == 0 && p.epi == GEMM_EPI_STORE && p.kmode == GEMM_K_FULL;
}

template <typename T>
int gemm_smallk(const GemmArgs<T>& p, cudaStream_t stream) {
  if (p.m == 0 || p.n == 0) return TG_OK;
  const bool vec = sizeof(T) == 4 && p.ldc % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(p.c) & 15) == 0;
  const int64_t work = p.m * ((p.n + 3) / 4);
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0) {
      cudaGetLastError();
      sms = 148;
    }
  }
  const int64_t cap = (int64_t)sms * 16;
  const int blocks = (int)((work + 255) / 256 < cap ? (work + 255) / 256 : cap);
  gemm_smallk_kernel<T><<<blocks, 256, 0, stream>>>(p, vec);
  return check_launch("gemm_smallk");
}

template bool gemm_smallk_applies<float>(const GemmArgs<float>&);
template bool gemm_smallk_applies<double>(const GemmArgs<double>&);
template int gemm_smallk<float>(const GemmArgs<float>&, cudaStream_t);
template int gemm_smallk<double>(const GemmArgs<double>&, cudaStream_t);

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
