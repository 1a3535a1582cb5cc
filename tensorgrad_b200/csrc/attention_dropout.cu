// Attention with dropout on the attention weights (ops/attention.py:59-116, 163-272 with
// dropout_p > 0 in training), fp32 and float64.
//
// The reference draws one keep-mask over the whole (B, H, Tq, Tk) probability array from its
// global PCG64 generator before the forward (_random.py:53-70) and uses the same mask in the
// VJP. Here the mask is never stored: the host passes the generator's state before that draw
// and both directions regenerate the mask on the device (pcg64.cuh), element e = ((b H + h)
// Tq + i) Tk + j using 16-bit word e of the stream, exactly as the reference views it.
//
// The products are the library's batched GEMMs over (batch, head) views (tensor cores for
// fp32, SIMT for float64), and the probabilities are materialised in `scratch` for the call:
//   forward : S = scale Q K^T; P = softmax(S) (causal/length mask; lse saved);
//             W = P o m (m = keep_scale where kept, else 0); O = W V
//   backward: S, P again (the same kernels, so the same P); W = P o m; dV = W^T dO;
//             dW = dO V^T; dP' = dW o m; dS = P o (dP' - rowsum(P o dP')) scale;
//             dQ = dS K; dK = dS^T Q
// which is the reference's attention_backward with its `ds *= keep; ds *= keep_scale` step.
#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"
#include "pcg64.cuh"

namespace tg {
namespace {

struct DropDims {
  int64_t B, H, Tq, Tk, D, BH, ld;  // ld: row stride of the (BH, Tq, ld) score blocks
  int causal;
};

DropDims dims_of(const tg_attn_shape* s, int dtype) {
  DropDims d;
  d.B = s->batch; d.H = s->heads; d.Tq = s->tq; d.Tk = s->tk; d.D = s->head_dim;
  d.BH = d.B * d.H;
  d.ld = dtype == TG_F32 ? (d.Tk + 3) / 4 * 4 : d.Tk;  // 16-byte rows for the TMA
  d.causal = s->causal;
  return d;
}

// Keys visible to query row i: j <= i + (Tk - Tq) when causal.
__device__ __forceinline__ int64_t visible(int64_t i, int64_t Tq, int64_t Tk, int causal) {
  if (!causal) return Tk;
  const int64_t v = i + 1 + (Tk - Tq);
  return v < 0 ? 0 : (v > Tk ? Tk : v);
}

// Row softmax of S (rows of the (BH, Tq, ld) block) in place, masked entries 0; lse per row.
// One warp per row; the maximum and the sum as the reference forms them (max, exp(s - max),
// sum, divide).
template <typename T>
__global__ void __launch_bounds__(256)
softmax_masked_rows(T* __restrict__ S, T* __restrict__ lse, DropDims d) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = d.BH * d.Tq;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    T* s = S + r * d.ld;
    const int64_t vis = visible(r % d.Tq, d.Tq, d.Tk, d.causal);
    T m = -INFINITY;
    for (int64_t k = lane; k < vis; k += 32) m = s[k] > m ? s[k] : m;
    m = warp_max(m);
    if (!(m > -INFINITY)) m = T(0);  // a row with no visible key: exp(-inf - 0) = 0
    T l = T(0);
    for (int64_t k = lane; k < vis; k += 32) l += dev_exp<T>(s[k] - m);
    l = warp_sum(l);
    const T inv = T(1) / l;
    for (int64_t k = lane; k < d.Tk; k += 32) s[k] = k < vis ? dev_exp<T>(s[k] - m) * inv : T(0);
    if (lane == 0) lse[r] = m + dev_log<T>(l);
  }
}

// dst[r, j] = src[r, j] * (keep(r Tk + j) ? keep_scale : 0) over the (BH Tq, Tk) block.
template <typename T>
__global__ void __launch_bounds__(256)
apply_keep_rows(const T* __restrict__ src, T* __restrict__ dst, DropDims d, uint64_t s_hi,
                uint64_t s_lo, uint64_t inc_hi, uint64_t inc_lo, uint32_t threshold, T scale) {
  const int64_t n = d.BH * d.Tq * d.Tk, words = (n + 3) / 4;
  const pcg::u128 s0 = pcg::make128(s_hi, s_lo), inc = pcg::make128(inc_hi, inc_lo);
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words;
       w += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t bits = pcg::output_at(s0, inc, (uint64_t)w);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t e = 4 * w + q;
      if (e < n) {
        const int64_t r = e / d.Tk, j = e - r * d.Tk;
        const uint32_t u = (uint32_t)(bits >> (16 * q)) & 0xFFFFu;
        dst[r * d.ld + j] = src[r * d.ld + j] * (u >= threshold ? scale : T(0));
      }
    }
  }
}

// dS = P o (dP' - rowsum(P o dP')) scale, in place over dP'.
template <typename T>
__global__ void __launch_bounds__(256)
ds_rows(const T* __restrict__ P, T* __restrict__ dP, DropDims d, T scale) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = d.BH * d.Tq;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const T* p = P + r * d.ld;
    T* g = dP + r * d.ld;
    T acc = T(0);
    for (int64_t k = lane; k < d.Tk; k += 32) acc += g[k] * p[k];
    acc = warp_sum(acc);
    for (int64_t k = lane; k < d.Tk; k += 32) g[k] = p[k] * (g[k] - acc) * scale;
  }
}

template <typename T>
struct V4 {  // a (B, H, T, D) operand through element strides
  const T* p;
  int64_t sb, sh, st;
};

template <typename T>
int bmm(int ta, int tb, int64_t m, int64_t n, int64_t k, T alpha, V4<T> a, V4<T> b, V4<T> c,
        const DropDims& d, cudaStream_t st) {
  GemmArgs<T> g;
  g.m = m; g.n = n; g.k = k;
  g.a = a.p; g.lda = a.st; g.stride_a = a.sb; g.stride_ah = a.sh;
  g.b = b.p; g.ldb = b.st; g.stride_b = b.sb; g.stride_bh = b.sh;
  g.c = const_cast<T*>(c.p); g.ldc = c.st; g.stride_c = c.sb; g.stride_ch = c.sh;
  g.bias = nullptr; g.alpha = alpha; g.beta = T(0);
  g.trans_a = ta; g.trans_b = tb;
  g.batch = d.BH; g.heads = d.H;
  return gemm_run<T>(g, st);
}

int rows_grid(int64_t rows) {
  return (int)std::min<int64_t>(std::max<int64_t>((rows + 7) / 8, 1), 148 * 16);
}

template <typename T>
V4<T> scores(const DropDims& d, const T* base) {
  return V4<T>{base, d.H * d.Tq * d.ld, d.Tq * d.ld, d.ld};
}

template <typename T>
int drop_forward(const tg_attn_shape* s, const DropDims& d, const T* q, const T* k, const T* v,
                 T* o, T* lse, const uint64_t* pcg, uint32_t threshold, double keep_scale,
                 T* S, cudaStream_t st) {
  const T scale = (T)(1.0 / sqrt((double)d.D));
  const V4<T> Q{q, s->q_sb, s->q_sh, s->q_st}, K{k, s->k_sb, s->k_sh, s->k_st};
  const V4<T> Vv{v, s->v_sb, s->v_sh, s->v_st}, O{o, s->o_sb, s->o_sh, s->o_st};
  int rc = bmm<T>(0, 1, d.Tq, d.Tk, d.D, scale, Q, K, scores<T>(d, S), d, st);
  if (rc) return rc;
  softmax_masked_rows<T><<<rows_grid(d.BH * d.Tq), 256, 0, st>>>(S, lse, d);
  const int64_t words = (d.BH * d.Tq * d.Tk + 3) / 4;
  const int g = (int)std::min<int64_t>((words + 255) / 256, 148 * 8);
  apply_keep_rows<T><<<g, 256, 0, st>>>(S, S, d, pcg[0], pcg[1], pcg[2], pcg[3], threshold,
                                       (T)keep_scale);
  rc = check_launch("attention dropout forward", 2);
  if (rc) return rc;
  return bmm<T>(0, 0, d.Tq, d.D, d.Tk, T(1), scores<T>(d, S), Vv, O, d, st);
}

template <typename T>
int drop_backward(const tg_attn_shape* s, const DropDims& d, const T* q, const T* k, const T* v,
                  const T* dout, T* dq, T* dk, T* dv, const uint64_t* pcg, uint32_t threshold,
                  double keep_scale, T* P, T* W, T* lse, cudaStream_t st) {
  const T scale = (T)(1.0 / sqrt((double)d.D));
  const V4<T> Q{q, s->q_sb, s->q_sh, s->q_st}, K{k, s->k_sb, s->k_sh, s->k_st};
  const V4<T> Vv{v, s->v_sb, s->v_sh, s->v_st}, dO{dout, s->o_sb, s->o_sh, s->o_st};
  const V4<T> dQ{dq, s->q_sb, s->q_sh, s->q_st}, dK{dk, s->k_sb, s->k_sh, s->k_st};
  const V4<T> dV{dv, s->v_sb, s->v_sh, s->v_st};
  const int64_t words = (d.BH * d.Tq * d.Tk + 3) / 4;
  const int g = (int)std::min<int64_t>((words + 255) / 256, 148 * 8);
  int rc = bmm<T>(0, 1, d.Tq, d.Tk, d.D, scale, Q, K, scores<T>(d, P), d, st);
  if (rc) return rc;
  softmax_masked_rows<T><<<rows_grid(d.BH * d.Tq), 256, 0, st>>>(P, lse, d);
  apply_keep_rows<T><<<g, 256, 0, st>>>(P, W, d, pcg[0], pcg[1], pcg[2], pcg[3], threshold,
                                       (T)keep_scale);
  if ((rc = check_launch("attention dropout backward", 2))) return rc;
  if ((rc = bmm<T>(1, 0, d.Tk, d.D, d.Tq, T(1), scores<T>(d, W), dO, dV, d, st))) return rc;
  if ((rc = bmm<T>(0, 1, d.Tq, d.Tk, d.D, T(1), dO, Vv, scores<T>(d, W), d, st))) return rc;
  apply_keep_rows<T><<<g, 256, 0, st>>>(W, W, d, pcg[0], pcg[1], pcg[2], pcg[3], threshold,
                                       (T)keep_scale);
  ds_rows<T><<<rows_grid(d.BH * d.Tq), 256, 0, st>>>(P, W, d, scale);
  if ((rc = check_launch("attention dropout backward", 2))) return rc;
  if ((rc = bmm<T>(0, 0, d.Tq, d.D, d.Tk, T(1), scores<T>(d, W), K, dQ, d, st))) return rc;
  return bmm<T>(1, 0, d.Tk, d.D, d.Tq, T(1), scores<T>(d, W), Q, dK, d, st);
}

size_t block_bytes(const DropDims& d, int dtype) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  return ((size_t)(d.BH * d.Tq * d.ld) * es + 255) / 256 * 256;
}

int check_shape(int dtype, const tg_attn_shape* s) {
  TG_CHECK_ARG(dtype == TG_F32 || dtype == TG_F64, "attention dropout: dtype %d", dtype);
  TG_CHECK_ARG(s != nullptr && s->batch > 0 && s->heads > 0 && s->tq > 0 && s->tk > 0 &&
                   s->head_dim > 0,
               "attention dropout: empty shape");
  return TG_OK;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

size_t tg_attention_dropout_scratch_bytes(int dtype, const tg_attn_shape* s) {
  if (check_shape(dtype, s) != TG_OK) return 0;
  const DropDims d = dims_of(s, dtype);
  const size_t es = dtype == TG_F64 ? 8 : 4;
  return 2 * block_bytes(d, dtype) + ((size_t)(d.BH * d.Tq) * es + 255) / 256 * 256;
}

int tg_attention_forward_dropout(int dtype, const tg_attn_shape* s, const void* q, const void* k,
                                 const void* v, void* o, void* lse, const uint64_t* pcg_state,
                                 uint32_t threshold, double keep_scale, void* scratch,
                                 void* stream) {
  int rc = check_shape(dtype, s);
  if (rc) return rc;
  TG_CHECK_ARG(pcg_state && scratch && threshold <= 65536, "attention dropout: bad arguments");
  const DropDims d = dims_of(s, dtype);
  cudaStream_t st = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    return drop_forward<T>(s, d, (const T*)q, (const T*)k, (const T*)v, (T*)o, (T*)lse,
                           pcg_state, threshold, keep_scale, (T*)scratch, st);
  });
}

int tg_attention_backward_dropout(int dtype, const tg_attn_shape* s, const void* q,
                                  const void* k, const void* v, const void* dout, void* dq,
                                  void* dk, void* dv, const uint64_t* pcg_state,
                                  uint32_t threshold, double keep_scale, void* scratch,
                                  void* stream) {
  int rc = check_shape(dtype, s);
  if (rc) return rc;
  TG_CHECK_ARG(pcg_state && scratch && threshold <= 65536, "attention dropout: bad arguments");
  const DropDims d = dims_of(s, dtype);
  cudaStream_t st = as_stream(stream);
  char* base = reinterpret_cast<char*>(scratch);
  const size_t blk = block_bytes(d, dtype);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    return drop_backward<T>(s, d, (const T*)q, (const T*)k, (const T*)v, (const T*)dout,
                            (T*)dq, (T*)dk, (T*)dv, pcg_state, threshold, keep_scale,
                            (T*)base, (T*)(base + blk), (T*)(base + 2 * blk), st);
  });
}

}  // extern "C"
