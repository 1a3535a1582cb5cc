// Attention on the tensor cores (fp32 operands, 3xTF32 GEMMs), for ops/attention.py:71-116.
//
// Per (batch, head) the score products are batched tcgen05 GEMMs; between them, warp-per-row
// kernels do the softmax work:
//   forward : S = scale Q K^T  ->  P = softmax(S) row-wise (saving lse)  ->  O = P V
//   backward: S = scale Q K^T, dP = dO V^T  ->  P = exp(S - lse), dS = P (dP - delta) scale
//             ->  dV = P^T dO, dQ = dS K, dK = dS^T Q
// The backward recomputes P from the forward's log-sum-exp instead of keeping P (the
// reference keeps it); S/P/dP/dS live in scratch for one op call only. With a causal mask
// (equal query and key lengths) the GEMM skips score tiles above the diagonal and limits the
// reductions to the triangle; the row kernels write every entry of a row up to the end of
// its 128-wide diagonal tile (zeros past the diagonal), which is exactly what those
// reductions read. Q/K/V/dO are first gathered into contiguous (B*H, T, D) blocks (the packed
// QKV projection is strided); gradients are scattered back the same way.
#include "common.cuh"
#include "gemm.cuh"

namespace tg {
namespace {

constexpr int kDiag = 128;  // GEMM output tile rows: the causal band granularity

struct Plan {
  int64_t B, H, Tq, Tk, D, BH, ldS;
  size_t blk_q, blk_k, blk_s;  // floats per contiguous block
};

Plan make_plan(const tg_attn_shape* s) {
  Plan p;
  p.B = s->batch; p.H = s->heads; p.Tq = s->tq; p.Tk = s->tk; p.D = s->head_dim;
  p.BH = p.B * p.H;
  p.ldS = (p.Tk + 3) / 4 * 4;  // 16-byte rows: S/P/dS are TMA operands of the next GEMMs
  p.blk_q = (size_t)(p.BH * p.Tq * p.D);
  p.blk_k = (size_t)(p.BH * p.Tk * p.D);
  p.blk_s = (size_t)(p.BH * p.Tq * p.ldS);
  return p;
}

// dst (B*H, T, D) contiguous <- src viewed through (batch, head, token) strides.
__global__ void gather_rows_kernel(const float* __restrict__ src, int64_t sb, int64_t sh,
                                   int64_t st, float* __restrict__ dst, int64_t H, int64_t T,
                                   int64_t D, int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = e % D, r = e / D, t = r % T, bh = r / T;
    dst[e] = src[(bh / H) * sb + (bh % H) * sh + t * st + d];
  }
}

__global__ void scatter_rows_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                    int64_t sb, int64_t sh, int64_t st, int64_t H, int64_t T,
                                    int64_t D, int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = e % D, r = e / D, t = r % T, bh = r / T;
    dst[(bh / H) * sb + (bh % H) * sh + t * st + d] = src[e];
  }
}

__device__ __forceinline__ int64_t row_valid(int64_t i, int64_t Tk, int causal) {
  return causal ? i + 1 : Tk;
}
__device__ __forceinline__ int64_t row_written(int64_t i, int64_t Tk, int causal) {
  if (!causal) return Tk;
  const int64_t e = (i / kDiag + 1) * kDiag;
  return e < Tk ? e : Tk;
}

// Row-wise softmax of S in place, one warp per row; lse[row] = max + log(sum).
__global__ void softmax_rows_kernel(float* __restrict__ S, int64_t ldS, float* __restrict__ lse,
                                    int64_t Tq, int64_t Tk, int causal, int64_t rows) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float* s = S + r * ldS;
    const int64_t i = r % Tq;
    const int64_t valid = row_valid(i, Tk, causal), written = row_written(i, Tk, causal);
    float m = -INFINITY, l = 0.f;
    for (int64_t k = lane; k < valid; k += 32) {
      const float x = s[k];
      if (x > m) {
        l = l * expf(m - x) + 1.f;
        m = x;
      } else {
        l += expf(x - m);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
      const float mm = fmaxf(m, m2);
      l = (mm == -INFINITY) ? 0.f : l * expf(m - mm) + l2 * expf(m2 - mm);
      m = mm;
    }
    const float inv = 1.f / l;
    for (int64_t k = lane; k < written; k += 32) s[k] = k < valid ? expf(s[k] - m) * inv : 0.f;
    if (lane == 0) lse[r] = m + logf(l);
  }
}

// P = exp(S - lse) and dS = P (dP - delta) scale, in place (S <- P, dP <- dS).
__global__ void softmax_bwd_rows_kernel(float* __restrict__ S, float* __restrict__ dP,
                                        int64_t ldS, const float* __restrict__ lse,
                                        const float* __restrict__ delta, int64_t Tq, int64_t Tk,
                                        int causal, float scale, int64_t rows) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float* s = S + r * ldS;
    float* dp = dP + r * ldS;
    const int64_t i = r % Tq;
    const int64_t valid = row_valid(i, Tk, causal), written = row_written(i, Tk, causal);
    const float l = lse[r], dl = delta[r];
    for (int64_t k = lane; k < written; k += 32) {
      const float p = k < valid ? expf(s[k] - l) : 0.f;
      s[k] = p;
      dp[k] = p * (dp[k] - dl) * scale;
    }
  }
}

// delta[row] = dO[row] . O[row] over contiguous (rows, D) blocks.
__global__ void row_dot_kernel(const float* __restrict__ a, const float* __restrict__ b,
                               float* __restrict__ out, int64_t rows, int64_t D) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float acc = 0.f;
    for (int64_t d = lane; d < D; d += 32) acc += a[r * D + d] * b[r * D + d];
    acc = warp_sum(acc);
    if (lane == 0) out[r] = acc;
  }
}

int gather(const float* src, int64_t sb, int64_t sh, int64_t st, float* dst, int64_t H, int64_t T,
           int64_t D, int64_t BH, cudaStream_t s) {
  const int64_t total = BH * T * D;
  gather_rows_kernel<<<grid_for(total, 256), 256, 0, s>>>(src, sb, sh, st, dst, H, T, D, total);
  return check_launch("attention gather");
}

int scatter(const float* src, float* dst, int64_t sb, int64_t sh, int64_t st, int64_t H, int64_t T,
            int64_t D, int64_t BH, cudaStream_t s) {
  const int64_t total = BH * T * D;
  scatter_rows_kernel<<<grid_for(total, 256), 256, 0, s>>>(src, dst, sb, sh, st, H, T, D, total);
  return check_launch("attention scatter");
}

// Batched C_i = alpha op(A_i) op(B_i) on the tensor-core path.
int bgemm(int ta, int tb, int64_t m, int64_t n, int64_t k, float alpha, const float* a,
          int64_t lda, int64_t sa, const float* b, int64_t ldb, int64_t sb, float* c, int64_t ldc,
          int64_t sc, int64_t batch, int kmode, cudaStream_t s) {
  GemmArgs<float> p;
  p.m = m; p.n = n; p.k = k;
  p.a = a; p.lda = lda; p.stride_a = sa;
  p.b = b; p.ldb = ldb; p.stride_b = sb;
  p.c = c; p.ldc = ldc; p.stride_c = sc;
  p.bias = nullptr; p.alpha = alpha; p.beta = 0.f;
  p.trans_a = ta; p.trans_b = tb; p.batch = batch; p.kmode = kmode;
  // attention_tc_supported() guarantees the tensor-core path's alignment rules; the causal
  // k-ranges are only meaningful there, so a refusal is an error, not a fallback.
  return gemm_tc_profiled(p, s);
}

}  // namespace

bool attention_tc_supported(int dtype, const tg_attn_shape* s) {
  return dtype == TG_F32 && s->head_dim % 4 == 0 && s->head_dim <= 256 &&
         (!s->causal || s->tq == s->tk) && s->batch * s->heads <= 65535;
}

size_t attention_tc_forward_scratch(const tg_attn_shape* s) {
  const Plan p = make_plan(s);
  return (2 * p.blk_q + 2 * p.blk_k + p.blk_s) * sizeof(float) + 2048;
}

size_t attention_tc_backward_scratch(const tg_attn_shape* s) {
  const Plan p = make_plan(s);
  return (3 * p.blk_q + 4 * p.blk_k + 2 * p.blk_s + p.BH * p.Tq) * sizeof(float) + 4096;
}

static float* carve(char*& cur, size_t floats) {
  float* out = reinterpret_cast<float*>(cur);
  cur += (floats * sizeof(float) + 255) / 256 * 256;
  return out;
}

int attention_tc_forward(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                         float* o, float* lse, void* scratch, cudaStream_t st) {
  const Plan p = make_plan(s);
  char* cur = reinterpret_cast<char*>(scratch);
  float* Qc = carve(cur, p.blk_q);
  float* Kc = carve(cur, p.blk_k);
  float* Vc = carve(cur, p.blk_k);
  float* Oc = carve(cur, p.blk_q);
  float* S = carve(cur, p.blk_s);
  const int causal = s->causal;
  const float scale = (float)(1.0 / sqrt((double)p.D));
  int rc;
  if ((rc = gather(q, s->q_sb, s->q_sh, s->q_st, Qc, p.H, p.Tq, p.D, p.BH, st))) return rc;
  if ((rc = gather(k, s->k_sb, s->k_sh, s->k_st, Kc, p.H, p.Tk, p.D, p.BH, st))) return rc;
  if ((rc = gather(v, s->v_sb, s->v_sh, s->v_st, Vc, p.H, p.Tk, p.D, p.BH, st))) return rc;
  // S = scale Q K^T  (K stored Tk x D: the "n x k" operand)
  if ((rc = bgemm(0, 1, p.Tq, p.Tk, p.D, scale, Qc, p.D, p.Tq * p.D, Kc, p.D, p.Tk * p.D, S, p.ldS,
                  p.Tq * p.ldS, p.BH, causal ? GEMM_K_SKIP_UPPER : GEMM_K_FULL, st)))
    return rc;
  const int64_t rows = p.BH * p.Tq;
  softmax_rows_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(S, p.ldS, lse, p.Tq, p.Tk, causal,
                                                                rows);
  if ((rc = check_launch("attention softmax"))) return rc;
  // O = P V  (V stored Tk x D: the "k x n" operand)
  if ((rc = bgemm(0, 0, p.Tq, p.D, p.Tk, 1.f, S, p.ldS, p.Tq * p.ldS, Vc, p.D, p.Tk * p.D, Oc, p.D,
                  p.Tq * p.D, p.BH, causal ? GEMM_K_UP_TO_ROW : GEMM_K_FULL, st)))
    return rc;
  return scatter(Oc, o, s->o_sb, s->o_sh, s->o_st, p.H, p.Tq, p.D, p.BH, st);
}

int attention_tc_backward(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                          const float* o, const float* lse, const float* dout, float* dq,
                          float* dk, float* dv, void* scratch, cudaStream_t st) {
  const Plan p = make_plan(s);
  char* cur = reinterpret_cast<char*>(scratch);
  float* Qc = carve(cur, p.blk_q);
  float* Kc = carve(cur, p.blk_k);
  float* Vc = carve(cur, p.blk_k);
  float* dOc = carve(cur, p.blk_q);
  float* Oc = carve(cur, p.blk_q);
  float* S = carve(cur, p.blk_s);
  float* dP = carve(cur, p.blk_s);
  float* delta = carve(cur, (size_t)(p.BH * p.Tq));
  float* dQc = Oc;  // O is only needed for delta
  float* dKc = carve(cur, p.blk_k);
  float* dVc = carve(cur, p.blk_k);
  const int causal = s->causal;
  const float scale = (float)(1.0 / sqrt((double)p.D));
  const int64_t rows = p.BH * p.Tq;
  int rc;
  if ((rc = gather(q, s->q_sb, s->q_sh, s->q_st, Qc, p.H, p.Tq, p.D, p.BH, st))) return rc;
  if ((rc = gather(k, s->k_sb, s->k_sh, s->k_st, Kc, p.H, p.Tk, p.D, p.BH, st))) return rc;
  if ((rc = gather(v, s->v_sb, s->v_sh, s->v_st, Vc, p.H, p.Tk, p.D, p.BH, st))) return rc;
  if ((rc = gather(dout, s->o_sb, s->o_sh, s->o_st, dOc, p.H, p.Tq, p.D, p.BH, st))) return rc;
  if ((rc = gather(o, s->o_sb, s->o_sh, s->o_st, Oc, p.H, p.Tq, p.D, p.BH, st))) return rc;
  row_dot_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(dOc, Oc, delta, rows, p.D);
  if ((rc = check_launch("attention delta"))) return rc;
  const int skip = causal ? GEMM_K_SKIP_UPPER : GEMM_K_FULL;
  if ((rc = bgemm(0, 1, p.Tq, p.Tk, p.D, scale, Qc, p.D, p.Tq * p.D, Kc, p.D, p.Tk * p.D, S, p.ldS,
                  p.Tq * p.ldS, p.BH, skip, st)))
    return rc;
  if ((rc = bgemm(0, 1, p.Tq, p.Tk, p.D, 1.f, dOc, p.D, p.Tq * p.D, Vc, p.D, p.Tk * p.D, dP, p.ldS,
                  p.Tq * p.ldS, p.BH, skip, st)))
    return rc;
  softmax_bwd_rows_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(S, dP, p.ldS, lse, delta,
                                                                    p.Tq, p.Tk, causal, scale,
                                                                    rows);
  if ((rc = check_launch("attention softmax backward"))) return rc;
  const int up = causal ? GEMM_K_UP_TO_ROW : GEMM_K_FULL;
  const int from = causal ? GEMM_K_FROM_ROW : GEMM_K_FULL;
  // dV = P^T dO: P stored Tq x Tk is the "k x m" operand.
  if ((rc = bgemm(1, 0, p.Tk, p.D, p.Tq, 1.f, S, p.ldS, p.Tq * p.ldS, dOc, p.D, p.Tq * p.D, dVc,
                  p.D, p.Tk * p.D, p.BH, from, st)))
    return rc;
  // dQ = dS K: K stored Tk x D is the "k x n" operand.
  if ((rc = bgemm(0, 0, p.Tq, p.D, p.Tk, 1.f, dP, p.ldS, p.Tq * p.ldS, Kc, p.D, p.Tk * p.D, dQc,
                  p.D, p.Tq * p.D, p.BH, up, st)))
    return rc;
  // dK = dS^T Q
  if ((rc = bgemm(1, 0, p.Tk, p.D, p.Tq, 1.f, dP, p.ldS, p.Tq * p.ldS, Qc, p.D, p.Tq * p.D, dKc,
                  p.D, p.Tk * p.D, p.BH, from, st)))
    return rc;
  if ((rc = scatter(dQc, dq, s->q_sb, s->q_sh, s->q_st, p.H, p.Tq, p.D, p.BH, st))) return rc;
  if ((rc = scatter(dKc, dk, s->k_sb, s->k_sh, s->k_st, p.H, p.Tk, p.D, p.BH, st))) return rc;
  return scatter(dVc, dv, s->v_sb, s->v_sh, s->v_st, p.H, p.Tk, p.D, p.BH, st);
}

}  // namespace tg
