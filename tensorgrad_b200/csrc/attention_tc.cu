// Attention on the tensor cores (fp32 operands, 3xTF32 GEMMs), for ops/attention.py:71-116.
//
// Per (batch, head) the products are batched tcgen05 GEMMs that read Q, K, V, O and dO in
// place through 4-D tensor maps (batch, head, token and feature strides: the packed QKV
// projection needs no gather) and write O, dQ, dK, dV straight into their strided outputs:
//   forward : S = scale Q K^T  ->  P = softmax(S) row-wise (saving lse)  ->  O = P V
//   backward: S = scale Q K^T;  dP = dO V^T with the softmax VJP in its epilogue:
//             P = exp(S - lse) over S, dS = P (dP - delta) scale, delta = rowsum(dO o O);
//             then dV = P^T dO, dQ = dS K, dK = dS^T Q
// The backward recomputes P from the forward's log-sum-exp instead of keeping P (the
// reference keeps it); S/P/dP/dS live in scratch for one op call only. With a causal mask
// (equal query and key lengths) the GEMMs skip score tiles above the diagonal and limit the
// reductions to the triangle; the softmax kernel and the epilogue write every entry of a row
// up to the end of its 128-wide diagonal tile (zeros past the diagonal), which is exactly
// what those reductions read.
#include "common.cuh"
#include "gemm.cuh"

namespace tg {
namespace {

constexpr int kDiag = 128;  // GEMM output tile rows: the causal band granularity

struct Plan {
  int64_t B, H, Tq, Tk, D, BH, ldS;
  size_t blk_s;  // floats of one (B*H, Tq, ldS) score block
};

Plan make_plan(const tg_attn_shape* s) {
  Plan p;
  p.B = s->batch; p.H = s->heads; p.Tq = s->tq; p.Tk = s->tk; p.D = s->head_dim;
  p.BH = p.B * p.H;
  p.ldS = (p.Tk + 3) / 4 * 4;  // 16-byte rows: S/P/dS are TMA operands of the next GEMMs
  p.blk_s = (size_t)(p.BH * p.Tq * p.ldS);
  return p;
}

// A (B, H, T, D) operand seen through element strides (batch, head, token; features dense).
struct View {
  const float* p;
  int64_t sb, sh, st;
};

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

// The same softmax with the row in registers (rows of up to 128 * NV keys): one 16-byte read
// and one 16-byte write per element, the maximum and the sum from registers.
template <int NV>
__global__ void __launch_bounds__(256)
softmax_rows_vec4(float* __restrict__ S, int64_t ldS, float* __restrict__ lse, int64_t Tq,
                  int64_t Tk, int causal, int64_t rows) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float4* s4 = reinterpret_cast<float4*>(S + r * ldS);
    const int64_t i = r % Tq;
    const int64_t valid = row_valid(i, Tk, causal), written = row_written(i, Tk, causal);
    const int64_t nv = (valid + 3) >> 2, nw = (written + 3) >> 2;
    float4 v[NV];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int64_t q = lane + 32 * j;
      v[j] = q < nv ? s4[q] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const int64_t c = 4 * q;
      if (c + 0 >= valid) v[j].x = -INFINITY;
      if (c + 1 >= valid) v[j].y = -INFINITY;
      if (c + 2 >= valid) v[j].z = -INFINITY;
      if (c + 3 >= valid) v[j].w = -INFINITY;
      m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
    }
    m = warp_max(m);
    float l = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      v[j].x = expf(v[j].x - m); v[j].y = expf(v[j].y - m);
      v[j].z = expf(v[j].z - m); v[j].w = expf(v[j].w - m);
      l += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    l = warp_sum(l);
    const float inv = 1.f / l;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int64_t q = lane + 32 * j;
      if (q < nw)
        s4[q] = make_float4(v[j].x * inv, v[j].y * inv, v[j].z * inv, v[j].w * inv);
    }
    if (lane == 0) lse[r] = m + logf(l);
  }
}

// delta[(b*H + h)*T + t] = dO[b, h, t, :] . O[b, h, t, :], one warp per row.
__global__ void row_dot_kernel(View a, View b, float* __restrict__ out, int64_t H, int64_t T,
                               int64_t D, int64_t rows) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t t = r % T, bh = r / T, bi = bh / H, hi = bh % H;
    const float* x = a.p + bi * a.sb + hi * a.sh + t * a.st;
    const float* y = b.p + bi * b.sb + hi * b.sh + t * b.st;
    float acc = 0.f;
    for (int64_t d = lane; d < D; d += 32) acc += x[d] * y[d];
    acc = warp_sum(acc);
    if (lane == 0) out[r] = acc;
  }
}

// The same with 16-byte loads: G = D / 4 lanes per row (D a multiple of 4, at most 128; the
// tensor-core path's strides are 16-byte multiples), 32 / G rows per warp, the row's dot
// product reduced within its lane group.
template <int G>
__global__ void __launch_bounds__(256)
row_dot_vec4_kernel(View a, View b, float* __restrict__ out, int64_t H, int64_t T, int64_t rows) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  constexpr int kRowsPerWarp = 32 / G;
  const int lane = threadIdx.x & 31, sub = lane / G, c = lane % G;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
       w * kRowsPerWarp < rows; w += warps) {
    const int64_t r = w * kRowsPerWarp + sub;
    float acc = 0.f;
    if (r < rows) {
      const int64_t t = r % T, bh = r / T, bi = bh / H, hi = bh % H;
      const float4 x = reinterpret_cast<const float4*>(a.p + bi * a.sb + hi * a.sh + t * a.st)[c];
      const float4 y = reinterpret_cast<const float4*>(b.p + bi * b.sb + hi * b.sh + t * b.st)[c];
      acc = (x.x * y.x + x.y * y.y) + (x.z * y.z + x.w * y.w);
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (r < rows && c == 0) out[r] = acc;
  }
}

int row_dot(View dO, View O, float* delta, const Plan& p, cudaStream_t st) {
  const int64_t rows = p.BH * p.Tq;
  const bool vec = p.D % 4 == 0 && p.D <= 128 &&
                   (reinterpret_cast<uintptr_t>(dO.p) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(O.p) & 15) == 0;
  if (!vec) {
    row_dot_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(dO, O, delta, p.H, p.Tq, p.D, rows);
    return check_launch("attention delta");
  }
  const int g = (int)(p.D / 4);
  const int64_t per_warp = 32 / (g >= 32 ? 32 : (g >= 16 ? 16 : (g >= 8 ? 8 : (g >= 4 ? 4 : (g >= 2 ? 2 : 1)))));
  const unsigned grid = (unsigned)grid_for((rows + per_warp - 1) / per_warp * 32, 256);
  switch (g) {
    case 32: launch_pdl(row_dot_vec4_kernel<32>, dim3(grid), dim3(256), 0, st, dO, O, delta, p.H,
                         p.Tq, rows); break;
    case 16: launch_pdl(row_dot_vec4_kernel<16>, dim3(grid), dim3(256), 0, st, dO, O, delta, p.H,
                         p.Tq, rows); break;
    case 8: launch_pdl(row_dot_vec4_kernel<8>, dim3(grid), dim3(256), 0, st, dO, O, delta, p.H,
                         p.Tq, rows); break;
    case 4: launch_pdl(row_dot_vec4_kernel<4>, dim3(grid), dim3(256), 0, st, dO, O, delta, p.H,
                         p.Tq, rows); break;
    case 2: row_dot_vec4_kernel<2><<<grid, 256, 0, st>>>(dO, O, delta, p.H, p.Tq, rows); break;
    case 1: row_dot_vec4_kernel<1><<<grid, 256, 0, st>>>(dO, O, delta, p.H, p.Tq, rows); break;
    default:
      row_dot_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(dO, O, delta, p.H, p.Tq, p.D, rows);
  }
  return check_launch("attention delta");
}

View score_view(const Plan& p, const float* base) {
  return View{base, p.H * p.Tq * p.ldS, p.Tq * p.ldS, p.ldS};
}

// Batched C_(b,h) = alpha op(A_(b,h)) op(B_(b,h)) over (batch, head) views, on the
// tensor-core path.
GemmArgs<float> bgemm_args(int ta, int tb, int64_t m, int64_t n, int64_t k, float alpha, View a,
                           View b, View c, const Plan& p, int kmode) {
  GemmArgs<float> g;
  g.m = m; g.n = n; g.k = k;
  g.a = a.p; g.lda = a.st; g.stride_a = a.sb; g.stride_ah = a.sh;
  g.b = b.p; g.ldb = b.st; g.stride_b = b.sb; g.stride_bh = b.sh;
  g.c = const_cast<float*>(c.p); g.ldc = c.st; g.stride_c = c.sb; g.stride_ch = c.sh;
  g.bias = nullptr; g.alpha = alpha; g.beta = 0.f;
  g.trans_a = ta; g.trans_b = tb; g.batch = p.BH; g.heads = p.H; g.kmode = kmode;
  return g;
}

// attention_tc_supported() guarantees the tensor-core path's alignment rules; the causal
// k-ranges are only meaningful there, so a refusal is an error, not a fallback.
int bgemm(const GemmArgs<float>& g, cudaStream_t s) { return gemm_tc_profiled(g, s); }

bool strides_ok(int64_t sb, int64_t sh, int64_t st) {
  return sb % 4 == 0 && sh % 4 == 0 && st % 4 == 0;
}

}  // namespace

bool attention_tc_supported(int dtype, const tg_attn_shape* s) {
  return dtype == TG_F32 && s->head_dim % 4 == 0 && s->head_dim <= 256 &&
         (!s->causal || s->tq == s->tk) && s->batch * s->heads <= 65535 &&
         strides_ok(s->q_sb, s->q_sh, s->q_st) && strides_ok(s->k_sb, s->k_sh, s->k_st) &&
         strides_ok(s->v_sb, s->v_sh, s->v_st) && strides_ok(s->o_sb, s->o_sh, s->o_st);
}

// Heads of 32 or 64 features take the fused kernels (flash_tc.cu).
bool flash_fwd_supported(const tg_attn_shape* s);

size_t attention_tc_forward_scratch(const tg_attn_shape* s) {
  if (flash_fwd_supported(s)) return 256;  // the fused forward keeps its scores on chip
  const Plan p = make_plan(s);
  return p.blk_s * sizeof(float) + 512;
}

size_t attention_tc_backward_scratch(const tg_attn_shape* s) {
  const Plan p = make_plan(s);
  return (2 * p.blk_s + p.BH * p.Tq) * sizeof(float) + 1024;
}

static float* carve(char*& cur, size_t floats) {
  float* out = reinterpret_cast<float*>(cur);
  cur += (floats * sizeof(float) + 255) / 256 * 256;
  return out;
}

// The fused kernels (flash_tc.cu), heads of 32 or 64 features (flash_fwd_supported, declared
// above): the forward, and P with dS of the backward.
int flash_fwd_tc(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                 float* o, float* lse, cudaStream_t st);
int attn_pds_tc(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                const float* dout, const float* lse, const float* delta, float* P, float* dS,
                int64_t ldS, cudaStream_t st);

int attention_tc_forward(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                         float* o, float* lse, void* scratch, cudaStream_t st) {
  if (flash_fwd_supported(s)) return flash_fwd_tc(s, q, k, v, o, lse, st);
  const Plan p = make_plan(s);
  char* cur = reinterpret_cast<char*>(scratch);
  float* S = carve(cur, p.blk_s);
  const int causal = s->causal;
  const float scale = (float)(1.0 / sqrt((double)p.D));
  const View Q{q, s->q_sb, s->q_sh, s->q_st}, K{k, s->k_sb, s->k_sh, s->k_st};
  const View V{v, s->v_sb, s->v_sh, s->v_st}, O{o, s->o_sb, s->o_sh, s->o_st};
  const View Sv = score_view(p, S);
  int rc;
  // S = scale Q K^T  (K stored Tk x D: the "n x k" operand)
  if ((rc = bgemm(bgemm_args(0, 1, p.Tq, p.Tk, p.D, scale, Q, K, Sv, p,
                             causal ? GEMM_K_SKIP_UPPER : GEMM_K_FULL), st)))
    return rc;
  const int64_t rows = p.BH * p.Tq;
  const unsigned grid = grid_for(rows * 32, 256, 148 * 64);
  const int64_t nv = (p.Tk + 127) / 128;  // float4 per lane for a whole row
  if (nv <= 1) softmax_rows_vec4<1><<<grid, 256, 0, st>>>(S, p.ldS, lse, p.Tq, p.Tk, causal, rows);
  else if (nv <= 2) softmax_rows_vec4<2><<<grid, 256, 0, st>>>(S, p.ldS, lse, p.Tq, p.Tk, causal, rows);
  else if (nv <= 4) softmax_rows_vec4<4><<<grid, 256, 0, st>>>(S, p.ldS, lse, p.Tq, p.Tk, causal, rows);
  else if (nv <= 8) softmax_rows_vec4<8><<<grid, 256, 0, st>>>(S, p.ldS, lse, p.Tq, p.Tk, causal, rows);
  else softmax_rows_kernel<<<grid, 256, 0, st>>>(S, p.ldS, lse, p.Tq, p.Tk, causal, rows);
  if ((rc = check_launch("attention softmax"))) return rc;
  // O = P V  (V stored Tk x D: the "k x n" operand)
  return bgemm(bgemm_args(0, 0, p.Tq, p.D, p.Tk, 1.f, Sv, V, O, p,
                          causal ? GEMM_K_UP_TO_ROW : GEMM_K_FULL), st);
}

int attention_tc_backward(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                          const float* o, const float* lse, const float* dout, float* dq,
                          float* dk, float* dv, void* scratch, cudaStream_t st) {
  const Plan p = make_plan(s);
  char* cur = reinterpret_cast<char*>(scratch);
  float* S = carve(cur, p.blk_s);
  float* dP = carve(cur, p.blk_s);
  float* delta = carve(cur, (size_t)(p.BH * p.Tq));
  const int causal = s->causal;
  const float scale = (float)(1.0 / sqrt((double)p.D));
  const int64_t rows = p.BH * p.Tq;
  const View Q{q, s->q_sb, s->q_sh, s->q_st}, K{k, s->k_sb, s->k_sh, s->k_st};
  const View V{v, s->v_sb, s->v_sh, s->v_st}, O{o, s->o_sb, s->o_sh, s->o_st};
  const View dO{dout, s->o_sb, s->o_sh, s->o_st};
  const View dQ{dq, s->q_sb, s->q_sh, s->q_st}, dK{dk, s->k_sb, s->k_sh, s->k_st};
  const View dV{dv, s->v_sb, s->v_sh, s->v_st};
  const View Sv = score_view(p, S), dPv = score_view(p, dP);
  int rc;
  if ((rc = row_dot(dO, O, delta, p, st))) return rc;
  const int skip = causal ? GEMM_K_SKIP_UPPER : GEMM_K_FULL;
  if (flash_fwd_supported(s)) {
    // Both score products on chip, P and dS written once (heads of 32 / 64).
    if ((rc = attn_pds_tc(s, q, k, v, dout, lse, delta, S, dP, p.ldS, st))) return rc;
  } else {
    // P = exp(scale Q K^T - lse) straight from the product's epilogue (the scores are never
    // stored), then dP = dO V^T with dS = P (dP - delta) scale produced by its epilogue.
    GemmArgs<float> gp = bgemm_args(0, 1, p.Tq, p.Tk, p.D, scale, Q, K, Sv, p, skip);
    gp.epi = GEMM_EPI_SOFTMAX_P;
    gp.rv0 = lse;
    if ((rc = bgemm(gp, st))) return rc;
    GemmArgs<float> g = bgemm_args(0, 1, p.Tq, p.Tk, p.D, scale, dO, V, dPv, p, skip);
    g.epi = GEMM_EPI_SOFTMAX_DS;
    g.rv1 = delta;
    g.aux = S;
    if ((rc = bgemm(g, st))) return rc;
  }
  const int up = causal ? GEMM_K_UP_TO_ROW : GEMM_K_FULL;
  const int from = causal ? GEMM_K_FROM_ROW : GEMM_K_FULL;
  // dV = P^T dO: P stored Tq x Tk is the "k x m" operand.
  if ((rc = bgemm(bgemm_args(1, 0, p.Tk, p.D, p.Tq, 1.f, Sv, dO, dV, p, from), st))) return rc;
  // dQ = dS K: K stored Tk x D is the "k x n" operand.
  if ((rc = bgemm(bgemm_args(0, 0, p.Tq, p.D, p.Tk, 1.f, dPv, K, dQ, p, up), st))) return rc;
  // dK = dS^T Q
  return bgemm(bgemm_args(1, 0, p.Tk, p.D, p.Tq, 1.f, dPv, Q, dK, p, from), st);
}

}  // namespace tg
