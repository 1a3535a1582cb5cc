// Fused softmax attention, flash style (ops/attention.py:71-116, 163-272): the CUDA-core path
// (float64, and fp32 shapes the tensor-core path of attention_tc.cu does not take).
//
// Forward: per (batch, head, block of query rows), keys/values stream through shared memory
// in tiles; each query row keeps a running max, running sum and output accumulator, so P is
// never stored. The row's log-sum-exp is saved for the backward pass.
// Backward: delta_i = dO_i . O_i; then one kernel owns a block of keys and accumulates
// dK, dV over all query tiles, and one owns a block of queries and accumulates dQ; both
// recompute P from Q, K and the saved log-sum-exp. Nothing is accumulated with atomics, so
// results are deterministic.
//
// Each query (or key) row is handled by TPR consecutive lanes that own DPT = D / TPR of its
// dimensions; dot products are finished with xor-shuffles inside the lane group.
#include <stdlib.h>

#include <initializer_list>

#include "common.cuh"

namespace tg {
namespace {

constexpr int kThreads = 128;
// Keys (forward, dQ) or queries (dK/dV) per shared-memory tile: two tiles of D-wide rows
// stay within the 48 KB of static shared memory (32 KB at most).
template <typename T, int D>
constexpr int kTileV = sizeof(T) * D >= 2048 ? 8 : (sizeof(T) * D >= 1024 ? 16 : 32);

template <int TPR, typename T>
__device__ __forceinline__ T group_sum(T v) {
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct AttnDims {
  int64_t B, H, Tq, Tk, D;
  int64_t q_sb, q_sh, q_st, k_sb, k_sh, k_st, v_sb, v_sh, v_st, o_sb, o_sh, o_st;
  int causal;
  double scale;
};

// Load `rows` x D elements starting at row r0 of a strided (token-stride st) matrix into
// shared memory tile[kTile][D]; out-of-range rows are zero.
template <typename T, int D, int kTile>
__device__ __forceinline__ void load_tile(T* tile, const T* __restrict__ base, int64_t st,
                                          int64_t r0, int64_t nrows) {
  for (int e = threadIdx.x; e < kTile * D; e += kThreads) {
    const int r = e / D, c = e % D;
    const int64_t gr = r0 + r;
    tile[e] = gr < nrows ? base[gr * st + c] : T(0);
  }
}

template <typename T, int D, int DPT>
__global__ void __launch_bounds__(kThreads)
attn_fwd_kernel(AttnDims p, const T* __restrict__ Q, const T* __restrict__ K,
                const T* __restrict__ V, T* __restrict__ O, T* __restrict__ LSE) {
  constexpr int TPR = D / DPT;
  constexpr int RPB = kThreads / TPR;
  constexpr int kTile = kTileV<T, D>;
  __shared__ T Ks[kTile * D];
  __shared__ T Vs[kTile * D];
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t q0 = (int64_t)blockIdx.x * RPB;
  const int row = threadIdx.x / TPR, part = threadIdx.x % TPR;
  const int64_t i = q0 + row;
  const bool live = i < p.Tq;
  const T scale = (T)p.scale;
  const T* qb = Q + b * p.q_sb + h * p.q_sh;
  const T* kb = K + b * p.k_sb + h * p.k_sh;
  const T* vb = V + b * p.v_sb + h * p.v_sh;
  const int64_t shift = p.Tk - p.Tq;  // causal: key j visible iff j <= i + shift

  T q[DPT], acc[DPT];
#pragma unroll
  for (int d = 0; d < DPT; ++d) {
    q[d] = live ? qb[i * p.q_st + part * DPT + d] : T(0);
    acc[d] = T(0);
  }
  T m = T(-INFINITY), l = T(0);
  int64_t kend = p.Tk;
  if (p.causal) {
    const int64_t last = q0 + RPB - 1 + shift + 1;
    kend = last < p.Tk ? (last > 0 ? last : 0) : p.Tk;
  }
  for (int64_t k0 = 0; k0 < kend; k0 += kTile) {
    __syncthreads();
    load_tile<T, D, kTile>(Ks, kb, p.k_st, k0, p.Tk);
    load_tile<T, D, kTile>(Vs, vb, p.v_st, k0, p.Tk);
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < kTile; ++j) {
      const int64_t kj = k0 + j;
      T s = T(0);
#pragma unroll
      for (int d = 0; d < DPT; ++d) s += q[d] * Ks[j * D + part * DPT + d];
      s = group_sum<TPR>(s) * scale;
      const bool ok = kj < p.Tk && (!p.causal || kj <= i + shift);
      if (!ok) continue;
      if (s > m) {
        const T corr = dev_exp<T>(m - s);  // exp(-inf) = 0 on the first visible key
        l = l * corr + T(1);
#pragma unroll
        for (int d = 0; d < DPT; ++d) acc[d] = acc[d] * corr + Vs[j * D + part * DPT + d];
        m = s;
      } else {
        const T pj = dev_exp<T>(s - m);
        l += pj;
#pragma unroll
        for (int d = 0; d < DPT; ++d) acc[d] += pj * Vs[j * D + part * DPT + d];
      }
    }
  }
  if (!live) return;
  const T inv = T(1) / l;  // a fully masked row gives 0 * inf = NaN, as the reference does
  T* ob = O + b * p.o_sb + h * p.o_sh + i * p.o_st + part * DPT;
#pragma unroll
  for (int d = 0; d < DPT; ++d) ob[d] = acc[d] * inv;
  if (part == 0) LSE[bh * p.Tq + i] = m + dev_log<T>(l);
}

// delta_i = sum_d dO[i, d] * O[i, d]; one warp per row.
template <typename T>
__global__ void attn_delta_kernel(AttnDims p, const T* __restrict__ O, const T* __restrict__ dO,
                                  T* __restrict__ delta) {
  const int64_t rows = p.B * p.H * p.Tq;
  const int lane = threadIdx.x & 31;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t i = r % p.Tq, bh = r / p.Tq, b = bh / p.H, h = bh % p.H;
    const int64_t off = b * p.o_sb + h * p.o_sh + i * p.o_st;
    T s = T(0);
    for (int64_t d = lane; d < p.D; d += 32) s += dO[off + d] * O[off + d];
    s = warp_sum(s);
    if (lane == 0) delta[r] = s;
  }
}

// dK, dV for a block of keys: loop over query tiles.
template <typename T, int D, int DPT>
__global__ void __launch_bounds__(kThreads)
attn_bwd_dkdv_kernel(AttnDims p, const T* __restrict__ Q, const T* __restrict__ K,
                     const T* __restrict__ V, const T* __restrict__ dO,
                     const T* __restrict__ LSE, const T* __restrict__ delta,
                     T* __restrict__ dK, T* __restrict__ dV) {
  constexpr int TPR = D / DPT;
  constexpr int RPB = kThreads / TPR;
  constexpr int kTile = kTileV<T, D>;
  __shared__ T Qs[kTile * D];
  __shared__ T dOs[kTile * D];
  __shared__ T Ls[kTile], Ds[kTile];
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t j0 = (int64_t)blockIdx.x * RPB;
  const int row = threadIdx.x / TPR, part = threadIdx.x % TPR;
  const int64_t j = j0 + row;
  const bool live = j < p.Tk;
  const T scale = (T)p.scale;
  const int64_t shift = p.Tk - p.Tq;
  const T* qb = Q + b * p.q_sb + h * p.q_sh;
  const T* ob = dO + b * p.o_sb + h * p.o_sh;

  T k[DPT], v[DPT], dk[DPT], dv[DPT];
#pragma unroll
  for (int d = 0; d < DPT; ++d) {
    k[d] = live ? K[b * p.k_sb + h * p.k_sh + j * p.k_st + part * DPT + d] : T(0);
    v[d] = live ? V[b * p.v_sb + h * p.v_sh + j * p.v_st + part * DPT + d] : T(0);
    dk[d] = dv[d] = T(0);
  }
  // Causal: only queries i >= j - shift see key j; the block's first key bounds the start.
  int64_t istart = 0;
  if (p.causal) {
    istart = j0 - shift;
    if (istart < 0) istart = 0;
    istart = (istart / kTile) * kTile;
  }
  for (int64_t i0 = istart; i0 < p.Tq; i0 += kTile) {
    __syncthreads();
    load_tile<T, D, kTile>(Qs, qb, p.q_st, i0, p.Tq);
    load_tile<T, D, kTile>(dOs, ob, p.o_st, i0, p.Tq);
    if (threadIdx.x < kTile) {
      const int64_t gi = i0 + threadIdx.x;
      Ls[threadIdx.x] = gi < p.Tq ? LSE[bh * p.Tq + gi] : T(0);
      Ds[threadIdx.x] = gi < p.Tq ? delta[bh * p.Tq + gi] : T(0);
    }
    __syncthreads();
#pragma unroll 2
    for (int ii = 0; ii < kTile; ++ii) {
      const int64_t gi = i0 + ii;
      T s = T(0), dp = T(0);
#pragma unroll
      for (int d = 0; d < DPT; ++d) {
        s += Qs[ii * D + part * DPT + d] * k[d];
        dp += dOs[ii * D + part * DPT + d] * v[d];
      }
      s = group_sum<TPR>(s) * scale;
      dp = group_sum<TPR>(dp);
      const bool ok = gi < p.Tq && (!p.causal || j <= gi + shift);
      const T pr = ok ? dev_exp<T>(s - Ls[ii]) : T(0);
      const T ds = pr * (dp - Ds[ii]) * scale;
#pragma unroll
      for (int d = 0; d < DPT; ++d) {
        dv[d] += pr * dOs[ii * D + part * DPT + d];
        dk[d] += ds * Qs[ii * D + part * DPT + d];
      }
    }
  }
  if (!live) return;
  T* dkb = dK + b * p.k_sb + h * p.k_sh + j * p.k_st + part * DPT;
  T* dvb = dV + b * p.v_sb + h * p.v_sh + j * p.v_st + part * DPT;
#pragma unroll
  for (int d = 0; d < DPT; ++d) {
    dkb[d] = dk[d];
    dvb[d] = dv[d];
  }
}

// dQ for a block of queries: loop over key tiles.
template <typename T, int D, int DPT>
__global__ void __launch_bounds__(kThreads)
attn_bwd_dq_kernel(AttnDims p, const T* __restrict__ Q, const T* __restrict__ K,
                   const T* __restrict__ V, const T* __restrict__ dO, const T* __restrict__ LSE,
                   const T* __restrict__ delta, T* __restrict__ dQ) {
  constexpr int TPR = D / DPT;
  constexpr int RPB = kThreads / TPR;
  constexpr int kTile = kTileV<T, D>;
  __shared__ T Ks[kTile * D];
  __shared__ T Vs[kTile * D];
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t q0 = (int64_t)blockIdx.x * RPB;
  const int row = threadIdx.x / TPR, part = threadIdx.x % TPR;
  const int64_t i = q0 + row;
  const bool live = i < p.Tq;
  const T scale = (T)p.scale;
  const int64_t shift = p.Tk - p.Tq;
  const T* kb = K + b * p.k_sb + h * p.k_sh;
  const T* vb = V + b * p.v_sb + h * p.v_sh;
  T q[DPT], go[DPT], dq[DPT];
#pragma unroll
  for (int d = 0; d < DPT; ++d) {
    q[d] = live ? Q[b * p.q_sb + h * p.q_sh + i * p.q_st + part * DPT + d] : T(0);
    go[d] = live ? dO[b * p.o_sb + h * p.o_sh + i * p.o_st + part * DPT + d] : T(0);
    dq[d] = T(0);
  }
  const T lse = live ? LSE[bh * p.Tq + i] : T(0);
  const T dl = live ? delta[bh * p.Tq + i] : T(0);
  int64_t kend = p.Tk;
  if (p.causal) {
    const int64_t last = q0 + RPB - 1 + shift + 1;
    kend = last < p.Tk ? (last > 0 ? last : 0) : p.Tk;
  }
  for (int64_t k0 = 0; k0 < kend; k0 += kTile) {
    __syncthreads();
    load_tile<T, D, kTile>(Ks, kb, p.k_st, k0, p.Tk);
    load_tile<T, D, kTile>(Vs, vb, p.v_st, k0, p.Tk);
    __syncthreads();
#pragma unroll 2
    for (int jj = 0; jj < kTile; ++jj) {
      const int64_t kj = k0 + jj;
      T s = T(0), dp = T(0);
#pragma unroll
      for (int d = 0; d < DPT; ++d) {
        s += q[d] * Ks[jj * D + part * DPT + d];
        dp += go[d] * Vs[jj * D + part * DPT + d];
      }
      s = group_sum<TPR>(s) * scale;
      dp = group_sum<TPR>(dp);
      const bool ok = kj < p.Tk && (!p.causal || kj <= i + shift);
      const T pr = ok ? dev_exp<T>(s - lse) : T(0);
      const T ds = pr * (dp - dl) * scale;
#pragma unroll
      for (int d = 0; d < DPT; ++d) dq[d] += ds * Ks[jj * D + part * DPT + d];
    }
  }
  if (!live) return;
  T* dqb = dQ + b * p.q_sb + h * p.q_sh + i * p.q_st + part * DPT;
#pragma unroll
  for (int d = 0; d < DPT; ++d) dqb[d] = dq[d];
}

AttnDims make_dims(const tg_attn_shape* s) {
  AttnDims d;
  d.B = s->batch; d.H = s->heads; d.Tq = s->tq; d.Tk = s->tk; d.D = s->head_dim;
  d.q_sb = s->q_sb; d.q_sh = s->q_sh; d.q_st = s->q_st;
  d.k_sb = s->k_sb; d.k_sh = s->k_sh; d.k_st = s->k_st;
  d.v_sb = s->v_sb; d.v_sh = s->v_sh; d.v_st = s->v_st;
  d.o_sb = s->o_sb; d.o_sh = s->o_sh; d.o_st = s->o_st;
  d.causal = s->causal;
  d.scale = 1.0 / sqrt((double)s->head_dim);
  return d;
}

template <typename T, int D>
int attn_forward_d(const AttnDims& p, const T* q, const T* k, const T* v, T* o, T* lse,
                   cudaStream_t s) {
  constexpr int DPT = (sizeof(T) == 4 ? 16 : 8) < D ? (sizeof(T) == 4 ? 16 : 8) : D;
  constexpr int RPB = kThreads / (D / DPT);
  dim3 grid((unsigned)((p.Tq + RPB - 1) / RPB), (unsigned)(p.B * p.H));
  attn_fwd_kernel<T, D, DPT><<<grid, kThreads, 0, s>>>(p, q, k, v, o, lse);
  return check_launch("attention_forward");
}

template <typename T, int D>
int attn_backward_d(const AttnDims& p, const T* q, const T* k, const T* v, const T* o,
                    const T* lse, const T* dout, T* dq, T* dk, T* dv, T* delta, cudaStream_t s) {
  constexpr int DPT = (sizeof(T) == 4 ? 16 : 8) < D ? (sizeof(T) == 4 ? 16 : 8) : D;
  constexpr int RPB = kThreads / (D / DPT);
  attn_delta_kernel<T><<<grid_for(p.B * p.H * p.Tq * 32, 256), 256, 0, s>>>(p, o, dout, delta);
  dim3 gk((unsigned)((p.Tk + RPB - 1) / RPB), (unsigned)(p.B * p.H));
  attn_bwd_dkdv_kernel<T, D, DPT><<<gk, kThreads, 0, s>>>(p, q, k, v, dout, lse, delta, dk, dv);
  dim3 gq((unsigned)((p.Tq + RPB - 1) / RPB), (unsigned)(p.B * p.H));
  attn_bwd_dq_kernel<T, D, DPT><<<gq, kThreads, 0, s>>>(p, q, k, v, dout, lse, delta, dq);
  return check_launch("attention_backward", 3);
}

template <typename T>
int attn_forward_any(const AttnDims& p, const T* q, const T* k, const T* v, T* o, T* lse,
                     cudaStream_t s) {
  switch (p.D) {
    case 8: return attn_forward_d<T, 8>(p, q, k, v, o, lse, s);
    case 16: return attn_forward_d<T, 16>(p, q, k, v, o, lse, s);
    case 32: return attn_forward_d<T, 32>(p, q, k, v, o, lse, s);
    case 64: return attn_forward_d<T, 64>(p, q, k, v, o, lse, s);
    case 128: return attn_forward_d<T, 128>(p, q, k, v, o, lse, s);
    case 256: return attn_forward_d<T, 256>(p, q, k, v, o, lse, s);
  }
  return set_error(TG_ERR_UNSUPPORTED, "attention: head_dim %lld (supported 8/16/32/64/128/256)",
                   (long long)p.D);
}

template <typename T>
int attn_backward_any(const AttnDims& p, const T* q, const T* k, const T* v, const T* o,
                      const T* lse, const T* dout, T* dq, T* dk, T* dv, T* delta,
                      cudaStream_t s) {
  switch (p.D) {
    case 8: return attn_backward_d<T, 8>(p, q, k, v, o, lse, dout, dq, dk, dv, delta, s);
    case 16: return attn_backward_d<T, 16>(p, q, k, v, o, lse, dout, dq, dk, dv, delta, s);
    case 32: return attn_backward_d<T, 32>(p, q, k, v, o, lse, dout, dq, dk, dv, delta, s);
    case 64: return attn_backward_d<T, 64>(p, q, k, v, o, lse, dout, dq, dk, dv, delta, s);
    case 128: return attn_backward_d<T, 128>(p, q, k, v, o, lse, dout, dq, dk, dv, delta, s);
    case 256: return attn_backward_d<T, 256>(p, q, k, v, o, lse, dout, dq, dk, dv, delta, s);
  }
  return set_error(TG_ERR_UNSUPPORTED, "attention: head_dim %lld (supported 8/16/32/64/128/256)",
                   (long long)p.D);
}

// Head sizes without kernels of their own (up to 256) run on the next wider kernel over
// zero-padded contiguous copies: zero features add nothing to q.k, the padded value columns
// give output features that are dropped, and the scale stays 1/sqrt(head_dim).
int64_t padded_head(int64_t d) {
  for (int64_t w : {8, 16, 32, 64, 128, 256})
    if (d <= w) return w;
  return 0;
}

bool native_head(int64_t d) {
  return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256;
}

constexpr int kPadThreads = 256;

// dst (B, H, n, dp), contiguous = src (strides sb, sh, st; d features), zero beyond d.
template <typename T>
__global__ void __launch_bounds__(kPadThreads)
head_pad_kernel(const T* __restrict__ src, int64_t sb, int64_t sh, int64_t st,
                T* __restrict__ dst, int64_t H, int64_t n, int64_t d, int64_t dp,
                int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = e % dp, r = e / dp, t = r % n, bh = r / n;
    const int64_t b = bh / H, h = bh % H;
    dst[e] = c < d ? src[b * sb + h * sh + t * st + c] : T(0);
  }
}

// The first d features of src (B, H, n, dp), contiguous, into dst (strides sb, sh, st).
template <typename T>
__global__ void __launch_bounds__(kPadThreads)
head_unpad_kernel(const T* __restrict__ src, T* __restrict__ dst, int64_t sb, int64_t sh,
                  int64_t st, int64_t H, int64_t n, int64_t d, int64_t dp, int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = e % d, r = e / d, t = r % n, bh = r / n;
    const int64_t b = bh / H, h = bh % H;
    dst[b * sb + h * sh + t * st + c] = src[r * dp + c];
  }
}

template <typename T>
void head_pad(const T* src, int64_t sb, int64_t sh, int64_t st, T* dst, const AttnDims& p,
              int64_t n, int64_t dp, cudaStream_t s) {
  const int64_t total = p.B * p.H * n * dp;
  head_pad_kernel<T><<<grid_for(total, kPadThreads), kPadThreads, 0, s>>>(
      src, sb, sh, st, dst, p.H, n, p.D, dp, total);
}

template <typename T>
void head_unpad(const T* src, T* dst, int64_t sb, int64_t sh, int64_t st, const AttnDims& p,
                int64_t n, int64_t dp, cudaStream_t s) {
  const int64_t total = p.B * p.H * n * p.D;
  head_unpad_kernel<T><<<grid_for(total, kPadThreads), kPadThreads, 0, s>>>(
      src, dst, sb, sh, st, p.H, n, p.D, dp, total);
}

// `p` with head size dp and contiguous (B, H, T, dp) strides for every operand.
AttnDims padded_dims(const AttnDims& p, int64_t dp) {
  AttnDims c = p;
  c.D = dp;
  c.q_sb = c.o_sb = p.H * p.Tq * dp;
  c.q_sh = c.o_sh = p.Tq * dp;
  c.k_sb = c.v_sb = p.H * p.Tk * dp;
  c.k_sh = c.v_sh = p.Tk * dp;
  c.q_st = c.k_st = c.v_st = c.o_st = dp;
  return c;  // the scale stays 1/sqrt(p.D)
}

// Scratch of the padded path, in elements: forward q, o (Tq rows) and k, v (Tk rows);
// backward q, o, dout, dq and k, v, dk, dv.
int64_t padded_elems(const tg_attn_shape* s, int per_side) {
  const int64_t dp = padded_head(s->head_dim);
  return (int64_t)per_side * s->batch * s->heads * (s->tq + s->tk) * dp;
}

template <typename T>
int attn_forward_padded(const AttnDims& p, const T* q, const T* k, const T* v, T* o, T* lse,
                        void* scratch, cudaStream_t s) {
  const int64_t dp = padded_head(p.D);
  const int64_t nq = p.B * p.H * p.Tq * dp, nk = p.B * p.H * p.Tk * dp;
  T* qp = reinterpret_cast<T*>(scratch);
  T* op = qp + nq;
  T* kp = op + nq;
  T* vp = kp + nk;
  head_pad<T>(q, p.q_sb, p.q_sh, p.q_st, qp, p, p.Tq, dp, s);
  head_pad<T>(k, p.k_sb, p.k_sh, p.k_st, kp, p, p.Tk, dp, s);
  head_pad<T>(v, p.v_sb, p.v_sh, p.v_st, vp, p, p.Tk, dp, s);
  int r = check_launch("attention(pad)", 3);
  if (r) return r;
  r = attn_forward_any<T>(padded_dims(p, dp), qp, kp, vp, op, lse, s);
  if (r) return r;
  head_unpad<T>(op, o, p.o_sb, p.o_sh, p.o_st, p, p.Tq, dp, s);
  return check_launch("attention(unpad)");
}

template <typename T>
int attn_backward_padded(const AttnDims& p, const T* q, const T* k, const T* v, const T* o,
                         const T* lse, const T* dout, T* dq, T* dk, T* dv, T* delta,
                         T* pad, cudaStream_t s) {
  const int64_t dp = padded_head(p.D);
  const int64_t nq = p.B * p.H * p.Tq * dp, nk = p.B * p.H * p.Tk * dp;
  T* qp = pad;
  T* op = qp + nq;
  T* gop = op + nq;
  T* dqp = gop + nq;
  T* kp = dqp + nq;
  T* vp = kp + nk;
  T* dkp = vp + nk;
  T* dvp = dkp + nk;
  head_pad<T>(q, p.q_sb, p.q_sh, p.q_st, qp, p, p.Tq, dp, s);
  head_pad<T>(o, p.o_sb, p.o_sh, p.o_st, op, p, p.Tq, dp, s);
  head_pad<T>(dout, p.o_sb, p.o_sh, p.o_st, gop, p, p.Tq, dp, s);
  head_pad<T>(k, p.k_sb, p.k_sh, p.k_st, kp, p, p.Tk, dp, s);
  head_pad<T>(v, p.v_sb, p.v_sh, p.v_st, vp, p, p.Tk, dp, s);
  int r = check_launch("attention backward(pad)", 5);
  if (r) return r;
  r = attn_backward_any<T>(padded_dims(p, dp), qp, kp, vp, op, lse, gop, dqp, dkp, dvp, delta,
                           s);
  if (r) return r;
  head_unpad<T>(dqp, dq, p.q_sb, p.q_sh, p.q_st, p, p.Tq, dp, s);
  head_unpad<T>(dkp, dk, p.k_sb, p.k_sh, p.k_st, p, p.Tk, dp, s);
  head_unpad<T>(dvp, dv, p.v_sb, p.v_sh, p.v_st, p, p.Tk, dp, s);
  return check_launch("attention backward(unpad)", 3);
}

}  // namespace
}  // namespace tg

namespace tg {
// Tensor-core path (attention_tc.cu).
bool attention_tc_supported(int dtype, const tg_attn_shape* s);
size_t attention_tc_forward_scratch(const tg_attn_shape* s);
size_t attention_tc_backward_scratch(const tg_attn_shape* s);
int attention_tc_forward(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                         float* o, float* lse, void* scratch, cudaStream_t st);
int attention_tc_backward(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                          const float* o, const float* lse, const float* dout, float* dq,
                          float* dk, float* dv, void* scratch, cudaStream_t st);
}  // namespace tg

using namespace tg;

namespace {
// TG_ATTENTION=simt forces the CUDA-core kernels (a debugging switch for users).
bool use_tc(int dtype, const tg_attn_shape* s) {
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("TG_ATTENTION");
    forced = (e && e[0] == 's') ? 1 : 0;
  }
  return !forced && attention_tc_supported(dtype, s);
}

// The tensor maps also need 16-byte aligned base addresses (known only at the call).
bool aligned(std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return false;
  return true;
}
}  // namespace

extern "C" {

size_t tg_attention_forward_scratch_bytes(int dtype, const tg_attn_shape* s) {
  if (use_tc(dtype, s)) return attention_tc_forward_scratch(s);
  if (native_head(s->head_dim) || padded_head(s->head_dim) == 0) return 16;
  return (size_t)padded_elems(s, 2) * (dtype == TG_F64 ? 8 : 4) + 16;
}

int tg_attention_forward(int dtype, const tg_attn_shape* s, const void* q, const void* k,
                         const void* v, void* o, void* lse, void* scratch, void* stream) {
  TG_CHECK_ARG(s && s->batch >= 0 && s->heads >= 0 && s->tq >= 0 && s->tk >= 0,
               "attention: bad shape");
  if (s->batch * s->heads * s->tq == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  if (use_tc(dtype, s) && aligned({q, k, v, o})) {
    TG_CHECK_ARG(scratch, "attention_forward: NULL scratch");
    return attention_tc_forward(s, (const float*)q, (const float*)k, (const float*)v, (float*)o,
                                (float*)lse, scratch, st);
  }
  const AttnDims p = make_dims(s);
  if (!native_head(s->head_dim)) {
    if (padded_head(s->head_dim) == 0)
      return set_error(TG_ERR_UNSUPPORTED, "attention: head_dim %lld (at most 256 here)",
                       (long long)s->head_dim);
    TG_CHECK_ARG(scratch, "attention_forward: NULL scratch");
    return TG_DISPATCH_FLOAT(dtype, T, [&] {
      return attn_forward_padded<T>(p, (const T*)q, (const T*)k, (const T*)v, (T*)o, (T*)lse,
                                    scratch, st);
    });
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    return attn_forward_any<T>(p, (const T*)q, (const T*)k, (const T*)v, (T*)o, (T*)lse, st);
  });
}

size_t tg_attention_backward_scratch_bytes(int dtype, const tg_attn_shape* s) {
  if (use_tc(dtype, s)) return attention_tc_backward_scratch(s);
  const size_t es = dtype == TG_F64 ? 8 : 4;
  size_t bytes = (size_t)(s->batch * s->heads * s->tq) * es + 16;
  if (!native_head(s->head_dim) && padded_head(s->head_dim) != 0)
    bytes += 256 + (size_t)padded_elems(s, 4) * es;
  return bytes;
}

int tg_attention_backward(int dtype, const tg_attn_shape* s, const void* q, const void* k,
                          const void* v, const void* o, const void* lse, const void* dout,
                          void* dq, void* dk, void* dv, void* scratch, void* stream) {
  TG_CHECK_ARG(s && scratch, "attention_backward: NULL shape or scratch");
  if (s->batch * s->heads * (s->tq + s->tk) == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  if (use_tc(dtype, s) && aligned({q, k, v, o, dout, dq, dk, dv}))
    return attention_tc_backward(s, (const float*)q, (const float*)k, (const float*)v,
                                 (const float*)o, (const float*)lse, (const float*)dout,
                                 (float*)dq, (float*)dk, (float*)dv, scratch, st);
  const AttnDims p = make_dims(s);
  if (!native_head(s->head_dim)) {
    if (padded_head(s->head_dim) == 0)
      return set_error(TG_ERR_UNSUPPORTED, "attention: head_dim %lld (at most 256 here)",
                       (long long)s->head_dim);
    return TG_DISPATCH_FLOAT(dtype, T, [&] {
      // delta (B H Tq) first, the padded copies from the next 256-byte boundary.
      const size_t off = ((size_t)(p.B * p.H * p.Tq) * sizeof(T) + 255) & ~(size_t)255;
      T* pad = reinterpret_cast<T*>(reinterpret_cast<uint8_t*>(scratch) + off);
      return attn_backward_padded<T>(p, (const T*)q, (const T*)k, (const T*)v, (const T*)o,
                                     (const T*)lse, (const T*)dout, (T*)dq, (T*)dk, (T*)dv,
                                     (T*)scratch, pad, st);
    });
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    return attn_backward_any<T>(p, (const T*)q, (const T*)k, (const T*)v, (const T*)o,
                                (const T*)lse, (const T*)dout, (T*)dq, (T*)dk, (T*)dv,
                                (T*)scratch, st);
  });
}

}  // extern "C"
