// Conv2d, BatchNorm (training mode) and MaxPool2d of the CNN path (ops/conv.py,
// ops/layers.py:144-189).
//
// Convolution = im2col patch matrix + the library GEMM (tcgen05 3xTF32 for fp32):
//   forward : y (NCHW) = cols W^T + b, the GEMM epilogue scattering rows (image, pixel) and
//             columns (channel) straight into NCHW, so no transpose pass;
//   weight  : dW = G^T cols, the reduction index running over (image, pixel) of the NCHW
//             gradient (a folded A operand), split over CTAs into a workspace when the
//             output has few tiles (c_out x c*kh*kw is small, the reduction is long);
//   input   : dcols = G W per image (A read MN-major from NCHW, W shared by the batch), then
//             col2im as a gather over the kernel offsets (no atomics: deterministic).
// Batch-norm statistics and the reductions of its VJP are per-channel sums accumulated in
// float64 per thread and block, combined in chunk order (deterministic).
#include "common.cuh"
#include "gemm.cuh"

namespace tg {
namespace {

constexpr int kThreads = 256;

inline int64_t cols_ld(const tg_conv_shape& s) { return (s.c * s.kh * s.kw + 3) / 4 * 4; }

inline size_t align256(size_t b) { return (b + 255) / 256 * 256; }

int check_conv(const tg_conv_shape* s, bool pool) {
  TG_CHECK_ARG(s, "conv2d: null shape");
  TG_CHECK_ARG(s->n >= 0 && s->c > 0 && s->h > 0 && s->w > 0 && s->kh > 0 && s->kw > 0 &&
                   s->sh > 0 && s->sw > 0 && s->ph >= 0 && s->pw >= 0 && (pool || s->c_out > 0),
               "conv2d: bad shape");
  TG_CHECK_ARG(s->c_out <= 65535, "conv2d: at most 65535 output channels");
  TG_CHECK_ARG(s->oh ==(s->h + 2 * s->ph - s->kh) / s->sh + 1 &&
                   s->ow == (s->w + 2 * s->pw - s->kw) / s->sw + 1 && s->oh > 0 && s->ow > 0,
               "conv2d: output size does not match the input, kernel, stride and padding");
  return TG_OK;
}

// ------------------------------------------------------------------ im2col / col2im
// cols[m][kk], m = (img, oy, ox), kk = (ch, i, j) < c*kh*kw, zero elsewhere. One thread per
// element of a row-major patch matrix: the stores are coalesced (the matrix is ~kh*kw times
// the input, so its writes dominate the traffic).
template <typename T>
__global__ void __launch_bounds__(kThreads)
im2col_kernel(const T* __restrict__ x, T* __restrict__ cols, tg_conv_shape s, int64_t ld) {
  const int64_t total = s.n * s.oh * s.ow * ld;
  const int64_t K = s.c * s.kh * s.kw;
  const int64_t khw = s.kh * s.kw, ohw = s.oh * s.ow;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = idx / ld, kk = idx - m * ld;
    T v = T(0);
    if (kk < K) {
      const int64_t ch = kk / khw, r = kk - ch * khw;
      const int64_t i = r / s.kw, j = r - i * s.kw;
      const int64_t img = m / ohw, p = m - img * ohw;
      const int64_t oy = p / s.ow, ox = p - oy * s.ow;
      const int64_t iy = oy * s.sh - s.ph + i, ix = ox * s.sw - s.pw + j;
      if (iy >= 0 && iy < s.h && ix >= 0 && ix < s.w)
        v = x[((img * s.c + ch) * s.h + iy) * s.w + ix];
    }
    cols[idx] = v;
  }
}

// dx[img][ch][y][x] = sum over kernel offsets (i, j) whose window covers (y, x) of
// dcols[(img, oy, ox)][(ch, i, j)], in ascending (i, j) (the reference's col2im order).
template <typename T>
__global__ void __launch_bounds__(kThreads)
col2im_kernel(const T* __restrict__ dcols, T* __restrict__ gx, tg_conv_shape s, int64_t ld) {
  const int64_t total = s.n * s.c * s.h * s.w;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t xw = idx % s.w;
    int64_t rest = idx / s.w;
    const int64_t yh = rest % s.h;
    rest /= s.h;
    const int64_t ch = rest % s.c, img = rest / s.c;
    T acc = T(0);
    for (int64_t i = 0; i < s.kh; ++i) {
      const int64_t ty = yh + s.ph - i;
      if (ty < 0 || ty % s.sh) continue;
      const int64_t oy = ty / s.sh;
      if (oy >= s.oh) continue;
      for (int64_t j = 0; j < s.kw; ++j) {
        const int64_t tx = xw + s.pw - j;
        if (tx < 0 || tx % s.sw) continue;
        const int64_t ox = tx / s.sw;
        if (ox >= s.ow) continue;
        acc += dcols[((img * s.oh + oy) * s.ow + ox) * ld + (ch * s.kh + i) * s.kw + j];
      }
    }
    gx[idx] = acc;
  }
}

// W (c_out, K) -> Wp (c_out, ld) with zero columns K..ld-1.
template <typename T>
__global__ void pad_rows_kernel(const T* __restrict__ w, T* __restrict__ wp, int64_t rows,
                                int64_t K, int64_t ld) {
  const int64_t total = rows * ld;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / ld, k = idx - r * ld;
    wp[idx] = k < K ? w[r * K + k] : T(0);
  }
}

// ------------------------------------------------------------------ per-channel sums
// Data (n, C, hw). Block (chunk, ch) sums images [chunk*n/chunks, (chunk+1)*n/chunks) of
// channel ch; partial[(ch * chunks + chunk) * 2 + {0, 1}] receives two float64 sums:
//   MODE_STATS: sum (x - x0), sum (x - x0)^2 with x0 = the channel's first element (a shift
//               that keeps the variance free of cancellation);
//   MODE_GRAD : sum g, sum g (x - mean[ch]);
//   MODE_SUM  : sum g (second slot 0).
enum { MODE_STATS = 0, MODE_GRAD = 1, MODE_SUM = 2 };

template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads)
channel_sums_kernel(const T* __restrict__ a, const T* __restrict__ x, const T* __restrict__ mean,
                    int64_t n, int64_t C, int64_t hw, int chunks, double* __restrict__ partial) {
  __shared__ double sh[32];
  const int64_t ch = blockIdx.y;
  const int chunk = blockIdx.x;
  const int64_t i0 = chunk * n / chunks, i1 = (chunk + 1) * n / chunks;
  double shift = 0.0;
  if (MODE == MODE_STATS) shift = (double)a[ch * hw];
  if (MODE == MODE_GRAD) shift = (double)mean[ch];
  double s0 = 0.0, s1 = 0.0;
  for (int64_t img = i0; img < i1; ++img) {
    const int64_t base = (img * C + ch) * hw;
    for (int64_t j = threadIdx.x; j < hw; j += blockDim.x) {
      const double v = (double)a[base + j];
      if (MODE == MODE_STATS) {
        const double d = v - shift;
        s0 += d;
        s1 += d * d;
      } else if (MODE == MODE_GRAD) {
        s0 += v;
        s1 += v * ((double)x[base + j] - shift);
      } else {
        s0 += v;
      }
    }
  }
  s0 = block_sum(s0, sh);
  if (MODE != MODE_SUM) s1 = block_sum(s1, sh);
  if (threadIdx.x == 0) {
    partial[(ch * chunks + chunk) * 2] = s0;
    partial[(ch * chunks + chunk) * 2 + 1] = MODE == MODE_SUM ? 0.0 : s1;
  }
}

inline int chunks_for(int64_t n, int64_t C) {
  int64_t want = (4 * 148 + C - 1) / C;
  if (want > n) want = n;
  if (want < 1) want = 1;
  return (int)want;
}

template <typename T>
__global__ void bn_stats_final_kernel(const double* __restrict__ partial, int chunks,
                                      const T* __restrict__ x, int64_t C, int64_t hw, double m,
                                      T* __restrict__ mean, T* __restrict__ rstd,
                                      T* __restrict__ running_mean, T* __restrict__ running_var,
                                      double momentum, double eps) {
  const int64_t ch = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= C) return;
  double s0 = 0.0, s1 = 0.0;
  for (int k = 0; k < chunks; ++k) {
    s0 += partial[(ch * chunks + k) * 2];
    s1 += partial[(ch * chunks + k) * 2 + 1];
  }
  const double d = s0 / m;
  double var = s1 / m - d * d;
  if (var < 0.0) var = 0.0;
  const double mu = (double)x[ch * hw] + d;
  mean[ch] = (T)mu;
  rstd[ch] = (T)(1.0 / sqrt(var + eps));
  if (running_mean && running_var) {
    const double unbiased = var * (m / (m > 1.0 ? m - 1.0 : 1.0));
    running_mean[ch] = (T)((double)running_mean[ch] * (1.0 - momentum) + momentum * mu);
    running_var[ch] = (T)((double)running_var[ch] * (1.0 - momentum) + momentum * unbiased);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
bn_apply_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
                const T* __restrict__ mean, const T* __restrict__ rstd, T* __restrict__ y,
                int64_t total, int64_t C, int64_t hw) {
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ch = (idx / hw) % C;
    T v = (x[idx] - mean[ch]) * rstd[ch];
    if (w) v = v * w[ch];
    if (b) v = v + b[ch];
    y[idx] = v;
  }
}

// Per channel: gb = sum g, gw = rstd * sum g (x - mean), and the coefficients of
// gx = k0 * (g - k1 - xhat * k2): k0 = rstd w, k1 = gb / m, k2 = gw / m.
template <typename T>
__global__ void bn_grad_final_kernel(const double* __restrict__ partial, int chunks, int64_t C,
                                     double m, const T* __restrict__ w,
                                     const T* __restrict__ rstd, T* __restrict__ gw,
                                     T* __restrict__ gb, T* __restrict__ coef) {
  const int64_t ch = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= C) return;
  double sg = 0.0, sgx = 0.0;
  for (int k = 0; k < chunks; ++k) {
    sg += partial[(ch * chunks + k) * 2];
    sgx += partial[(ch * chunks + k) * 2 + 1];
  }
  const double r = (double)rstd[ch];
  const double dw = sgx * r;
  if (gb) gb[ch] = (T)sg;
  if (gw) gw[ch] = (T)dw;
  if (coef) {
    coef[3 * ch] = (T)(r * (w ? (double)w[ch] : 1.0));
    coef[3 * ch + 1] = (T)(sg / m);
    coef[3 * ch + 2] = (T)(dw / m);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
bn_grad_input_kernel(const T* __restrict__ g, const T* __restrict__ x,
                     const T* __restrict__ mean, const T* __restrict__ rstd,
                     const T* __restrict__ coef, T* __restrict__ gx, int64_t total, int64_t C,
                     int64_t hw) {
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ch = (idx / hw) % C;
    const T xhat = (x[idx] - mean[ch]) * rstd[ch];
    gx[idx] = coef[3 * ch] * (g[idx] - coef[3 * ch + 1] - xhat * coef[3 * ch + 2]);
  }
}

template <typename T>
__global__ void channel_total_kernel(const double* __restrict__ partial, int chunks, int64_t C,
                                     T* __restrict__ out) {
  const int64_t ch = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= C) return;
  double s = 0.0;
  for (int k = 0; k < chunks; ++k) s += partial[(ch * chunks + k) * 2];
  out[ch] = (T)s;
}

// ------------------------------------------------------------------ max pooling
template <typename T>
__device__ __forceinline__ bool is_nan(T v) { return v != v; }

template <typename T>
__global__ void __launch_bounds__(kThreads)
maxpool_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, uint8_t* __restrict__ arg,
                   tg_conv_shape s) {
  const int64_t total = s.n * s.c * s.oh * s.ow;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ox = idx % s.ow;
    int64_t rest = idx / s.ow;
    const int64_t oy = rest % s.oh;
    const int64_t plane = rest / s.oh;
    const T* xp = x + plane * s.h * s.w;
    T best = T(0);
    int bk = -1;
    for (int64_t i = 0; i < s.kh; ++i) {
      const int64_t iy = oy * s.sh - s.ph + i;
      for (int64_t j = 0; j < s.kw; ++j) {
        const int64_t ix = ox * s.sw - s.pw + j;
        const bool inside = iy >= 0 && iy < s.h && ix >= 0 && ix < s.w;
        const T v = inside ? xp[iy * s.w + ix] : T(-INFINITY);
        // First maximum in row-major order; a NaN wins and stays.
        if (bk < 0 || v > best || (is_nan(v) && !is_nan(best))) {
          best = v;
          bk = (int)(i * s.kw + j);
        }
      }
    }
    y[idx] = best;
    arg[idx] = (uint8_t)bk;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
maxpool_bwd_kernel(const T* __restrict__ g, const uint8_t* __restrict__ arg, T* __restrict__ gx,
                   tg_conv_shape s) {
  const int64_t total = s.n * s.c * s.h * s.w;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t xw = idx % s.w;
    int64_t rest = idx / s.w;
    const int64_t yh = rest % s.h;
    const int64_t plane = rest / s.h;
    // Windows (oy, ox) whose cell (i, j) = (yh + ph - oy*sh, xw + pw - ox*sw) is in range.
    int64_t oy0 = yh + s.ph - s.kh + 1;
    oy0 = oy0 <= 0 ? 0 : (oy0 + s.sh - 1) / s.sh;
    int64_t oy1 = (yh + s.ph) / s.sh;
    if (oy1 > s.oh - 1) oy1 = s.oh - 1;
    int64_t ox0 = xw + s.pw - s.kw + 1;
    ox0 = ox0 <= 0 ? 0 : (ox0 + s.sw - 1) / s.sw;
    int64_t ox1 = (xw + s.pw) / s.sw;
    if (ox1 > s.ow - 1) ox1 = s.ow - 1;
    T acc = T(0);
    for (int64_t oy = oy0; oy <= oy1; ++oy) {
      const int64_t i = yh + s.ph - oy * s.sh;
      for (int64_t ox = ox0; ox <= ox1; ++ox) {
        const int64_t j = xw + s.pw - ox * s.sw;
        const int64_t o = (plane * s.oh + oy) * s.ow + ox;
        if ((int64_t)arg[o] == i * s.kw + j) acc += g[o];
      }
    }
    gx[idx] = acc;
  }
}

// ------------------------------------------------------------------ scratch layout
struct ConvScratch {
  size_t wpad, ws, dcols, partial, total;
};

ConvScratch conv_bwd_layout(int dtype, const tg_conv_shape& s, bool need_gx) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const int64_t ld = cols_ld(s), K = s.c * s.kh * s.kw;
  ConvScratch L{};
  L.wpad = (ld != K) ? align256((size_t)(s.c_out * ld) * es) : 0;
  // Split-K partials of dW: up to one split per SM.
  L.ws = dtype == TG_F32 ? align256((size_t)148 * (size_t)(s.c_out * K) * sizeof(float)) : 0;
  L.dcols = need_gx ? align256((size_t)(s.n * s.oh * s.ow * ld) * es) : 0;
  L.partial = align256((size_t)s.c_out * chunks_for(s.n, s.c_out) * 2 * sizeof(double));
  L.total = L.wpad + L.ws + L.dcols + L.partial;
  return L;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int64_t tg_conv2d_cols_ld(const tg_conv_shape* s) { return s ? cols_ld(*s) : 0; }

size_t tg_conv2d_forward_scratch_bytes(int dtype, const tg_conv_shape* s) {
  if (!s) return 0;
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const int64_t ld = cols_ld(*s), K = s->c * s->kh * s->kw;
  return ld != K ? align256((size_t)(s->c_out * ld) * es) : 16;
}

int tg_conv2d_forward(int dtype, const tg_conv_shape* s, const void* x, const void* w,
                      const void* b, void* y, void* cols, void* scratch, void* stream) {
  int rc = check_conv(s, false);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  const int64_t ld = cols_ld(*s), K = s->c * s->kh * s->kw;
  const int64_t rows = s->n * s->oh * s->ow, ohw = s->oh * s->ow;
  if (rows == 0) return TG_OK;
  TG_CHECK_ARG(ld == K || scratch, "conv2d: scratch required");
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    im2col_kernel<T><<<grid_for(rows * ld, kThreads, 148 * 64), kThreads, 0, st>>>(
        (const T*)x, (T*)cols, *s, ld);
    int launched = 1;
    const T* wk = (const T*)w;
    if (ld != K) {
      pad_rows_kernel<T><<<grid_for(s->c_out * ld, kThreads), kThreads, 0, st>>>(
          (const T*)w, (T*)scratch, s->c_out, K, ld);
      wk = (const T*)scratch;
      ++launched;
    }
    int r = check_launch("conv2d(im2col)", launched);
    if (r) return r;
    GemmArgs<T> p{};
    p.m = rows; p.n = s->c_out; p.k = ld;
    p.a = (const T*)cols; p.lda = ld; p.stride_a = 0;
    p.b = wk; p.ldb = ld; p.stride_b = 0;
    p.c = (T*)y; p.ldc = ohw; p.stride_c = s->c_out * ohw;
    p.bias = (const T*)b;
    p.alpha = T(1); p.beta = T(0);
    p.trans_a = 0; p.trans_b = 1;
    p.batch = 1;
    p.c_hw = ohw;
    return gemm_run<T>(p, st);
  });
}

size_t tg_conv2d_backward_scratch_bytes(int dtype, const tg_conv_shape* s, int need_gx) {
  if (!s) return 0;
  const size_t t = conv_bwd_layout(dtype, *s, need_gx != 0).total;
  return t ? t : 16;
}

int tg_conv2d_backward(int dtype, const tg_conv_shape* s, const void* g, const void* cols,
                       const void* w, void* gx, void* gw, void* gb, void* scratch,
                       void* stream) {
  int rc = check_conv(s, false);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  const int64_t ld = cols_ld(*s), K = s->c * s->kh * s->kw;
  const int64_t rows = s->n * s->oh * s->ow, ohw = s->oh * s->ow;
  const ConvScratch L = conv_bwd_layout(dtype, *s, gx != nullptr);
  TG_CHECK_ARG(L.total == 0 || scratch, "conv2d backward: scratch required");
  uint8_t* base = (uint8_t*)scratch;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    if (rows == 0) {
      // Empty batch: zero gradients for the weights and the bias.
      if (gw) cudaMemsetAsync(gw, 0, (size_t)(s->c_out * K) * sizeof(T), st);
      if (gb) cudaMemsetAsync(gb, 0, (size_t)s->c_out * sizeof(T), st);
      return check_launch("conv2d backward(empty)", 0);
    }
    if (gw) {
      GemmArgs<T> p{};
      p.m = s->c_out; p.n = K; p.k = rows;
      p.a = (const T*)g; p.lda = ohw; p.stride_a = s->c_out * ohw; p.a_fold = ohw;
      p.b = (const T*)cols; p.ldb = ld; p.stride_b = 0;
      p.c = (T*)gw; p.ldc = K; p.stride_c = 0;
      p.alpha = T(1); p.beta = T(0);
      p.trans_a = 0; p.trans_b = 0;
      p.batch = 1;
      if (L.ws) {
        p.workspace = reinterpret_cast<float*>(base + L.wpad);
        p.workspace_bytes = L.ws;
      }
      int r = gemm_run<T>(p, st);
      if (r) return r;
    }
    if (gb) {
      const int chunks = chunks_for(s->n, s->c_out);
      double* partial = reinterpret_cast<double*>(base + L.wpad + L.ws + L.dcols);
      channel_sums_kernel<T, MODE_SUM><<<dim3(chunks, (unsigned)s->c_out), kThreads, 0, st>>>(
          (const T*)g, nullptr, nullptr, s->n, s->c_out, ohw, chunks, partial);
      channel_total_kernel<T><<<(unsigned)((s->c_out + 127) / 128), 128, 0, st>>>(
          partial, chunks, s->c_out, (T*)gb);
      int r = check_launch("conv2d backward(bias)", 2);
      if (r) return r;
    }
    if (gx) {
      const T* wk = (const T*)w;
      if (ld != K) {
        pad_rows_kernel<T><<<grid_for(s->c_out * ld, kThreads), kThreads, 0, st>>>(
            (const T*)w, (T*)base, s->c_out, K, ld);
        int r = check_launch("conv2d backward(pad)");
        if (r) return r;
        wk = (const T*)base;
      }
      T* dcols = reinterpret_cast<T*>(base + L.wpad + L.ws);
      GemmArgs<T> p{};
      p.m = ohw; p.n = ld; p.k = s->c_out;
      p.a = (const T*)g; p.lda = ohw; p.stride_a = s->c_out * ohw;
      p.b = wk; p.ldb = ld; p.stride_b = 0;
      p.c = dcols; p.ldc = ld; p.stride_c = ohw * ld;
      p.alpha = T(1); p.beta = T(0);
      p.trans_a = 1; p.trans_b = 0;
      p.batch = s->n;
      int r = gemm_run<T>(p, st);
      if (r) return r;
      col2im_kernel<T><<<grid_for(s->n * s->c * s->h * s->w, kThreads, 148 * 64), kThreads, 0,
                         st>>>(dcols, (T*)gx, *s, ld);
      r = check_launch("conv2d backward(col2im)");
      if (r) return r;
    }
    return (int)TG_OK;
  });
}

size_t tg_batch_norm_scratch_bytes(int dtype, int64_t n, int64_t c, int64_t hw) {
  (void)hw;
  const size_t es = dtype == TG_F64 ? 8 : 4;
  return align256((size_t)c * chunks_for(n, c) * 2 * sizeof(double)) + align256((size_t)c * 3 * es);
}

int tg_batch_norm_forward(int dtype, int64_t n, int64_t c, int64_t hw, const void* x,
                          const void* w, const void* b, void* y, void* mean, void* rstd,
                          void* running_mean, void* running_var, double momentum, double eps,
                          void* scratch, void* stream) {
  TG_CHECK_ARG(n > 0 && c > 0 && hw > 0 && c <= 65535, "batch_norm: bad shape");
  TG_CHECK_ARG(scratch && mean && rstd, "batch_norm: scratch/mean/rstd required");
  cudaStream_t st = as_stream(stream);
  const int chunks = chunks_for(n, c);
  double* partial = reinterpret_cast<double*>(scratch);
  const int64_t total = n * c * hw;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    channel_sums_kernel<T, MODE_STATS><<<dim3(chunks, (unsigned)c), kThreads, 0, st>>>(
        (const T*)x, nullptr, nullptr, n, c, hw, chunks, partial);
    bn_stats_final_kernel<T><<<(unsigned)((c + 127) / 128), 128, 0, st>>>(
        partial, chunks, (const T*)x, c, hw, (double)(n * hw), (T*)mean, (T*)rstd,
        (T*)running_mean, (T*)running_var, momentum, eps);
    bn_apply_kernel<T><<<grid_for(total, kThreads, 148 * 64), kThreads, 0, st>>>(
        (const T*)x, (const T*)w, (const T*)b, (const T*)mean, (const T*)rstd, (T*)y, total, c,
        hw);
    return check_launch("batch_norm", 3);
  });
}

int tg_batch_norm_backward(int dtype, int64_t n, int64_t c, int64_t hw, const void* g,
                           const void* x, const void* w, const void* mean, const void* rstd,
                           void* gx, void* gw, void* gb, void* scratch, void* stream) {
  TG_CHECK_ARG(n > 0 && c > 0 && hw > 0 && c <= 65535, "batch_norm backward: bad shape");
  TG_CHECK_ARG(scratch, "batch_norm backward: scratch required");
  cudaStream_t st = as_stream(stream);
  const int chunks = chunks_for(n, c);
  double* partial = reinterpret_cast<double*>(scratch);
  const size_t coef_off = align256((size_t)c * chunks * 2 * sizeof(double));
  const int64_t total = n * c * hw;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* coef = reinterpret_cast<T*>((uint8_t*)scratch + coef_off);
    channel_sums_kernel<T, MODE_GRAD><<<dim3(chunks, (unsigned)c), kThreads, 0, st>>>(
        (const T*)g, (const T*)x, (const T*)mean, n, c, hw, chunks, partial);
    bn_grad_final_kernel<T><<<(unsigned)((c + 127) / 128), 128, 0, st>>>(
        partial, chunks, c, (double)(n * hw), (const T*)w, (const T*)rstd, (T*)gw, (T*)gb,
        gx ? coef : nullptr);
    int launched = 2;
    if (gx) {
      bn_grad_input_kernel<T><<<grid_for(total, kThreads, 148 * 64), kThreads, 0, st>>>(
          (const T*)g, (const T*)x, (const T*)mean, (const T*)rstd, coef, (T*)gx, total, c, hw);
      ++launched;
    }
    return check_launch("batch_norm backward", launched);
  });
}

int tg_max_pool2d_forward(int dtype, const tg_conv_shape* s, const void* x, void* y,
                          uint8_t* argmax, void* stream) {
  int rc = check_conv(s, true);
  if (rc) return rc;
  TG_CHECK_ARG(s->kh * s->kw <= 256, "max_pool2d: at most 256 cells per window");
  TG_CHECK_ARG(2 * s->ph <= s->kh && 2 * s->pw <= s->kw,
               "max_pool2d: padding must be at most half the kernel size");
  const int64_t total = s->n * s->c * s->oh * s->ow;
  if (total == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    maxpool_fwd_kernel<T><<<grid_for(total, kThreads, 148 * 64), kThreads, 0, st>>>(
        (const T*)x, (T*)y, argmax, *s);
    return check_launch("max_pool2d");
  });
}

int tg_max_pool2d_backward(int dtype, const tg_conv_shape* s, const void* g,
                           const uint8_t* argmax, void* gx, void* stream) {
  int rc = check_conv(s, true);
  if (rc) return rc;
  const int64_t total = s->n * s->c * s->h * s->w;
  if (total == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    maxpool_bwd_kernel<T><<<grid_for(total, kThreads, 148 * 64), kThreads, 0, st>>>(
        (const T*)g, argmax, (T*)gx, *s);
    return check_launch("max_pool2d backward");
  });
}

}  // extern "C"
