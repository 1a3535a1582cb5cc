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
#include <algorithm>
#include <initializer_list>
#include <type_traits>

#include "common.cuh"
#include "gemm.cuh"

namespace tg {
namespace {

constexpr int kThreads = 256;

// V consecutive elements moved as one access (16 bytes for float x 4).
template <typename T, int V>
struct alignas(sizeof(T) * V) Vec {
  T v[V];
};

// Patch rows (c*kh*kw rounded up to 4: the filter matrix's rows then suit the TMA) and the
// patch matrix's row stride (n*oh*ow rounded up to 4).
inline int64_t patch_rows(const tg_conv_shape& s) { return (s.c * s.kh * s.kw + 3) / 4 * 4; }
inline int64_t patch_ld(const tg_conv_shape& s) { return (s.n * s.oh * s.ow + 3) / 4 * 4; }

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
  TG_CHECK_ARG(s->h * s->w < INT32_MAX && s->oh * s->ow < INT32_MAX && s->kh * s->kw < 65536,
               "conv2d: planes of at most 2^31 pixels, windows of at most 65535 cells");
  return TG_OK;
}

// ------------------------------------------------------------------ im2col / col2im
// The patch matrix is stored patch-major: cols[kk][m], kk = (ch, i, j) < kp (rows kk >= c*kh*kw
// zero), m = image * oh*ow + pixel < n*oh*ow, row stride ldm (a multiple of 4).
//
// Index arithmetic by runtime sizes (divisions) costs more than the bytes each element moves,
// so every kernel below fixes a thread's position inside a plane (decoded once) and walks the
// planes (images, channels) with constant strides: the loop body is a few loads and a store.
// Grids: x over in-plane positions (one per thread), y and z over plane ranges. In-plane
// indices are 32-bit (the host checks planes of fewer than 2^31 pixels).

// Image range [i0, i1) of block z out of gridDim.z.
__device__ __forceinline__ void image_range(int64_t n, int64_t& i0, int64_t& i1) {
  i0 = (int64_t)blockIdx.z * n / gridDim.z;
  i1 = ((int64_t)blockIdx.z + 1) * n / gridDim.z;
}

// Grid (pixel blocks, patch rows, image ranges). Consecutive threads take consecutive output
// pixels: stores are whole lines and (for stride 1) loads are unit-stride runs of x.
template <typename T>
__global__ void __launch_bounds__(kThreads)
im2col_kernel(const T* __restrict__ x, T* __restrict__ cols, tg_conv_shape s, int64_t K,
              int64_t kp, int64_t ldm) {
  const int ohw = (int)(s.oh * s.ow);
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= ohw) return;
  const int ow = (int)s.ow, h = (int)s.h, w = (int)s.w;
  const int oy = p / ow, ox = p - oy * ow;
  const int khw = (int)(s.kh * s.kw), kw = (int)s.kw;
  const int64_t plane = (int64_t)h * w, img_stride = s.c * plane;
  int64_t i0, i1;
  image_range(s.n, i0, i1);
  for (int64_t kk = blockIdx.y; kk < kp; kk += gridDim.y) {
    T* out = cols + kk * ldm + p;
    bool live = kk < K;
    int64_t src = 0;
    if (live) {
      const int64_t ch = kk / khw;
      const int r = (int)(kk - ch * khw), i = r / kw, j = r - i * kw;
      const int iy = oy * (int)s.sh - (int)s.ph + i, ix = ox * (int)s.sw - (int)s.pw + j;
      live = iy >= 0 && iy < h && ix >= 0 && ix < w;
      src = ch * plane + (int64_t)iy * w + ix;
    }
    if (live) {
#pragma unroll 4
      for (int64_t img = i0; img < i1; ++img) out[img * ohw] = x[img * img_stride + src];
    } else {
#pragma unroll 4
      for (int64_t img = i0; img < i1; ++img) out[img * ohw] = T(0);
    }
  }
}

// dx[img][ch][y][x] = sum over kernel offsets (i, j) whose window covers (y, x) of
// dcols[(ch, i, j)][(img, oy, ox)], in ascending (i, j) (the reference's col2im order).
// Grid (pixel blocks, channels, image ranges). The covering windows of a pixel are the same
// for every image and channel: found once, as an output row per kernel row and an output
// column per kernel column (-1: no window), for windows of up to MAXW x MAXW.
template <typename T, int MAXW>
__global__ void __launch_bounds__(kThreads)
col2im_kernel(const T* __restrict__ dcols, T* __restrict__ gx, tg_conv_shape s, int64_t ldm) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int hw = (int)(s.h * s.w);
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= hw) return;
  const int w = (int)s.w, yh = q / w, xw = q - yh * w;
  const int kh = (int)s.kh, kw = (int)s.kw, sh = (int)s.sh, sw = (int)s.sw;
  const int oh = (int)s.oh, ow = (int)s.ow, ohw = oh * ow;
  int oyv[MAXW], oxv[MAXW];
#pragma unroll
  for (int i = 0; i < MAXW; ++i) {
    const int ty = yh + (int)s.ph - i;
    oyv[i] = (i < kh && ty >= 0 && ty % sh == 0 && ty / sh < oh) ? ty / sh : -1;
  }
#pragma unroll
  for (int j = 0; j < MAXW; ++j) {
    const int tx = xw + (int)s.pw - j;
    oxv[j] = (j < kw && tx >= 0 && tx % sw == 0 && tx / sw < ow) ? tx / sw : -1;
  }
  int64_t i0, i1;
  image_range(s.n, i0, i1);
  for (int64_t ch = blockIdx.y; ch < s.c; ch += gridDim.y) {
    const T* base = dcols + ch * kh * kw * ldm;
    for (int64_t img = i0; img < i1; ++img) {
      const T* bi = base + img * ohw;
      T acc = T(0);
#pragma unroll
      for (int i = 0; i < MAXW; ++i) {
        if (oyv[i] < 0) continue;
#pragma unroll
        for (int j = 0; j < MAXW; ++j) {
          if (oxv[j] < 0) continue;
          acc += bi[(int64_t)(i * kw + j) * ldm + oyv[i] * ow + oxv[j]];
        }
      }
      gx[(img * s.c + ch) * hw + q] = acc;
    }
  }
}

// Four neighbouring output pixels of one row per thread (fp32, rows of a multiple of 4
// pixels, 16-byte aligned patch rows): one 16-byte store per patch row and image, the same
// values as im2col_kernel. (Gathering four pixels per thread in col2im measured slower on
// B200, 176 against 158 us at the CNN's second layer, so col2im keeps one pixel per thread.)
__global__ void __launch_bounds__(kThreads)
im2col4_kernel(const float* __restrict__ x, float* __restrict__ cols, tg_conv_shape s,
               int64_t K, int64_t kp, int64_t ldm) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int ohw = (int)(s.oh * s.ow);
  const int p = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (p >= ohw) return;
  const int ow = (int)s.ow, h = (int)s.h, w = (int)s.w;
  const int oy = p / ow, ox = p - oy * ow;
  const int khw = (int)(s.kh * s.kw), kw = (int)s.kw, sw = (int)s.sw;
  const int64_t plane = (int64_t)h * w, img_stride = s.c * plane;
  int64_t i0, i1;
  image_range(s.n, i0, i1);
  for (int64_t kk = blockIdx.y; kk < kp; kk += gridDim.y) {
    float4* out = reinterpret_cast<float4*>(cols + kk * ldm + p);
    int64_t src[4];
    bool live[4];
    if (kk < K) {
      const int64_t ch = kk / khw;
      const int r = (int)(kk - ch * khw), i = r / kw, j = r - i * kw;
      const int iy = oy * (int)s.sh - (int)s.ph + i;
      const int ix0 = ox * sw - (int)s.pw + j;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ix = ix0 + e * sw;
        live[e] = iy >= 0 && iy < h && ix >= 0 && ix < w;
        src[e] = live[e] ? ch * plane + (int64_t)iy * w + ix : 0;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        live[e] = false;
        src[e] = 0;
      }
    }
#pragma unroll 2
    for (int64_t img = i0; img < i1; ++img) {
      const float* xi = x + img * img_stride;
      float4 v;
      v.x = live[0] ? __ldg(xi + src[0]) : 0.f;
      v.y = live[1] ? __ldg(xi + src[1]) : 0.f;
      v.z = live[2] ? __ldg(xi + src[2]) : 0.f;
      v.w = live[3] ? __ldg(xi + src[3]) : 0.f;
      out[img * (ohw / 4)] = v;
    }
  }
}

// Whether im2col can take four output pixels per thread.
template <typename T>
bool conv_vec4(const tg_conv_shape& s, std::initializer_list<const void*> ptrs) {
  if (!std::is_same<T, float>::value || s.ow % 4 || s.w % 4 || s.ow * s.oh > INT32_MAX / 4)
    return false;
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return false;
  return true;
}

// The same for windows larger than 16 x 16: the covering windows found per image.
template <typename T>
__global__ void __launch_bounds__(kThreads)
col2im_large_kernel(const T* __restrict__ dcols, T* __restrict__ gx, tg_conv_shape s,
                    int64_t ldm) {
  const int hw = (int)(s.h * s.w);
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= hw) return;
  const int w = (int)s.w, yh = q / w, xw = q - yh * w;
  const int kh = (int)s.kh, kw = (int)s.kw, sh = (int)s.sh, sw = (int)s.sw;
  const int oh = (int)s.oh, ow = (int)s.ow, ohw = oh * ow;
  int64_t i0, i1;
  image_range(s.n, i0, i1);
  for (int64_t ch = blockIdx.y; ch < s.c; ch += gridDim.y) {
    const T* base = dcols + ch * kh * kw * ldm;
    for (int64_t img = i0; img < i1; ++img) {
      T acc = T(0);
      for (int i = 0; i < kh; ++i) {
        const int ty = yh + (int)s.ph - i;
        if (ty < 0 || ty % sh || ty / sh >= oh) continue;
        for (int j = 0; j < kw; ++j) {
          const int tx = xw + (int)s.pw - j;
          if (tx < 0 || tx % sw || tx / sw >= ow) continue;
          acc += base[(int64_t)(i * kw + j) * ldm + img * ohw + (ty / sh) * ow + tx / sw];
        }
      }
      gx[(img * s.c + ch) * hw + q] = acc;
    }
  }
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline unsigned clamp_grid(int64_t v, int64_t cap) { return (unsigned)(v < 1 ? 1 : v > cap ? cap : v); }

// About 16 resident-sized blocks per SM in total: enough to cover the memory latency, while
// each block loops over many planes (a block per plane would be too little work to pay for
// its own launch).
constexpr int64_t kGridTarget = 148 * 16;

// x over in-plane positions (one per thread), y (and z) over plane ranges: about
// kGridTarget blocks in all, each plane range walked by one block.
inline dim3 position_grid(int64_t positions, int64_t ranges_y, int64_t ranges_z = 1) {
  const int64_t x = ceil_div(positions, kThreads);
  const int64_t y = std::min<int64_t>(ranges_y, 65535);
  const int64_t want_z = ceil_div(kGridTarget, x * y);
  const int64_t z = std::max<int64_t>(1, std::min<int64_t>({want_z, ranges_z, 65535}));
  if (ranges_z > 1) return dim3((unsigned)x, (unsigned)y, (unsigned)z);
  const int64_t yy = std::max<int64_t>(1, std::min<int64_t>({ceil_div(kGridTarget, x), ranges_y,
                                                            65535}));
  return dim3((unsigned)x, (unsigned)yy, 1);
}

// x over groups of a plane (kThreads per block, at most 16 blocks), y over planes.
inline dim3 plane_grid(int64_t groups, int64_t planes) {
  const unsigned x = clamp_grid(ceil_div(groups, kThreads), 16);
  return dim3(x, clamp_grid(planes < ceil_div(kGridTarget, x) ? planes : ceil_div(kGridTarget, x),
                            65535));
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

template <typename T, int MODE, int V>
__global__ void __launch_bounds__(kThreads)
channel_sums_kernel(const T* __restrict__ a, const T* __restrict__ x, const T* __restrict__ mean,
                    int64_t n, int64_t C, int64_t hw, int chunks, double* __restrict__ partial) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  __shared__ double sh[32];
  const int64_t ch = blockIdx.y;
  const int chunk = blockIdx.x;
  const int64_t i0 = chunk * n / chunks, i1 = (chunk + 1) * n / chunks;
  double shift = 0.0;
  if (MODE == MODE_STATS) shift = (double)a[ch * hw];
  if (MODE == MODE_GRAD) shift = (double)mean[ch];
  double s0 = 0.0, s1 = 0.0;
  const int64_t nv = hw / V;
  for (int64_t img = i0; img < i1; ++img) {
    const int64_t base = (img * C + ch) * hw;
    const Vec<T, V>* av = reinterpret_cast<const Vec<T, V>*>(a + base);
    const Vec<T, V>* xv = reinterpret_cast<const Vec<T, V>*>(MODE == MODE_GRAD ? x + base : a + base);
    for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
      const Vec<T, V> va = av[j];
      Vec<T, V> vx;
      if (MODE == MODE_GRAD) vx = xv[j];
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const double v = (double)va.v[e];
        if (MODE == MODE_STATS) {
          const double d = v - shift;
          s0 += d;
          s1 += d * d;
        } else if (MODE == MODE_GRAD) {
          s0 += v;
          s1 += v * ((double)vx.v[e] - shift);
        } else {
          s0 += v;
        }
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
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
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

// Grid: x over V-element groups of a plane (image, channel), y over planes; the channel's
// statistics are loaded once per plane.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads)
bn_apply_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
                const T* __restrict__ mean, const T* __restrict__ rstd, T* __restrict__ y,
                int64_t planes, int64_t C, int64_t hw) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int64_t nv = hw / V;
  for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
    const int64_t ch = plane % C;
    const T mu = mean[ch], r = rstd[ch];
    const Vec<T, V>* xv = reinterpret_cast<const Vec<T, V>*>(x + plane * hw);
    Vec<T, V>* yv = reinterpret_cast<Vec<T, V>*>(y + plane * hw);
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < nv;
         j += (int64_t)gridDim.x * blockDim.x) {
      Vec<T, V> v = xv[j];
#pragma unroll
      for (int e = 0; e < V; ++e) {
        T t = (v.v[e] - mu) * r;
        if (w) t = t * w[ch];
        if (b) t = t + b[ch];
        v.v[e] = t;
      }
      yv[j] = v;
    }
  }
}

// Per channel: gb = sum g, gw = rstd * sum g (x - mean), and the coefficients of
// gx = k0 * (g - k1 - xhat * k2): k0 = rstd w, k1 = gb / m, k2 = gw / m.
template <typename T>
__global__ void bn_grad_final_kernel(const double* __restrict__ partial, int chunks, int64_t C,
                                     double m, const T* __restrict__ w,
                                     const T* __restrict__ rstd, T* __restrict__ gw,
                                     T* __restrict__ gb, T* __restrict__ coef) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
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

template <typename T, int V>
__global__ void __launch_bounds__(kThreads)
bn_grad_input_kernel(const T* __restrict__ g, const T* __restrict__ x,
                     const T* __restrict__ mean, const T* __restrict__ rstd,
                     const T* __restrict__ coef, T* __restrict__ gx, int64_t planes, int64_t C,
                     int64_t hw) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int64_t nv = hw / V;
  for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
    const int64_t ch = plane % C;
    const T mu = mean[ch], r = rstd[ch];
    const T k0 = coef[3 * ch], k1 = coef[3 * ch + 1], k2 = coef[3 * ch + 2];
    const Vec<T, V>* gv = reinterpret_cast<const Vec<T, V>*>(g + plane * hw);
    const Vec<T, V>* xv = reinterpret_cast<const Vec<T, V>*>(x + plane * hw);
    Vec<T, V>* ov = reinterpret_cast<Vec<T, V>*>(gx + plane * hw);
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < nv;
         j += (int64_t)gridDim.x * blockDim.x) {
      const Vec<T, V> a = gv[j], xx = xv[j];
      Vec<T, V> o;
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const T xhat = (xx.v[e] - mu) * r;
        o.v[e] = k0 * (a.v[e] - k1 - xhat * k2);
      }
      ov[j] = o;
    }
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

// Pooling grids: x over in-plane positions (one per thread, decoded once), y over plane
// (image, channel) ranges.
__device__ __forceinline__ void plane_range(int64_t planes, int64_t& p0, int64_t& p1) {
  p0 = (int64_t)blockIdx.y * planes / gridDim.y;
  p1 = ((int64_t)blockIdx.y + 1) * planes / gridDim.y;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
maxpool_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, uint8_t* __restrict__ arg,
                   tg_conv_shape s) {
  const int ohw = (int)(s.oh * s.ow);
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= ohw) return;
  const int h = (int)s.h, w = (int)s.w, ow = (int)s.ow, hw = h * w;
  const int kh = (int)s.kh, kw = (int)s.kw;
  const int oy = o / ow, ox = o - oy * ow;
  const int iy0 = oy * (int)s.sh - (int)s.ph, ix0 = ox * (int)s.sw - (int)s.pw;
  int64_t p0, p1;
  plane_range(s.n * s.c, p0, p1);
  for (int64_t plane = p0; plane < p1; ++plane) {
    const T* xp = x + plane * hw;
    T best = T(0);
    int bk = -1;
    for (int i = 0; i < kh; ++i) {
      const int iy = iy0 + i;
      for (int j = 0; j < kw; ++j) {
        const int ix = ix0 + j;
        const bool inside = iy >= 0 && iy < h && ix >= 0 && ix < w;
        const T v = inside ? xp[iy * w + ix] : T(-INFINITY);
        // First maximum in row-major order; a NaN wins and stays.
        if (bk < 0 || v > best || (is_nan(v) && !is_nan(best))) {
          best = v;
          bk = i * kw + j;
        }
      }
    }
    y[plane * ohw + o] = best;
    arg[plane * ohw + o] = (uint8_t)bk;
  }
}

// gx[cell] = sum of g over the windows whose winner is that cell. With windows that do not
// overlap (stride >= kernel) a cell lies in at most one window: one load of its winner byte.
template <typename T, bool DISJOINT>
__global__ void __launch_bounds__(kThreads)
maxpool_bwd_kernel(const T* __restrict__ g, const uint8_t* __restrict__ arg, T* __restrict__ gx,
                   tg_conv_shape s) {
  const int h = (int)s.h, w = (int)s.w, hw = h * w;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= hw) return;
  const int oh = (int)s.oh, ow = (int)s.ow, ohw = oh * ow;
  const int kh = (int)s.kh, kw = (int)s.kw, sh = (int)s.sh, sw = (int)s.sw;
  const int ph = (int)s.ph, pw = (int)s.pw;
  const int yh = q / w, xw = q - yh * w;
  int64_t p0, p1;
  plane_range(s.n * s.c, p0, p1);
  if (DISJOINT) {
    const int oy = (yh + ph) / sh, ox = (xw + pw) / sw;
    const int i = yh + ph - oy * sh, j = xw + pw - ox * sw;
    const bool covered = oy < oh && ox < ow && i < kh && j < kw;
    const int o = covered ? oy * ow + ox : 0, cell = i * kw + j;
    for (int64_t plane = p0; plane < p1; ++plane) {
      T v = T(0);
      if (covered && (int)arg[plane * ohw + o] == cell) v = g[plane * ohw + o];
      gx[plane * hw + q] = v;
    }
  } else {
    // Windows (oy, ox) whose cell (i, j) = (yh + ph - oy*sh, xw + pw - ox*sw) is in range.
    int oy0 = yh + ph - kh + 1;
    oy0 = oy0 <= 0 ? 0 : (oy0 + sh - 1) / sh;
    const int oy1 = min((yh + ph) / sh, oh - 1);
    int ox0 = xw + pw - kw + 1;
    ox0 = ox0 <= 0 ? 0 : (ox0 + sw - 1) / sw;
    const int ox1 = min((xw + pw) / sw, ow - 1);
    for (int64_t plane = p0; plane < p1; ++plane) {
      const T* gp = g + plane * ohw;
      const uint8_t* ap = arg + plane * ohw;
      T acc = T(0);
      for (int oy = oy0; oy <= oy1; ++oy) {
        const int i = yh + ph - oy * sh;
        for (int ox = ox0; ox <= ox1; ++ox) {
          const int j = xw + pw - ox * sw;
          const int o = oy * ow + ox;
          if ((int)ap[o] == i * kw + j) acc += gp[o];
        }
      }
      gx[plane * hw + q] = acc;
    }
  }
}

// The adjoint of maxpool_bwd_kernel (used by differentiable pooling VJPs): each output takes
// the value of u at its window's recorded winner; a winner in the padding reads 0.
template <typename T>
__global__ void __launch_bounds__(kThreads)
maxpool_gather_kernel(const T* __restrict__ u, const uint8_t* __restrict__ arg,
                      T* __restrict__ out, tg_conv_shape s) {
  const int ohw = (int)(s.oh * s.ow);
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= ohw) return;
  const int h = (int)s.h, w = (int)s.w, ow = (int)s.ow, hw = h * w, kw = (int)s.kw;
  const int oy = o / ow, ox = o - oy * ow;
  const int iy0 = oy * (int)s.sh - (int)s.ph, ix0 = ox * (int)s.sw - (int)s.pw;
  int64_t p0, p1;
  plane_range(s.n * s.c, p0, p1);
  for (int64_t plane = p0; plane < p1; ++plane) {
    const int cell = (int)arg[plane * ohw + o];
    const int iy = iy0 + cell / kw, ix = ix0 + cell % kw;
    const bool inside = iy >= 0 && iy < h && ix >= 0 && ix < w;
    out[plane * ohw + o] = inside ? u[plane * hw + iy * w + ix] : T(0);
  }
}

// 2 x 2 windows, stride 2, no padding, rows of a multiple of 4 floats (the CNN's pooling):
// each thread takes two neighbouring outputs of one output row, from one 16-byte load per
// input row, and writes both maxima (8 bytes) and both winner bytes (2 bytes). Same rule as
// maxpool_fwd_kernel: first maximum in row-major order, a NaN wins and stays.
__device__ __forceinline__ void pool4_first_max(float v0, float v1, float v2, float v3,
                                                float& best, int& bk) {
  best = v0;
  bk = 0;
  const float v[3] = {v1, v2, v3};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    if (v[k] > best || (v[k] != v[k] && best == best)) {
      best = v[k];
      bk = k + 1;
    }
  }
}

__global__ void __launch_bounds__(kThreads)
maxpool2x2_fwd_kernel(const float* __restrict__ x, float* __restrict__ y,
                      uint8_t* __restrict__ arg, int64_t planes, int h, int w) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int oh = h / 2, ow = w / 2, quads = w / 4;
  const int64_t per_plane = (int64_t)oh * quads, total = planes * per_plane;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t plane = t / per_plane;
    const int rem = (int)(t - plane * per_plane);
    const int oy = rem / quads, qx = rem - oy * quads;
    const float* r0 = x + plane * h * w + (int64_t)(2 * oy) * w + 4 * qx;
    const float4 a = __ldg(reinterpret_cast<const float4*>(r0));
    const float4 b = __ldg(reinterpret_cast<const float4*>(r0 + w));
    float m0, m1;
    int k0, k1;
    pool4_first_max(a.x, a.y, b.x, b.y, m0, k0);
    pool4_first_max(a.z, a.w, b.z, b.w, m1, k1);
    const int64_t o = plane * oh * ow + (int64_t)oy * ow + 2 * qx;
    *reinterpret_cast<float2*>(y + o) = make_float2(m0, m1);
    *reinterpret_cast<uint16_t*>(arg + o) = (uint16_t)(k0 | (k1 << 8));
  }
}

// The VJP of the 2 x 2 case: each thread reads two outputs' gradients and winner bytes and
// writes their two windows (two 16-byte rows of gx); cells that did not win get 0.
__global__ void __launch_bounds__(kThreads)
maxpool2x2_bwd_kernel(const float* __restrict__ g, const uint8_t* __restrict__ arg,
                      float* __restrict__ gx, int64_t planes, int h, int w) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int oh = h / 2, ow = w / 2, quads = w / 4;
  const int64_t per_plane = (int64_t)oh * quads, total = planes * per_plane;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t plane = t / per_plane;
    const int rem = (int)(t - plane * per_plane);
    const int oy = rem / quads, qx = rem - oy * quads;
    const int64_t o = plane * oh * ow + (int64_t)oy * ow + 2 * qx;
    const float2 gv = __ldg(reinterpret_cast<const float2*>(g + o));
    const uint16_t kk = __ldg(reinterpret_cast<const unsigned short*>(arg + o));
    const int k0 = kk & 0xff, k1 = kk >> 8;
    float* r0 = gx + plane * h * w + (int64_t)(2 * oy) * w + 4 * qx;
    *reinterpret_cast<float4*>(r0) = make_float4(k0 == 0 ? gv.x : 0.f, k0 == 1 ? gv.x : 0.f,
                                                 k1 == 0 ? gv.y : 0.f, k1 == 1 ? gv.y : 0.f);
    *reinterpret_cast<float4*>(r0 + w) = make_float4(k0 == 2 ? gv.x : 0.f,
                                                     k0 == 3 ? gv.x : 0.f,
                                                     k1 == 2 ? gv.y : 0.f,
                                                     k1 == 3 ? gv.y : 0.f);
  }
}

// Whether a pooling call is the 2 x 2 / stride 2 case the kernels above take.
template <typename T>
bool pool2x2(const tg_conv_shape& s, std::initializer_list<const void*> ptrs) {
  if (!std::is_same<T, float>::value) return false;
  if (s.kh != 2 || s.kw != 2 || s.sh != 2 || s.sw != 2 || s.ph || s.pw) return false;
  if (s.h % 2 || s.w % 4 || s.h * s.w > INT32_MAX) return false;
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return false;
  return true;
}

inline int pool_blocks(int64_t work) {
  const int64_t cap = (int64_t)kGridTarget;
  const int64_t b = ceil_div(work, kThreads);
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

// Per-plane kernels take 16-byte groups when T is float, planes hold a multiple of 4 elements
// and every buffer is 16-byte aligned.
template <typename T>
bool plane_vec4(int64_t hw, std::initializer_list<const void*> ptrs) {
  if (!std::is_same<T, float>::value || hw % 4) return false;
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return false;
  return true;
}

template <typename T, int MODE>
void launch_channel_sums(const T* a, const T* x, const T* mean, int64_t n, int64_t C,
                         int64_t hw, int chunks, double* partial, cudaStream_t st) {
  const dim3 grid(chunks, (unsigned)C);
  if (plane_vec4<T>(hw, {a, x}))
    launch_pdl(channel_sums_kernel<T, MODE, 4>, dim3(grid), dim3(kThreads), 0, st,
               a, x, mean, n, C, hw, chunks, partial);
  else
    launch_pdl(channel_sums_kernel<T, MODE, 1>, dim3(grid), dim3(kThreads), 0, st,
               a, x, mean, n, C, hw, chunks, partial);
}

// ------------------------------------------------------------------ scratch layout
struct ConvScratch {
  size_t wpad, ws, dcols, partial, total;
};

ConvScratch conv_bwd_layout(int dtype, const tg_conv_shape& s, bool need_gx) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const int64_t kp = patch_rows(s), K = s.c * s.kh * s.kw;
  ConvScratch L{};
  L.wpad = (kp != K) ? align256((size_t)(s.c_out * kp) * es) : 0;
  // Split-K partials of dW: up to one split per SM.
  L.ws = dtype == TG_F32 ? align256((size_t)148 * (size_t)(s.c_out * kp) * sizeof(float)) : 0;
  L.dcols = need_gx ? align256((size_t)(kp * patch_ld(s)) * es) : 0;
  L.partial = align256((size_t)s.c_out * chunks_for(s.n, s.c_out) * 2 * sizeof(double));
  L.total = L.wpad + L.ws + L.dcols + L.partial;
  return L;
}

}  // namespace
}  // namespace tg

using namespace tg;

namespace tg {
namespace {

// The patch matrix of x (layout of tg_conv2d_cols_shape): rows of whole 16-byte groups of
// pixels when the shape allows, else one pixel per thread.
template <typename T>
void launch_im2col(const tg_conv_shape& s, const void* x, void* cols, cudaStream_t st) {
  const int64_t kp = patch_rows(s), ldm = patch_ld(s), K = s.c * s.kh * s.kw;
  const int64_t ohw = s.oh * s.ow;
  if (conv_vec4<T>(s, {cols}) && ldm % 4 == 0) {
    const dim3 grid = position_grid(ohw / 4, kp, s.n);
    launch_pdl(im2col4_kernel, dim3(grid), dim3(kThreads), 0, st,
               (const float*)x, (float*)cols, s, K, kp, ldm);
  } else {
    const dim3 grid = position_grid(ohw, kp, s.n);
    im2col_kernel<T><<<grid, kThreads, 0, st>>>((const T*)x, (T*)cols, s, K, kp, ldm);
  }
}

}  // namespace
}  // namespace tg

extern "C" {

int tg_conv2d_cols_shape(const tg_conv_shape* s, int64_t* rows, int64_t* ld) {
  TG_CHECK_ARG(s && rows && ld, "conv2d: null argument");
  *rows = patch_rows(*s);
  *ld = patch_ld(*s);
  return TG_OK;
}

size_t tg_conv2d_forward_scratch_bytes(int dtype, const tg_conv_shape* s) {
  if (!s) return 0;
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const int64_t kp = patch_rows(*s), K = s->c * s->kh * s->kw;
  return kp != K ? align256((size_t)(s->c_out * kp) * es) : 16;
}

int tg_conv2d_im2col(int dtype, const tg_conv_shape* s, const void* x, void* cols,
                     void* stream) {
  int rc = check_conv(s, false);
  if (rc) return rc;
  if (s->n * s->oh * s->ow == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    launch_im2col<T>(*s, x, cols, st);
    return check_launch("conv2d(im2col)");
  });
}

int tg_conv2d_forward(int dtype, const tg_conv_shape* s, const void* x, const void* w,
                      const void* b, void* y, void* cols, void* scratch, void* stream) {
  int rc = check_conv(s, false);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  const int64_t kp = patch_rows(*s), ldm = patch_ld(*s), K = s->c * s->kh * s->kw;
  const int64_t rows = s->n * s->oh * s->ow, ohw = s->oh * s->ow;
  if (rows == 0) return TG_OK;
  TG_CHECK_ARG(kp == K || scratch, "conv2d: scratch required");
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    launch_im2col<T>(*s, x, cols, st);
    int launched = 1;
    const T* wk = (const T*)w;
    if (kp != K) {
      pad_rows_kernel<T><<<grid_for(s->c_out * kp, kThreads), kThreads, 0, st>>>(
          (const T*)w, (T*)scratch, s->c_out, K, kp);
      wk = (const T*)scratch;
      ++launched;
    }
    int r = check_launch("conv2d(im2col)", launched);
    if (r) return r;
    // y(image*ohw + pixel, channel) = sum_kk cols[kk][m] W[channel][kk] + b: A is the
    // patch matrix read MN-major, the epilogue writes NCHW.
    GemmArgs<T> p{};
    p.m = rows; p.n = s->c_out; p.k = kp;
    p.a = (const T*)cols; p.lda = ldm; p.stride_a = 0;
    p.b = wk; p.ldb = kp; p.stride_b = 0;
    p.c = (T*)y; p.ldc = ohw; p.stride_c = s->c_out * ohw;
    p.bias = (const T*)b;
    p.alpha = T(1); p.beta = T(0);
    p.trans_a = 1; p.trans_b = 1;
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
  const int64_t kp = patch_rows(*s), ldm = patch_ld(*s), K = s->c * s->kh * s->kw;
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
      // dW[channel][kk] = sum over (image, pixel) of G[image][channel][pixel] cols[kk][m]:
      // both operands K-major, A folded over the images of the NCHW gradient. The product
      // has kp columns; columns K..kp-1 (zero patch rows) are not stored.
      GemmArgs<T> p{};
      p.m = s->c_out; p.n = K; p.k = rows;
      p.a = (const T*)g; p.lda = ohw; p.stride_a = s->c_out * ohw; p.a_fold = ohw;
      p.b = (const T*)cols; p.ldb = ldm; p.stride_b = 0;
      p.c = (T*)gw; p.ldc = K; p.stride_c = 0;
      p.alpha = T(1); p.beta = T(0);
      p.trans_a = 0; p.trans_b = 1;
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
      launch_channel_sums<T, MODE_SUM>((const T*)g, nullptr, nullptr, s->n, s->c_out, ohw,
                                       chunks, partial, st);
      channel_total_kernel<T><<<(unsigned)((s->c_out + 127) / 128), 128, 0, st>>>(
          partial, chunks, s->c_out, (T*)gb);
      int r = check_launch("conv2d backward(bias)", 2);
      if (r) return r;
    }
    if (gx) {
      const T* wk = (const T*)w;
      if (kp != K) {
        pad_rows_kernel<T><<<grid_for(s->c_out * kp, kThreads), kThreads, 0, st>>>(
            (const T*)w, (T*)base, s->c_out, K, kp);
        int r = check_launch("conv2d backward(pad)");
        if (r) return r;
        wk = (const T*)base;
      }
      // dcols[kk][image*ohw + pixel] = sum_ch G[image][ch][pixel] W[ch][kk], per image: rows
      // = pixels (A = the image's gradient, MN-major), columns = patch rows (B = W, shared),
      // written column-major by the NCHW epilogue so the patch-major layout comes out.
      T* dcols = reinterpret_cast<T*>(base + L.wpad + L.ws);
      GemmArgs<T> p{};
      p.m = ohw; p.n = kp; p.k = s->c_out;
      p.a = (const T*)g; p.lda = ohw; p.stride_a = s->c_out * ohw;
      p.b = wk; p.ldb = kp; p.stride_b = 0;
      p.c = dcols; p.ldc = ldm; p.stride_c = 0; p.stride_ch = ohw;
      p.alpha = T(1); p.beta = T(0);
      p.trans_a = 1; p.trans_b = 0;
      p.batch = s->n;
      p.c_hw = ohw;
      int r = gemm_run<T>(p, st);
      if (r) return r;
      const dim3 grid = position_grid(s->h * s->w, s->c, s->n);
      const int64_t win = std::max(s->kh, s->kw);
      if (win <= 3)
        launch_pdl(col2im_kernel<T, 3>, dim3(grid), dim3(kThreads), 0, st,
                   dcols, (T*)gx, *s, ldm);
      else if (win <= 7)
        launch_pdl(col2im_kernel<T, 7>, dim3(grid), dim3(kThreads), 0, st,
                   dcols, (T*)gx, *s, ldm);
      else if (win <= 16)
        launch_pdl(col2im_kernel<T, 16>, dim3(grid), dim3(kThreads), 0, st,
                   dcols, (T*)gx, *s, ldm);
      else
        col2im_large_kernel<T><<<grid, kThreads, 0, st>>>(dcols, (T*)gx, *s, ldm);
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
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    launch_channel_sums<T, MODE_STATS>((const T*)x, nullptr, nullptr, n, c, hw, chunks, partial,
                                       st);
    launch_pdl(bn_stats_final_kernel<T>, dim3((unsigned)((c + 127) / 128)), dim3(128), 0, st,
               partial, chunks, (const T*)x, c, hw, (double)(n * hw), (T*)mean, (T*)rstd,
               (T*)running_mean, (T*)running_var, momentum, eps);
    if (plane_vec4<T>(hw, {x, y}))
      launch_pdl(bn_apply_kernel<T, 4>, dim3(plane_grid(hw / 4, n * c)), dim3(kThreads), 0, st,
                 (const T*)x, (const T*)w, (const T*)b, (const T*)mean, (const T*)rstd, (T*)y,
                 n * c, c, hw);
    else
      launch_pdl(bn_apply_kernel<T, 1>, dim3(plane_grid(hw, n * c)), dim3(kThreads), 0, st,
                 (const T*)x, (const T*)w, (const T*)b, (const T*)mean, (const T*)rstd, (T*)y,
                 n * c, c, hw);
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
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* coef = reinterpret_cast<T*>((uint8_t*)scratch + coef_off);
    launch_channel_sums<T, MODE_GRAD>((const T*)g, (const T*)x, (const T*)mean, n, c, hw,
                                      chunks, partial, st);
    launch_pdl(bn_grad_final_kernel<T>, dim3((unsigned)((c + 127) / 128)), dim3(128), 0, st,
               partial, chunks, c, (double)(n * hw), (const T*)w, (const T*)rstd, (T*)gw, (T*)gb,
               gx ? coef : nullptr);
    int launched = 2;
    if (gx) {
      if (plane_vec4<T>(hw, {g, x, gx}))
        launch_pdl(bn_grad_input_kernel<T, 4>, dim3(plane_grid(hw / 4, n * c)), dim3(kThreads), 0,
                   st,
                   (const T*)g, (const T*)x, (const T*)mean, (const T*)rstd, coef, (T*)gx, n * c,
                   c, hw);
      else
        launch_pdl(bn_grad_input_kernel<T, 1>, dim3(plane_grid(hw, n * c)), dim3(kThreads), 0, st,
                   (const T*)g, (const T*)x, (const T*)mean, (const T*)rstd, coef, (T*)gx, n * c,
                   c, hw);
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
    if (pool2x2<T>(*s, {x, y, argmax})) {
      const int64_t planes = s->n * s->c;
      launch_pdl(maxpool2x2_fwd_kernel, dim3(pool_blocks(planes * (s->h / 2) * (s->w / 4))),
                 dim3(kThreads), 0, st,
                 (const float*)x, (float*)y, argmax, planes, (int)s->h, (int)s->w);
      return check_launch("max_pool2d");
    }
    const dim3 grid = position_grid(s->oh * s->ow, s->n * s->c);
    maxpool_fwd_kernel<T><<<grid, kThreads, 0, st>>>((const T*)x, (T*)y, argmax, *s);
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
    if (pool2x2<T>(*s, {g, argmax, gx})) {
      const int64_t planes = s->n * s->c;
      launch_pdl(maxpool2x2_bwd_kernel, dim3(pool_blocks(planes * (s->h / 2) * (s->w / 4))),
                 dim3(kThreads), 0, st,
                 (const float*)g, argmax, (float*)gx, planes, (int)s->h, (int)s->w);
      return check_launch("max_pool2d backward");
    }
    const dim3 grid = position_grid(s->h * s->w, s->n * s->c);
    if (s->sh >= s->kh && s->sw >= s->kw)
      maxpool_bwd_kernel<T, true><<<grid, kThreads, 0, st>>>((const T*)g, argmax, (T*)gx, *s);
    else
      maxpool_bwd_kernel<T, false><<<grid, kThreads, 0, st>>>((const T*)g, argmax, (T*)gx, *s);
    return check_launch("max_pool2d backward");
  });
}

int tg_max_pool2d_gather(int dtype, const tg_conv_shape* s, const void* u,
                         const uint8_t* argmax, void* out, void* stream) {
  int rc = check_conv(s, true);
  if (rc) return rc;
  TG_CHECK_ARG(s->kh * s->kw <= 256, "max_pool2d: at most 256 cells per window");
  if (s->n * s->c * s->oh * s->ow == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const dim3 grid = position_grid(s->oh * s->ow, s->n * s->c);
    maxpool_gather_kernel<T><<<grid, kThreads, 0, st>>>((const T*)u, argmax, (T*)out, *s);
    return check_launch("max_pool2d gather");
  });
}

}  // extern "C"
