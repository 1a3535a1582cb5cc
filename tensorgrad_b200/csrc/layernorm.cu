// Row-wise LayerNorm forward and VJP (ops/layers.py:65-141).
//
// One warp per row with the row held in registers (cols <= 1024): the mean is taken first
// and the variance from the centred values, as the reference does, so nothing is re-read
// from HBM. fp32 rows whose length is a multiple of 4 move as 16-byte vectors; other shapes
// and float64 use the scalar kernels. The weight/bias gradients are column sums over rows:
// each block reduces its warps' per-lane sums in shared memory and writes one partial row to
// `scratch`; a second kernel sums the partial rows in a fixed order (deterministic), 32
// columns x 8 row groups per block.
#include <algorithm>
#include <initializer_list>

#include "common.cuh"
#include "reduce.cuh"

namespace tg {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxPartials = 2 * 148;  // blocks of the backward pass (partial rows)

// ---------------------------------------------------------------- scalar kernels
template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32)
ln_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
              T* __restrict__ y, T* __restrict__ mean_out, T* __restrict__ rstd_out,
              int64_t rows, int cols, T eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const T* xr = x + r * cols;
    T v[V];
    T s = T(0);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int c = lane + 32 * j;
      v[j] = c < cols ? xr[c] : T(0);
      s += v[j];
    }
    const T mean = warp_sum(s) / T(cols);
    T q = T(0);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int c = lane + 32 * j;
      v[j] = c < cols ? v[j] - mean : T(0);
      q += v[j] * v[j];
    }
    const T rstd = T(1) / dev_sqrt<T>(warp_sum(q) / T(cols) + eps);
    T* yr = y + r * cols;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int c = lane + 32 * j;
      if (c < cols) {
        T o = v[j] * rstd;
        if (w) o *= w[c];
        if (b) o += b[c];
        yr[c] = o;
      }
    }
    if (lane == 0) {
      mean_out[r] = mean;
      rstd_out[r] = rstd;
    }
  }
}

// Block-level reduction of per-lane column sums (sh: [kWarps][2][cols]) into one partial row.
template <typename T>
__device__ __forceinline__ void ln_block_partials(T* sh, T* __restrict__ part_w,
                                                  T* __restrict__ part_b, int cols) {
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    T sw = T(0), sb = T(0);
#pragma unroll
    for (int i = 0; i < kWarps; ++i) {
      sw += sh[(i * 2 + 0) * cols + c];
      sb += sh[(i * 2 + 1) * cols + c];
    }
    part_w[(int64_t)blockIdx.x * cols + c] = sw;
    part_b[(int64_t)blockIdx.x * cols + c] = sb;
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32)
ln_bwd_kernel(const T* __restrict__ g, const T* __restrict__ x, const T* __restrict__ w,
              const T* __restrict__ mean_in, const T* __restrict__ rstd_in, T* __restrict__ gx,
              T* __restrict__ part_w, T* __restrict__ part_b, int64_t rows, int cols) {
  extern __shared__ unsigned char smem_raw[];
  T* sh = reinterpret_cast<T*>(smem_raw);  // [kWarps][2][cols]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t warp0 = (int64_t)blockIdx.x * kWarps + wid;
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  const bool want_wb = part_w != nullptr;
  T aw[V], ab[V];
#pragma unroll
  for (int j = 0; j < V; ++j) aw[j] = ab[j] = T(0);
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const T* xr = x + r * cols;
    const T* gr = g + r * cols;
    const T mean = mean_in[r], rstd = rstd_in[r];
    T xh[V], gh[V];
    T s1 = T(0), s2 = T(0);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int c = lane + 32 * j;
      if (c < cols) {
        xh[j] = (xr[c] - mean) * rstd;
        const T gv = gr[c];
        aw[j] += gv * xh[j];
        ab[j] += gv;
        gh[j] = w ? gv * w[c] : gv;
      } else {
        xh[j] = gh[j] = T(0);
      }
      s1 += gh[j];
      s2 += gh[j] * xh[j];
    }
    if (gx) {
      const T m1 = warp_sum(s1) / T(cols), m2 = warp_sum(s2) / T(cols);
      T* gxr = gx + r * cols;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int c = lane + 32 * j;
        if (c < cols) gxr[c] = rstd * (gh[j] - m1 - xh[j] * m2);
      }
    }
  }
  if (!want_wb) return;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c = lane + 32 * j;
    if (c < cols) {
      sh[(wid * 2 + 0) * cols + c] = aw[j];
      sh[(wid * 2 + 1) * cols + c] = ab[j];
    }
  }
  ln_block_partials<T>(sh, part_w, part_b, cols);
}

// ---------------------------------------------------------------- fp32 16-byte kernels
// Lane `lane` holds the float4 vectors lane, lane + 32, ... of its row (NV of them).
__device__ __forceinline__ float sum4(float4 v) { return (v.x + v.y) + (v.z + v.w); }

template <int NV>
__global__ void __launch_bounds__(kWarps * 32)
ln_fwd_vec4(const float* __restrict__ x, const float* __restrict__ w,
            const float* __restrict__ b, float* __restrict__ y, float* __restrict__ mean_out,
            float* __restrict__ rstd_out, int64_t rows, int cols, float eps) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int nv = cols >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + r * cols);
  float4 v[NV];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = lane + 32 * j;
    v[j] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += sum4(v[j]);
  }
  const float mean = warp_sum(s) / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      v[j].x -= mean; v[j].y -= mean; v[j].z -= mean; v[j].w -= mean;
      q += (v[j].x * v[j].x + v[j].y * v[j].y) + (v[j].z * v[j].z + v[j].w * v[j].w);
    }
  }
  const float rstd = 1.f / sqrtf(warp_sum(q) / (float)cols + eps);
  float4* yr = reinterpret_cast<float4*>(y + r * cols);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = lane + 32 * j;
    if (i < nv) {
      float4 o = make_float4(v[j].x * rstd, v[j].y * rstd, v[j].z * rstd, v[j].w * rstd);
      if (w) {
        const float4 ww = w4[i];
        o.x *= ww.x; o.y *= ww.y; o.z *= ww.z; o.w *= ww.w;
      }
      if (b) {
        const float4 bb = b4[i];
        o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
      }
      yr[i] = o;
    }
  }
  if (lane == 0) {
    mean_out[r] = mean;
    rstd_out[r] = rstd;
  }
}

// The fp32 VJP with 16-byte rows. The weight/bias column sums accumulate in shared memory
// (each warp its own pair of rows there), not in registers: that keeps a thread near 64
// registers, so three or four blocks share an SM and more rows are in flight (a warp's loads
// of one row are its only memory-level parallelism). Up to kMaxPartialsVec blocks.
template <int NV>
__global__ void __launch_bounds__(kWarps * 32, 3)
ln_bwd_vec4(const float* __restrict__ g, const float* __restrict__ x,
            const float* __restrict__ w, const float* __restrict__ mean_in,
            const float* __restrict__ rstd_in, float* __restrict__ gx,
            float* __restrict__ part_w, float* __restrict__ part_b, int64_t rows, int cols) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  extern __shared__ unsigned char smem_raw[];
  float* sh = reinterpret_cast<float*>(smem_raw);  // [kWarps][2][cols]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t warp0 = (int64_t)blockIdx.x * kWarps + wid;
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  const int nv = cols >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4* acc_w = reinterpret_cast<float4*>(sh + (wid * 2 + 0) * cols);
  float4* acc_b = reinterpret_cast<float4*>(sh + (wid * 2 + 1) * cols);
  if (part_w) {
    for (int i = lane; i < nv; i += 32) acc_w[i] = acc_b[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * cols);
    const float4* gr = reinterpret_cast<const float4*>(g + r * cols);
    const float mean = mean_in[r], rstd = rstd_in[r];
    float4 xv[NV], gv[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      xv[j] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      gv[j] = i < nv ? gr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      // xv becomes xhat, gv becomes g * w (the column sums take the raw g first).
      xv[j] = make_float4((xv[j].x - mean) * rstd, (xv[j].y - mean) * rstd,
                          (xv[j].z - mean) * rstd, (xv[j].w - mean) * rstd);
      if (part_w && i < nv) {
        float4 a = acc_w[i], b = acc_b[i];
        a.x += gv[j].x * xv[j].x; a.y += gv[j].y * xv[j].y;
        a.z += gv[j].z * xv[j].z; a.w += gv[j].w * xv[j].w;
        b.x += gv[j].x; b.y += gv[j].y; b.z += gv[j].z; b.w += gv[j].w;
        acc_w[i] = a;
        acc_b[i] = b;
      }
      if (w && i < nv) {
        const float4 ww = w4[i];
        gv[j] = make_float4(gv[j].x * ww.x, gv[j].y * ww.y, gv[j].z * ww.z, gv[j].w * ww.w);
      }
      s1 += sum4(gv[j]);
      s2 += (gv[j].x * xv[j].x + gv[j].y * xv[j].y) + (gv[j].z * xv[j].z + gv[j].w * xv[j].w);
    }
    if (gx) {
      const float m1 = warp_sum(s1) / (float)cols, m2 = warp_sum(s2) / (float)cols;
      float4* gxr = reinterpret_cast<float4*>(gx + r * cols);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = lane + 32 * j;
        if (i < nv)
          gxr[i] = make_float4(rstd * (gv[j].x - m1 - xv[j].x * m2),
                               rstd * (gv[j].y - m1 - xv[j].y * m2),
                               rstd * (gv[j].z - m1 - xv[j].z * m2),
                               rstd * (gv[j].w - m1 - xv[j].w * m2));
      }
    }
  }
  if (!part_w) return;
  ln_block_partials<float>(sh, part_w, part_b, cols);
}

// Sum of the partial rows: block (32 columns x 8 row groups), then the 8 group sums in order.
template <typename T>
__global__ void __launch_bounds__(256)
ln_final_kernel(const T* __restrict__ part_w, const T* __restrict__ part_b, T* __restrict__ gw,
                T* __restrict__ gb, int nparts, int cols) {
  __shared__ T sw_sh[8][32], sb_sh[8][32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  T sw = T(0), sb = T(0);
  if (c < cols) {
#pragma unroll 4
    for (int i = ty; i < nparts; i += 8) {
      sw += part_w[(int64_t)i * cols + c];
      sb += part_b[(int64_t)i * cols + c];
    }
  }
  sw_sh[ty][tx] = sw;
  sb_sh[ty][tx] = sb;
  __syncthreads();
  if (ty == 0 && c < cols) {
    T tw = T(0), tb = T(0);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      tw += sw_sh[k][tx];
      tb += sb_sh[k][tx];
    }
    if (gw) gw[c] = tw;
    if (gb) gb[c] = tb;
  }
}

// fp32 partial rows of a multiple of 4 columns: a block covers 32 columns as 8 float4 lanes
// by 32 row groups (each group sums every 32nd partial row, four independent chains), then the
// 32 group sums are added in order. Four times the row parallelism of the scalar kernel: its
// threads are latency-bound on the serial partial-row loads.
__global__ void __launch_bounds__(256)
ln_final_vec4(const float4* __restrict__ part_w, const float4* __restrict__ part_b,
              float* __restrict__ gw, float* __restrict__ gb, int nparts, int cols) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  __shared__ float4 sw_sh[32][8], sb_sh[32][8];
  const int q = threadIdx.x & 7, grp = threadIdx.x >> 3;
  const int nq = cols >> 2, cq = blockIdx.x * 8 + q;
  float4 w0 = make_float4(0.f, 0.f, 0.f, 0.f), w1 = w0, b0 = w0, b1 = w0;
  if (cq < nq) {
    int i = grp;
    for (; i + 32 < nparts; i += 64) {
      const float4 a = part_w[(int64_t)i * nq + cq], a2 = part_w[(int64_t)(i + 32) * nq + cq];
      const float4 b = part_b[(int64_t)i * nq + cq], b2 = part_b[(int64_t)(i + 32) * nq + cq];
      w0.x += a.x; w0.y += a.y; w0.z += a.z; w0.w += a.w;
      w1.x += a2.x; w1.y += a2.y; w1.z += a2.z; w1.w += a2.w;
      b0.x += b.x; b0.y += b.y; b0.z += b.z; b0.w += b.w;
      b1.x += b2.x; b1.y += b2.y; b1.z += b2.z; b1.w += b2.w;
    }
    if (i < nparts) {
      const float4 a = part_w[(int64_t)i * nq + cq], b = part_b[(int64_t)i * nq + cq];
      w0.x += a.x; w0.y += a.y; w0.z += a.z; w0.w += a.w;
      b0.x += b.x; b0.y += b.y; b0.z += b.z; b0.w += b.w;
    }
  }
  sw_sh[grp][q] = make_float4(w0.x + w1.x, w0.y + w1.y, w0.z + w1.z, w0.w + w1.w);
  sb_sh[grp][q] = make_float4(b0.x + b1.x, b0.y + b1.y, b0.z + b1.z, b0.w + b1.w);
  __syncthreads();
  if (grp == 0 && cq < nq) {
    float4 tw = make_float4(0.f, 0.f, 0.f, 0.f), tb = tw;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float4 a = sw_sh[k][q], b = sb_sh[k][q];
      tw.x += a.x; tw.y += a.y; tw.z += a.z; tw.w += a.w;
      tb.x += b.x; tb.y += b.y; tb.z += b.z; tb.w += b.w;
    }
    if (gw) reinterpret_cast<float4*>(gw)[cq] = tw;
    if (gb) reinterpret_cast<float4*>(gb)[cq] = tb;
  }
}

int ln_blocks(int64_t rows) {
  int64_t b = (rows + kWarps - 1) / kWarps;
  if (b > kMaxPartials) b = kMaxPartials;
  if (b < 1) b = 1;
  return (int)b;
}

// The vector VJP's grid: three blocks per SM (its occupancy), each warp a row at a time.
constexpr int kMaxPartialsVec = 3 * 148;
int ln_blocks_vec(int64_t rows) {
  int64_t b = (rows + kWarps - 1) / kWarps;
  if (b > kMaxPartialsVec) b = kMaxPartialsVec;
  if (b < 1) b = 1;
  return (int)b;
}

bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T, int V>
int ln_forward_v(const T* x, const T* w, const T* b, T* y, T* mean, T* rstd, int64_t rows,
                 int cols, T eps, cudaStream_t s) {
  ln_fwd_kernel<T, V><<<ln_blocks(rows), kWarps * 32, 0, s>>>(x, w, b, y, mean, rstd, rows,
                                                              cols, eps);
  return check_launch("layer_norm_forward");
}

template <int NV>
int ln_forward_vec(const float* x, const float* w, const float* b, float* y, float* mean,
                   float* rstd, int64_t rows, int cols, float eps, cudaStream_t s) {
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  launch_pdl(ln_fwd_vec4<NV>, dim3(grid), dim3(kWarps * 32), 0, s,
             x, w, b, y, mean, rstd, rows, cols, eps);
  return check_launch("layer_norm_forward");
}

template <typename K>
int set_smem(K kernel, size_t smem) {
  if (smem > 48 * 1024)
    TG_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
  return TG_OK;
}

template <typename T, int V>
int ln_backward_v(const T* g, const T* x, const T* w, const T* mean, const T* rstd, T* gx,
                  T* gw, T* gb, int64_t rows, int cols, void* scratch, cudaStream_t s) {
  const int nb = ln_blocks(rows);
  T* part_w = nullptr;
  T* part_b = nullptr;
  if (gw || gb) {
    part_w = reinterpret_cast<T*>(scratch);
    part_b = part_w + (int64_t)nb * cols;
  }
  const size_t smem = (gw || gb) ? (size_t)kWarps * 2 * cols * sizeof(T) : 0;
  int rc = set_smem(ln_bwd_kernel<T, V>, smem);
  if (rc) return rc;
  ln_bwd_kernel<T, V><<<nb, kWarps * 32, smem, s>>>(g, x, w, mean, rstd, gx, part_w, part_b,
                                                    rows, cols);
  if (gw || gb)
    ln_final_kernel<T><<<(cols + 31) / 32, 256, 0, s>>>(part_w, part_b, gw, gb, nb, cols);
  return check_launch("layer_norm_backward", (gw || gb) ? 2 : 1);
}

template <int NV>
int ln_backward_vec(const float* g, const float* x, const float* w, const float* mean,
                    const float* rstd, float* gx, float* gw, float* gb, int64_t rows, int cols,
                    void* scratch, cudaStream_t s) {
  const int nb = ln_blocks_vec(rows);
  float* part_w = nullptr;
  float* part_b = nullptr;
  if (gw || gb) {
    part_w = reinterpret_cast<float*>(scratch);
    part_b = part_w + (int64_t)nb * cols;
  }
  const size_t smem = (gw || gb) ? (size_t)kWarps * 2 * cols * sizeof(float) : 0;
  int rc = set_smem(ln_bwd_vec4<NV>, smem);
  if (rc) return rc;
  launch_pdl(ln_bwd_vec4<NV>, dim3(nb), dim3(kWarps * 32), smem, s,
             g, x, w, mean, rstd, gx, part_w, part_b, rows,
                                                cols);
  if ((gw || gb) && aligned16(gw) && aligned16(gb) && aligned16(part_w))
    launch_pdl(ln_final_vec4, dim3((cols + 31) / 32), dim3(256), 0, s,
               reinterpret_cast<const float4*>(part_w),
                                                   reinterpret_cast<const float4*>(part_b), gw,
                                                   gb, nb, cols);
  else if (gw || gb)
    ln_final_kernel<float><<<(cols + 31) / 32, 256, 0, s>>>(part_w, part_b, gw, gb, nb, cols);
  return check_launch("layer_norm_backward", (gw || gb) ? 2 : 1);
}

// fp32 rows of a multiple of 4 columns with 16-byte aligned buffers take the vector kernels.
bool use_vec4(int cols, std::initializer_list<const void*> ptrs) {
  if (cols % 4) return false;
  for (const void* p : ptrs)
    if (!aligned16(p)) return false;
  return true;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int tg_layer_norm_forward(int dtype, const void* x, const void* w, const void* b, void* y,
                          void* mean, void* rstd, int64_t rows, int64_t cols, double eps,
                          void* stream) {
  TG_CHECK_ARG(cols > 0 && cols <= 1024, "layer_norm: %lld columns (supported: 1..1024)",
               (long long)cols);
  if (rows <= 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == TG_F32 && use_vec4((int)cols, {x, w, b, y})) {
    const int c = (int)cols, nv = (c / 4 + 31) / 32;
    auto* X = (const float*)x; auto* W = (const float*)w; auto* B = (const float*)b;
    auto* Y = (float*)y; auto* M = (float*)mean; auto* R = (float*)rstd;
    const float e = (float)eps;
    if (nv <= 1) return ln_forward_vec<1>(X, W, B, Y, M, R, rows, c, e, s);
    if (nv <= 2) return ln_forward_vec<2>(X, W, B, Y, M, R, rows, c, e, s);
    if (nv <= 4) return ln_forward_vec<4>(X, W, B, Y, M, R, rows, c, e, s);
    if (nv <= 6) return ln_forward_vec<6>(X, W, B, Y, M, R, rows, c, e, s);
    return ln_forward_vec<8>(X, W, B, Y, M, R, rows, c, e, s);
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const int c = (int)cols;
    auto* X = (const T*)x; auto* W = (const T*)w; auto* B = (const T*)b;
    auto* Y = (T*)y; auto* M = (T*)mean; auto* R = (T*)rstd;
    if (c <= 128) return ln_forward_v<T, 4>(X, W, B, Y, M, R, rows, c, (T)eps, s);
    if (c <= 256) return ln_forward_v<T, 8>(X, W, B, Y, M, R, rows, c, (T)eps, s);
    if (c <= 512) return ln_forward_v<T, 16>(X, W, B, Y, M, R, rows, c, (T)eps, s);
    return ln_forward_v<T, 32>(X, W, B, Y, M, R, rows, c, (T)eps, s);
  });
}

size_t tg_layer_norm_scratch_bytes(int dtype, int64_t rows, int64_t cols) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const int64_t nb = std::max<int64_t>(ln_blocks(rows), dtype == TG_F32 ? ln_blocks_vec(rows) : 0);
  return (size_t)nb * 2 * (size_t)cols * es;
}

int tg_layer_norm_backward(int dtype, const void* g, const void* x, const void* w,
                           const void* mean, const void* rstd, void* gx, void* gw, void* gb,
                           int64_t rows, int64_t cols, unsigned need, void* scratch,
                           void* stream) {
  TG_CHECK_ARG(cols > 0 && cols <= 1024, "layer_norm: %lld columns (supported: 1..1024)",
               (long long)cols);
  if (!(need & 1)) gx = nullptr;
  if (!(need & 2)) gw = nullptr;
  if (!(need & 4)) gb = nullptr;
  if (gw || gb) TG_CHECK_ARG(scratch != nullptr, "layer_norm_backward: scratch is NULL");
  cudaStream_t s = as_stream(stream);
  if (rows <= 0) {
    if (gw) TG_CUDA_TRY(cudaMemsetAsync(gw, 0, cols * (dtype == TG_F64 ? 8 : 4), s));
    if (gb) TG_CUDA_TRY(cudaMemsetAsync(gb, 0, cols * (dtype == TG_F64 ? 8 : 4), s));
    return TG_OK;
  }
  if (dtype == TG_F32 && use_vec4((int)cols, {g, x, w, gx})) {
    const int c = (int)cols, nv = (c / 4 + 31) / 32;
    auto* G = (const float*)g; auto* X = (const float*)x; auto* W = (const float*)w;
    auto* M = (const float*)mean; auto* R = (const float*)rstd;
    auto* GX = (float*)gx; auto* GW = (float*)gw; auto* GB = (float*)gb;
    if (nv <= 1) return ln_backward_vec<1>(G, X, W, M, R, GX, GW, GB, rows, c, scratch, s);
    if (nv <= 2) return ln_backward_vec<2>(G, X, W, M, R, GX, GW, GB, rows, c, scratch, s);
    if (nv <= 4) return ln_backward_vec<4>(G, X, W, M, R, GX, GW, GB, rows, c, scratch, s);
    if (nv <= 6) return ln_backward_vec<6>(G, X, W, M, R, GX, GW, GB, rows, c, scratch, s);
    return ln_backward_vec<8>(G, X, W, M, R, GX, GW, GB, rows, c, scratch, s);
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const int c = (int)cols;
    auto* G = (const T*)g; auto* X = (const T*)x; auto* W = (const T*)w;
    auto* M = (const T*)mean; auto* R = (const T*)rstd;
    if (c <= 128) return ln_backward_v<T, 4>(G, X, W, M, R, (T*)gx, (T*)gw, (T*)gb, rows, c, scratch, s);
    if (c <= 256) return ln_backward_v<T, 8>(G, X, W, M, R, (T*)gx, (T*)gw, (T*)gb, rows, c, scratch, s);
    if (c <= 512) return ln_backward_v<T, 16>(G, X, W, M, R, (T*)gx, (T*)gw, (T*)gb, rows, c, scratch, s);
    return ln_backward_v<T, 32>(G, X, W, M, R, (T*)gx, (T*)gw, (T*)gb, rows, c, scratch, s);
  });
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory for the VJP's scratch: a C or FFI host that
// binds this library without any CUDA allocator of its own, or a latency-critical path
// where cudaMalloc (which may synchronise the whole device) is not acceptable. For them
// the weight/bias partial sums live in one file-scope device array of a fixed size, shared
// by every call on a device.
#include <mutex>

namespace tg {
namespace {

constexpr size_t kLnStaticScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_ln_static_scratch[kLnStaticScratchBytes];

void* g_ln_static_ptr[kMaxDevices] = {};
std::mutex g_ln_static_mutex;

// Device address of the array on the current device. Host code only sees a stand-in
// symbol, so the address is looked up with that device current: on every call made outside
// stream capture (the lookup is cheap, and a context rebuilt after cudaDeviceReset may place
// the array elsewhere), and from the cache while `stream` is being captured, which therefore
// needs one earlier uncaptured call on the device.
int ln_static_scratch(void** out, cudaStream_t stream) {
  int dev = 0;
  TG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(TG_ERR_UNSUPPORTED, "device %d", dev);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  TG_CUDA_TRY(cudaStreamIsCapturing(stream, &capture));
  std::lock_guard<std::mutex> lock(g_ln_static_mutex);
  if (capture == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    TG_CUDA_TRY(cudaGetSymbolAddress(&p, g_ln_static_scratch));
    g_ln_static_ptr[dev] = p;
  } else if (!g_ln_static_ptr[dev]) {
    return set_error(TG_ERR_ARG,
                     "layer_norm_backward_noalloc: the first call on device %d is being "
                     "captured; make one call outside capture first", dev);
  }
  *out = g_ln_static_ptr[dev];
  return TG_OK;
}

}  // namespace
}  // namespace tg

extern "C" int tg_layer_norm_backward_noalloc(int dtype, const void* g, const void* x,
                                              const void* w, const void* mean, const void* rstd,
                                              void* gx, void* gw, void* gb, int64_t rows,
                                              int64_t cols, unsigned need, void* stream) {
  TG_CHECK_ARG(cols > 0 && cols <= 1024, "layer_norm: %lld columns (supported: 1..1024)",
               (long long)cols);
  const bool partials = (need & 2) || (need & 4);
  const size_t bytes = partials ? tg_layer_norm_scratch_bytes(dtype, rows, cols) : 0;
  if (bytes > tg::kLnStaticScratchBytes)
    return tg::set_error(TG_ERR_ARG,
                         "layer_norm_backward_noalloc: %zu bytes of partial sums exceed the "
                         "%zu-byte static scratch (rows %lld, cols %lld)",
                         bytes, tg::kLnStaticScratchBytes, (long long)rows, (long long)cols);
  void* scratch = nullptr;
  if (partials) {
    const int rc = tg::ln_static_scratch(&scratch, static_cast<cudaStream_t>(stream));
    if (rc != TG_OK) return rc;
  }
  // Every partial the second pass reads is written by the first pass of the same call, so
  // the array's previous contents never matter and nothing needs clearing.
  return tg_layer_norm_backward(dtype, g, x, w, mean, rstd, gx, gw, gb, rows, cols, need,
                                scratch, stream);
}
