// Embedding gather / scatter-add (ops/layers.py:192-232) and softmax cross-entropy with the
// class axis last (ops/loss.py:23-97, ops/activation.py:48-52).
#include "common.cuh"

namespace tg {
namespace {

// ---------------------------------------------------------------- embedding
template <typename T>
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ w,
                                 T* __restrict__ out, int64_t n, int64_t dim) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const T* src = w + ids[r] * dim;
    T* dst = out + r * dim;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) dst[c] = src[c];
  }
}

__global__ void embed_fwd_vec4_kernel(const int64_t* __restrict__ ids, const float4* __restrict__ w,
                                      float4* __restrict__ out, int64_t n, int64_t dim4) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const float4* src = w + ids[r] * dim4;
    float4* dst = out + r * dim4;
    for (int64_t c = threadIdx.x; c < dim4; c += blockDim.x) dst[c] = src[c];
  }
}

// One block per run of equal ids in the stably sorted order: sums that id's gradient rows in
// sorted order (the reference's argsort + add.reduceat), then writes or adds the row.
template <typename T>
__global__ void embed_bwd_kernel(const T* __restrict__ g, const int64_t* __restrict__ order,
                                 const int64_t* __restrict__ seg_start,
                                 const int64_t* __restrict__ seg_id, int64_t nseg,
                                 T* __restrict__ gw, int64_t dim, int accumulate) {
  for (int64_t s = blockIdx.x; s < nseg; s += gridDim.x) {
    const int64_t a = seg_start[s], e = seg_start[s + 1];
    T* dst = gw + seg_id[s] * dim;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
      T acc = T(0);
      for (int64_t i = a; i < e; ++i) acc += g[order[i] * dim + c];
      dst[c] = accumulate ? dst[c] + acc : acc;
    }
  }
}

// ---------------------------------------------------------------- cross entropy
template <typename T>
struct MaxSum {
  T m, s;
};

template <typename T>
__device__ __forceinline__ MaxSum<T> ms_combine(MaxSum<T> a, MaxSum<T> b) {
  const T m = fmax(a.m, b.m);
  if (m == T(-INFINITY)) return {m, T(0)};
  return {m, a.s * dev_exp<T>(a.m - m) + b.s * dev_exp<T>(b.m - m)};
}

template <typename T>
__device__ __forceinline__ void ms_push(MaxSum<T>& a, T x) {
  if (x > a.m) {
    a.s = a.s * dev_exp<T>(a.m - x) + T(1);
    a.m = x;
  } else {
    a.s += dev_exp<T>(x - a.m);
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
ce_fwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ targets,
              T* __restrict__ lse_out, T* __restrict__ row_loss, int64_t rows, int64_t classes,
              int64_t ignore_index, int* bad_target) {
  __shared__ T shm[32], shs[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* x = logits + r * classes;
    MaxSum<T> acc{T(-INFINITY), T(0)};
    if (VEC) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      for (int64_t c = threadIdx.x; c < classes / 4; c += blockDim.x) {
        const float4 v = x4[c];
        ms_push<T>(acc, (T)v.x); ms_push<T>(acc, (T)v.y);
        ms_push<T>(acc, (T)v.z); ms_push<T>(acc, (T)v.w);
      }
    } else {
      for (int64_t c = threadIdx.x; c < classes; c += blockDim.x) ms_push<T>(acc, x[c]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum<T> other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
      acc = ms_combine(acc, other);
    }
    if (lane == 0) { shm[wid] = acc.m; shs[wid] = acc.s; }
    __syncthreads();
    if (threadIdx.x == 0) {
      MaxSum<T> t{shm[0], shs[0]};
      for (int i = 1; i < (int)(blockDim.x >> 5); ++i) t = ms_combine(t, MaxSum<T>{shm[i], shs[i]});
      const T lse = t.m == T(-INFINITY) ? t.m : t.m + dev_log<T>(t.s);
      lse_out[r] = lse;
      const int64_t tg = targets[r];
      T loss = T(0);
      if (tg != ignore_index) {
        if (tg < 0 || tg >= classes) {
          if (bad_target) *bad_target = 1;
        } else {
          loss = lse - x[tg];
        }
      }
      row_loss[r] = loss;
    }
    __syncthreads();
  }
}

template <typename T>
__global__ void ce_reduce_kernel(const T* __restrict__ row_loss, const int64_t* __restrict__ targets,
                                 int64_t rows, int64_t ignore_index, int reduction,
                                 T* __restrict__ out, int64_t* __restrict__ n_valid_out) {
  __shared__ double sh[32];
  double s = 0.0, cnt = 0.0;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    s += (double)row_loss[r];
    cnt += targets[r] != ignore_index ? 1.0 : 0.0;
  }
  s = block_sum(s, sh);
  cnt = block_sum(cnt, sh);
  if (threadIdx.x == 0) {
    const int64_t nv = (int64_t)cnt;
    if (n_valid_out) *n_valid_out = nv;
    if (reduction == 0) out[0] = (T)(s / (double)(nv > 1 ? nv : 1));
    else out[0] = (T)s;
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
ce_bwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ targets,
              const T* __restrict__ lse, const T* __restrict__ g, const int64_t* __restrict__ n_valid,
              T* __restrict__ grad, int64_t rows, int64_t classes, int64_t ignore_index,
              int reduction) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t tg = targets[r];
    const bool valid = tg != ignore_index;
    T scale;
    if (reduction == 2) scale = g[r];
    else if (reduction == 0) scale = g[0] / (T)(n_valid[0] > 1 ? n_valid[0] : 1);
    else scale = g[0];
    if (!valid) scale = T(0);
    const T l = lse[r];
    const T* x = logits + r * classes;
    T* d = grad + r * classes;
    if (VEC) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      float4* d4 = reinterpret_cast<float4*>(d);
      for (int64_t c = threadIdx.x; c < classes / 4; c += blockDim.x) {
        const float4 v = x4[c];
        float4 o;
        o.x = (float)((dev_exp<T>((T)v.x - l) - (4 * c + 0 == tg ? T(1) : T(0))) * scale);
        o.y = (float)((dev_exp<T>((T)v.y - l) - (4 * c + 1 == tg ? T(1) : T(0))) * scale);
        o.z = (float)((dev_exp<T>((T)v.z - l) - (4 * c + 2 == tg ? T(1) : T(0))) * scale);
        o.w = (float)((dev_exp<T>((T)v.w - l) - (4 * c + 3 == tg ? T(1) : T(0))) * scale);
        d4[c] = o;
      }
    } else {
      for (int64_t c = threadIdx.x; c < classes; c += blockDim.x)
        d[c] = (dev_exp<T>(x[c] - l) - (c == tg ? T(1) : T(0))) * scale;
    }
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int tg_embedding_forward(int dtype, const int64_t* ids, const void* w, void* out, int64_t n,
                         int64_t num, int64_t dim, void* stream) {
  (void)num;
  if (n <= 0 || dim <= 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  const unsigned grid = (unsigned)(n < 148 * 16 ? n : 148 * 16);
  if (dtype == TG_F32 && dim % 4 == 0 && aligned16(w) && aligned16(out)) {
    embed_fwd_vec4_kernel<<<grid, 128, 0, s>>>(ids, (const float4*)w, (float4*)out, n, dim / 4);
    return check_launch("embedding_forward");
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    embed_fwd_kernel<T><<<grid, 128, 0, s>>>(ids, (const T*)w, (T*)out, n, dim);
    return check_launch("embedding_forward");
  });
}

int tg_embedding_backward(int dtype, const void* g, const int64_t* order,
                          const int64_t* seg_start, const int64_t* seg_id, int64_t nseg,
                          void* gw, int64_t num, int64_t dim, int accumulate, void* stream) {
  cudaStream_t s = as_stream(stream);
  const size_t es = dtype == TG_F64 ? 8 : 4;
  if (!accumulate && num * dim > 0) TG_CUDA_TRY(cudaMemsetAsync(gw, 0, num * dim * es, s));
  if (nseg <= 0 || dim <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const unsigned grid = (unsigned)(nseg < 148 * 32 ? nseg : 148 * 32);
    const int threads = dim >= 256 ? 256 : (dim >= 128 ? 128 : 64);
    embed_bwd_kernel<T><<<grid, threads, 0, s>>>((const T*)g, order, seg_start, seg_id, nseg,
                                                 (T*)gw, dim, 1);
    return check_launch("embedding_backward");
  });
}

int tg_cross_entropy_forward(int dtype, const void* logits, const int64_t* targets, void* lse,
                             void* row_loss, void* out, int64_t rows, int64_t classes,
                             int64_t ignore_index, int reduction, int64_t* n_valid_dev,
                             int* bad_target_dev, void* stream) {
  TG_CHECK_ARG(classes > 0 && rows >= 0, "cross_entropy: bad shape");
  TG_CHECK_ARG(reduction >= 0 && reduction <= 2, "cross_entropy: bad reduction %d", reduction);
  cudaStream_t s = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    if (rows > 0) {
      const unsigned grid = (unsigned)(rows < 148 * 16 ? rows : 148 * 16);
      if (sizeof(T) == 4 && classes % 4 == 0 && aligned16(logits))
        ce_fwd_kernel<T, true><<<grid, 256, 0, s>>>((const T*)logits, targets, (T*)lse,
                                                    (T*)row_loss, rows, classes, ignore_index,
                                                    bad_target_dev);
      else
        ce_fwd_kernel<T, false><<<grid, 256, 0, s>>>((const T*)logits, targets, (T*)lse,
                                                     (T*)row_loss, rows, classes, ignore_index,
                                                     bad_target_dev);
    }
    if (reduction != 2)
      ce_reduce_kernel<T><<<1, 1024, 0, s>>>((const T*)row_loss, targets, rows, ignore_index,
                                             reduction, (T*)out, n_valid_dev);
    return check_launch("cross_entropy_forward", (rows > 0 ? 1 : 0) + (reduction != 2 ? 1 : 0));
  });
}

int tg_cross_entropy_backward(int dtype, const void* logits, const int64_t* targets,
                              const void* lse, const void* g_dev, const int64_t* n_valid_dev,
                              void* grad, int64_t rows, int64_t classes, int64_t ignore_index,
                              int reduction, void* stream) {
  if (rows <= 0) return TG_OK;
  TG_CHECK_ARG(reduction != 0 || n_valid_dev, "cross_entropy_backward: n_valid is NULL");
  cudaStream_t s = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const unsigned grid = (unsigned)(rows < 148 * 16 ? rows : 148 * 16);
    if (sizeof(T) == 4 && classes % 4 == 0 && aligned16(logits) && aligned16(grad))
      ce_bwd_kernel<T, true><<<grid, 256, 0, s>>>((const T*)logits, targets, (const T*)lse,
                                                  (const T*)g_dev, n_valid_dev, (T*)grad, rows,
                                                  classes, ignore_index, reduction);
    else
      ce_bwd_kernel<T, false><<<grid, 256, 0, s>>>((const T*)logits, targets, (const T*)lse,
                                                   (const T*)g_dev, n_valid_dev, (T*)grad, rows,
                                                   classes, ignore_index, reduction);
    return check_launch("cross_entropy_backward");
  });
}

}  // extern "C"
