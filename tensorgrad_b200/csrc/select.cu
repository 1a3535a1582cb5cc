// Selection and extrema: the broadcasting select behind where / masked_fill
// (ops/shape.py:290-328), the keep-axis max / min reductions (ops/reduce.py:70-105) and the
// non-differentiable all / any / argmax of Tensor (tensor.py:418-435).
// Both are HBM-bound grid-stride loops; neither is on a training step of the measured
// configurations, they complete the op set.
#include "common.cuh"
#include "reduce.cuh"

namespace tg {
namespace {

struct SelectDims {
  int ndim;
  int64_t shape[kMaxDims];
  int64_t sc[kMaxDims], sa[kMaxDims], sb[kMaxDims];
};

template <typename T, typename C>
__global__ void where_kernel(const C* __restrict__ cond, const T* __restrict__ a,
                             const T* __restrict__ b, T* __restrict__ out, int64_t n,
                             SelectDims d) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, oc = 0, oa = 0, ob = 0;
    for (int k = d.ndim - 1; k >= 0; --k) {
      const int64_t idx = rem % d.shape[k];
      rem /= d.shape[k];
      oc += idx * d.sc[k];
      oa += idx * d.sa[k];
      ob += idx * d.sb[k];
    }
    out[i] = cond[oc] != C(0) ? a[oa] : b[ob];
  }
}

// Elementwise comparison into bytes (Tensor's ==, !=, <, <=, >, >=): IEEE semantics, so a
// NaN compares unequal to everything, as in NumPy.
template <typename T>
__global__ void compare_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                               uint8_t* __restrict__ out, int64_t n, SelectDims d) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, oa = 0, ob = 0;
    for (int k = d.ndim - 1; k >= 0; --k) {
      const int64_t idx = rem % d.shape[k];
      rem /= d.shape[k];
      oa += idx * d.sa[k];
      ob += idx * d.sb[k];
    }
    const T x = a[oa], y = b[ob];
    bool r;
    switch (op) {
      case 0: r = x == y; break;
      case 1: r = x != y; break;
      case 2: r = x < y; break;
      case 3: r = x <= y; break;
      case 4: r = x > y; break;
      default: r = x >= y; break;
    }
    out[i] = r ? 1 : 0;
  }
}

// The extremum of two values, NaN-propagating as np.max / np.min are.
template <typename T>
__device__ __forceinline__ T pick(T x, T y, bool is_min) {
  if (x != x) return x;
  if (y != y) return y;
  return is_min ? (y < x ? y : x) : (y > x ? y : x);
}

template <typename T>
__device__ T block_extremum(T v, bool is_min, T* sh) {
  for (int o = 16; o > 0; o >>= 1) v = pick(v, __shfl_xor_sync(0xffffffffu, v, o), is_min);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  const int warps = (blockDim.x + 31) >> 5;
  if (warp == 0) {
    v = lane < warps ? sh[lane] : sh[0];
    for (int o = 16; o > 0; o >>= 1) v = pick(v, __shfl_xor_sync(0xffffffffu, v, o), is_min);
  }
  return v;
}

// One block per output element; threads stride the reduced index space.
template <typename T>
__global__ void extremum_keep_kernel(const T* __restrict__ x, T* __restrict__ out,
                                     ReduceDims d, bool is_min) {
  __shared__ T sh[32];
  for (int64_t o = blockIdx.x; o < d.out_count; o += gridDim.x) {
    int64_t base = 0, rem = o;
    for (int i = d.n_keep - 1; i >= 0; --i) {
      base += (rem % d.keep_size[i]) * d.keep_stride[i];
      rem /= d.keep_size[i];
    }
    T acc = x[base];  // the reduced set is not empty (checked by the caller)
    for (int64_t r = threadIdx.x; r < d.red_count; r += blockDim.x) {
      int64_t off = base, rr = r;
      for (int i = d.n_red - 1; i >= 0; --i) {
        off += (rr % d.red_size[i]) * d.red_stride[i];
        rr /= d.red_size[i];
      }
      acc = pick(acc, x[off], is_min);
    }
    acc = block_extremum(acc, is_min, sh);
    if (threadIdx.x == 0) out[o] = acc;
    __syncthreads();
  }
}

// all / any: one block per output element; __syncthreads_and / _or finish the block.
template <typename C>
__global__ void truth_keep_kernel(const C* __restrict__ x, uint8_t* __restrict__ out,
                                  ReduceDims d, bool is_all) {
  for (int64_t o = blockIdx.x; o < d.out_count; o += gridDim.x) {
    int64_t base = 0, rem = o;
    for (int i = d.n_keep - 1; i >= 0; --i) {
      base += (rem % d.keep_size[i]) * d.keep_stride[i];
      rem /= d.keep_size[i];
    }
    bool acc = is_all;
    for (int64_t r = threadIdx.x; r < d.red_count; r += blockDim.x) {
      int64_t off = base, rr = r;
      for (int i = d.n_red - 1; i >= 0; --i) {
        off += (rr % d.red_size[i]) * d.red_stride[i];
        rr /= d.red_size[i];
      }
      const bool nz = x[off] != C(0);  // NaN counts as true, as in NumPy
      acc = is_all ? (acc && nz) : (acc || nz);
    }
    const int res = is_all ? __syncthreads_and(acc) : __syncthreads_or(acc);
    if (threadIdx.x == 0) out[o] = res ? 1 : 0;
  }
}

// argmax: the first index of the maximum in row-major order of the reduced axes; a NaN is
// the maximum (its first occurrence), as np.argmax has it.
template <typename T>
__device__ __forceinline__ void arg_take(T& bv, int64_t& bi, T v, int64_t i) {
  bool take;
  if (bv != bv) take = (v != v) && i < bi;
  else if (v != v) take = true;
  else take = v > bv || (v == bv && i < bi);
  if (take) {
    bv = v;
    bi = i;
  }
}

template <typename T>
__global__ void argmax_keep_kernel(const T* __restrict__ x, int64_t* __restrict__ out,
                                   ReduceDims d) {
  __shared__ T sv[32];
  __shared__ int64_t si[32];
  for (int64_t o = blockIdx.x; o < d.out_count; o += gridDim.x) {
    int64_t base = 0, rem = o;
    for (int i = d.n_keep - 1; i >= 0; --i) {
      base += (rem % d.keep_size[i]) * d.keep_stride[i];
      rem /= d.keep_size[i];
    }
    T bv = x[base];  // element 0 of the reduced set (not empty: checked by the caller)
    int64_t bi = 0;
    for (int64_t r = threadIdx.x; r < d.red_count; r += blockDim.x) {
      int64_t off = base, rr = r;
      for (int i = d.n_red - 1; i >= 0; --i) {
        off += (rr % d.red_size[i]) * d.red_stride[i];
        rr /= d.red_size[i];
      }
      arg_take(bv, bi, x[off], r);
    }
    for (int s = 16; s > 0; s >>= 1)
      arg_take(bv, bi, __shfl_xor_sync(0xffffffffu, bv, s), __shfl_xor_sync(0xffffffffu, bi, s));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    if (lane == 0) {
      sv[warp] = bv;
      si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
      bv = lane < warps ? sv[lane] : sv[0];
      bi = lane < warps ? si[lane] : si[0];
      for (int s = 16; s > 0; s >>= 1)
        arg_take(bv, bi, __shfl_xor_sync(0xffffffffu, bv, s),
                 __shfl_xor_sync(0xffffffffu, bi, s));
      if (lane == 0) out[o] = bi;
    }
    __syncthreads();
  }
}

// Keep-axis bookkeeping shared by the reductions of this file.
ReduceDims reduce_dims(int ndim, const int64_t* in_shape, const int* keep) {
  ReduceDims d{};
  int64_t stride = 1;
  int64_t strides[kMaxDims];
  for (int i = ndim - 1; i >= 0; --i) {
    strides[i] = stride;
    stride *= in_shape[i];
  }
  d.out_count = 1;
  d.red_count = 1;
  for (int i = 0; i < ndim; ++i) {
    if (keep[i]) {
      d.keep_size[d.n_keep] = in_shape[i];
      d.keep_stride[d.n_keep++] = strides[i];
      d.out_count *= in_shape[i];
    } else {
      d.red_size[d.n_red] = in_shape[i];
      d.red_stride[d.n_red++] = strides[i];
      d.red_count *= in_shape[i];
    }
  }
  return d;
}

unsigned reduce_grid(const ReduceDims& d) {
  return (unsigned)(d.out_count < 148 * 16 ? d.out_count : 148 * 16);
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int tg_where(int dtype, int cond_dtype, int ndim, const int64_t* shape, const void* cond,
             const int64_t* cond_strides, const void* a, const int64_t* a_strides,
             const void* b, const int64_t* b_strides, void* out, void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "where: ndim %d out of range", ndim);
  TG_CHECK_ARG(cond_dtype >= -1 && cond_dtype <= TG_I64, "where: bad condition dtype %d",
               cond_dtype);
  SelectDims d{};
  d.ndim = ndim;
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    d.shape[i] = shape[i];
    d.sc[i] = cond_strides[i];
    d.sa[i] = a_strides[i];
    d.sb[i] = b_strides[i];
    n *= shape[i];
  }
  if (n == 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const unsigned grid = grid_for(n, 256);
    cudaStream_t st = as_stream(stream);
    switch (cond_dtype) {
      case TG_F32:
        where_kernel<T, float><<<grid, 256, 0, st>>>((const float*)cond, (const T*)a,
                                                     (const T*)b, (T*)out, n, d);
        break;
      case TG_F64:
        where_kernel<T, double><<<grid, 256, 0, st>>>((const double*)cond, (const T*)a,
                                                      (const T*)b, (T*)out, n, d);
        break;
      case TG_I64:
        where_kernel<T, int64_t><<<grid, 256, 0, st>>>((const int64_t*)cond, (const T*)a,
                                                       (const T*)b, (T*)out, n, d);
        break;
      default:
        where_kernel<T, uint8_t><<<grid, 256, 0, st>>>((const uint8_t*)cond, (const T*)a,
                                                       (const T*)b, (T*)out, n, d);
    }
    return check_launch("where");
  });
}

int tg_compare(int dtype, int op, int ndim, const int64_t* shape, const void* a,
               const int64_t* a_strides, const void* b, const int64_t* b_strides, uint8_t* out,
               void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "compare: ndim %d out of range", ndim);
  TG_CHECK_ARG(op >= 0 && op <= 5, "compare: bad op %d", op);
  SelectDims d{};
  d.ndim = ndim;
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    d.shape[i] = shape[i];
    d.sa[i] = a_strides[i];
    d.sb[i] = b_strides[i];
    n *= shape[i];
  }
  if (n == 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    compare_kernel<T><<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
        op, (const T*)a, (const T*)b, out, n, d);
    return check_launch("compare");
  });
}

int tg_reduce_extremum(int dtype, int is_min, int ndim, const int64_t* in_shape,
                       const int* keep, const void* x, void* out, void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "max/min: ndim %d out of range", ndim);
  const ReduceDims d = reduce_dims(ndim, in_shape, keep);
  if (d.out_count == 0) return TG_OK;
  TG_CHECK_ARG(d.red_count > 0, "max/min: zero-size reduction has no identity");
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    extremum_keep_kernel<T><<<reduce_grid(d), 256, 0, as_stream(stream)>>>(
        (const T*)x, (T*)out, d, is_min != 0);
    return check_launch(is_min ? "min" : "max");
  });
}

int tg_reduce_truth(int in_dtype, int is_all, int ndim, const int64_t* in_shape,
                    const int* keep, const void* x, uint8_t* out, void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "all/any: ndim %d out of range", ndim);
  TG_CHECK_ARG(in_dtype >= -1 && in_dtype <= TG_I64, "all/any: bad dtype %d", in_dtype);
  const ReduceDims d = reduce_dims(ndim, in_shape, keep);
  if (d.out_count == 0) return TG_OK;
  cudaStream_t st = as_stream(stream);
  const unsigned grid = reduce_grid(d);
  const bool all = is_all != 0;
  switch (in_dtype) {
    case TG_F32: truth_keep_kernel<float><<<grid, 256, 0, st>>>((const float*)x, out, d, all); break;
    case TG_F64: truth_keep_kernel<double><<<grid, 256, 0, st>>>((const double*)x, out, d, all); break;
    case TG_I64: truth_keep_kernel<int64_t><<<grid, 256, 0, st>>>((const int64_t*)x, out, d, all); break;
    default: truth_keep_kernel<uint8_t><<<grid, 256, 0, st>>>((const uint8_t*)x, out, d, all);
  }
  return check_launch(all ? "all" : "any");
}

int tg_argmax(int dtype, int ndim, const int64_t* in_shape, const int* keep, const void* x,
              int64_t* out, void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "argmax: ndim %d out of range", ndim);
  const ReduceDims d = reduce_dims(ndim, in_shape, keep);
  if (d.out_count == 0) return TG_OK;
  TG_CHECK_ARG(d.red_count > 0, "argmax: attempt to get argmax of an empty sequence");
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    argmax_keep_kernel<T><<<reduce_grid(d), 256, 0, as_stream(stream)>>>((const T*)x, out, d);
    return check_launch("argmax");
  });
}

}  // extern "C"
