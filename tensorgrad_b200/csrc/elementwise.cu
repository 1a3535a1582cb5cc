// Elementwise kernels: broadcast binary arithmetic, unary functions and their VJPs, GELU
// (tanh approximation) and ReLU. All are HBM-bound grid-stride loops; contiguous operands
// take a 16-byte vectorised path.
#include "common.cuh"
#include "reduce.cuh"

namespace tg {
namespace {

struct BcastDims {
  int ndim;
  int64_t shape[kMaxDims];
  int64_t sa[kMaxDims], sb[kMaxDims];
};

template <typename T>
__device__ __forceinline__ T apply_binary(int op, T x, T y) {
  switch (op) {
    case TG_ADD: return x + y;
    case TG_SUB: return x - y;
    case TG_MUL: return x * y;
    case TG_DIV: return x / y;
    case TG_EQ: return x == y ? T(1) : T(0);
    default: return pow(x, y);
  }
}

template <typename T, int OP>
__global__ void binary_contig_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                     T* __restrict__ out, int64_t n, int64_t a_mod,
                                     int64_t b_mod) {
  // a_mod / b_mod: the operand repeats every *_mod elements (1 = scalar, n = full).
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const T x = a_mod == n ? a[i] : a[i % a_mod];
    const T y = b_mod == n ? b[i] : b[i % b_mod];
    out[i] = apply_binary<T>(OP, x, y);
  }
}

template <typename T>
__global__ void binary_add_vec4_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                       float4* __restrict__ out, int64_t n4) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 x = a[i], y = b[i];
    out[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
  }
}

template <typename T>
__global__ void binary_strided_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                                      T* __restrict__ out, int64_t n, BcastDims d) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, oa = 0, ob = 0;
    for (int k = d.ndim - 1; k >= 0; --k) {
      const int64_t idx = rem % d.shape[k];
      rem /= d.shape[k];
      oa += idx * d.sa[k];
      ob += idx * d.sb[k];
    }
    out[i] = apply_binary<T>(op, a[oa], b[ob]);
  }
}

template <typename T>
__global__ void axpby_kernel(int64_t n, T alpha, const T* __restrict__ x, T beta,
                             const T* __restrict__ y, T* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    T v = alpha * x[i];
    if (y) v += beta * y[i];
    out[i] = v;
  }
}

template <typename T>
__global__ void scale_dev_kernel(int64_t n, const T* __restrict__ x, const T* __restrict__ s,
                                 T alpha, T* __restrict__ out) {
  const T f = alpha * s[0];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = x[i] * f;
}

template <typename T>
__device__ __forceinline__ T apply_unary(int op, T x, T a) {
  switch (op) {
    case TG_NEG: return -x;
    case TG_EXP: return dev_exp<T>(x);
    case TG_LOG: return dev_log<T>(x);
    case TG_SQRT: return dev_sqrt<T>(x);
    case TG_TANH: return dev_tanh<T>(x);
    case TG_SIGMOID: {
      // Overflow-free logistic: exp of a non-positive argument only.
      const T e = dev_exp<T>(-fabs(x));
      return x >= T(0) ? T(1) / (T(1) + e) : e / (T(1) + e);
    }
    case TG_RELU: return x > T(0) ? x : T(0);
    case TG_SQUARE: return x * x;
    case TG_FILL: return a;
    case TG_ABS: return fabs(x);
    case TG_FINITE_OR_ZERO: return isfinite(x) ? x : T(0);
    case TG_LOG1P: return log1p(x);
    case TG_POWS: return pow(x, a);
    default: return pow(x, a);
  }
}

template <typename T>
__global__ void unary_kernel(int op, int64_t n, const T* __restrict__ x, T alpha,
                             T* __restrict__ out) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = apply_unary<T>(op, op == TG_FILL ? T(0) : x[i], alpha);
}

template <typename T>
__global__ void unary_backward_kernel(int op, int64_t n, const T* __restrict__ g,
                                      const T* __restrict__ x, const T* __restrict__ y, T a,
                                      T* __restrict__ gx) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const T gi = g[i];
    T r;
    switch (op) {
      case TG_EXP: r = gi * y[i]; break;
      case TG_LOG: r = gi / x[i]; break;
      case TG_SQRT: r = gi / (T(2) * y[i]); break;
      case TG_TANH: r = gi * (T(1) - y[i] * y[i]); break;
      case TG_SIGMOID: r = gi * y[i] * (T(1) - y[i]); break;
      case TG_NEG: r = -gi; break;
      default: r = gi * a * pow(x[i], a - T(1)); break;
    }
    gx[i] = r;
  }
}

// GELU(x) = 0.5 x (1 + tanh(c (x + a x^3))), c = sqrt(2/pi), a = 0.044715.
template <typename T>
__device__ __forceinline__ T gelu_t(T x) {
  const T c = T(0.7978845608028654), a = T(0.044715);
  return dev_tanh<T>(c * x * (T(1) + a * x * x));
}

template <typename T>
__global__ void gelu_fwd_kernel(int64_t n, const T* __restrict__ x, T* __restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const T v = x[i];
    y[i] = T(0.5) * v * (T(1) + gelu_t(v));
  }
}

__global__ void gelu_fwd_vec4_kernel(int64_t n4, const float4* __restrict__ x,
                                     float4* __restrict__ y) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = x[i];
    v.x = 0.5f * v.x * (1.f + gelu_t(v.x));
    v.y = 0.5f * v.y * (1.f + gelu_t(v.y));
    v.z = 0.5f * v.z * (1.f + gelu_t(v.z));
    v.w = 0.5f * v.w * (1.f + gelu_t(v.w));
    y[i] = v;
  }
}

// d/dx = 0.5 (1 + t) + 0.5 x (1 - t^2) c (1 + 3 a x^2)  (ops/elementwise.py:297-312).
template <typename T>
__device__ __forceinline__ T gelu_grad(T x) {
  const T c = T(0.7978845608028654), a = T(0.044715);
  const T t = gelu_t(x);
  const T d = c + T(3) * a * c * x * x;
  return T(0.5) * ((T(1) - t * t) * d * x + t + T(1));
}

template <typename T>
__global__ void gelu_bwd_kernel(int64_t n, const T* __restrict__ g, const T* __restrict__ x,
                                T* __restrict__ gx) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    gx[i] = gelu_grad(x[i]) * g[i];
}

__global__ void gelu_bwd_vec4_kernel(int64_t n4, const float4* __restrict__ g,
                                     const float4* __restrict__ x, float4* __restrict__ gx) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = x[i], w = g[i];
    gx[i] = make_float4(gelu_grad(v.x) * w.x, gelu_grad(v.y) * w.y, gelu_grad(v.z) * w.z,
                        gelu_grad(v.w) * w.w);
  }
}

template <typename T>
__global__ void relu_bwd_kernel(int64_t n, const T* __restrict__ g, const T* __restrict__ x,
                                T* __restrict__ gx) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    gx[i] = x[i] > T(0) ? g[i] : T(0);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int tg_binary(int dtype, int op, int ndim, const int64_t* shape, const void* a,
              const int64_t* a_strides, const void* b, const int64_t* b_strides, void* out,
              void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "binary: ndim %d out of range", ndim);
  TG_CHECK_ARG(op >= TG_ADD && op <= TG_EQ, "binary: bad op %d", op);
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= shape[i];
  if (n == 0) return TG_OK;
  // An operand is "simple" when its value at flat output index i is x[i % mod]: contiguous
  // over a suffix of the axes and broadcast (stride 0) over the rest. mod = n is a full
  // operand, mod = 1 a scalar.
  auto classify = [&](const int64_t* st, int64_t* mod) -> bool {
    int64_t expect = 1;
    int k = ndim - 1;
    for (; k >= 0; --k) {
      if (shape[k] == 1) continue;
      if (st[k] != expect) break;
      expect *= shape[k];
    }
    for (int j = k; j >= 0; --j)
      if (shape[j] != 1 && st[j] != 0) return false;
    *mod = expect;
    return true;
  };
  int64_t am = 0, bm = 0;
  const bool simple = classify(a_strides, &am) && classify(b_strides, &bm);
  cudaStream_t s = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const unsigned grid = grid_for(n, 256);
    if (simple && am == n && bm == n && op == TG_ADD && sizeof(T) == 4 && n % 4 == 0 &&
        aligned16(a) && aligned16(b) && aligned16(out)) {
      launch_pdl(binary_add_vec4_kernel<T>, dim3(grid_for(n / 4, 256)), dim3(256), 0, s,
          (const float4*)a, (const float4*)b, (float4*)out, n / 4);
    } else if (simple) {
      switch (op) {
        case TG_ADD: binary_contig_kernel<T, TG_ADD><<<grid, 256, 0, s>>>((const T*)a, (const T*)b, (T*)out, n, am, bm); break;
        case TG_SUB: binary_contig_kernel<T, TG_SUB><<<grid, 256, 0, s>>>((const T*)a, (const T*)b, (T*)out, n, am, bm); break;
        case TG_MUL: binary_contig_kernel<T, TG_MUL><<<grid, 256, 0, s>>>((const T*)a, (const T*)b, (T*)out, n, am, bm); break;
        case TG_DIV: binary_contig_kernel<T, TG_DIV><<<grid, 256, 0, s>>>((const T*)a, (const T*)b, (T*)out, n, am, bm); break;
        case TG_EQ: binary_contig_kernel<T, TG_EQ><<<grid, 256, 0, s>>>((const T*)a, (const T*)b, (T*)out, n, am, bm); break;
        default: binary_contig_kernel<T, TG_POW><<<grid, 256, 0, s>>>((const T*)a, (const T*)b, (T*)out, n, am, bm); break;
      }
    } else {
      BcastDims d{};
      d.ndim = ndim;
      for (int i = 0; i < ndim; ++i) {
        d.shape[i] = shape[i];
        d.sa[i] = a_strides[i];
        d.sb[i] = b_strides[i];
      }
      binary_strided_kernel<T><<<grid, 256, 0, s>>>(op, (const T*)a, (const T*)b, (T*)out, n, d);
    }
    return check_launch("binary");
  });
}

int tg_axpby(int dtype, int64_t n, double alpha, const void* x, double beta, const void* y,
             void* out, void* stream) {
  if (n <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    axpby_kernel<T><<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
        n, (T)alpha, (const T*)x, (T)beta, beta == 0.0 ? nullptr : (const T*)y, (T*)out);
    return check_launch("axpby");
  });
}

int tg_scale_by_device_scalar(int dtype, int64_t n, const void* x, const void* scale_dev,
                              double alpha, void* out, void* stream) {
  if (n <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    scale_dev_kernel<T><<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
        n, (const T*)x, (const T*)scale_dev, (T)alpha, (T*)out);
    return check_launch("scale_by_device_scalar");
  });
}

int tg_unary(int dtype, int op, int64_t n, const void* x, double alpha, void* out, void* stream) {
  TG_CHECK_ARG(op >= TG_NEG && op <= TG_LOG1P, "unary: bad op %d", op);
  if (n <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    launch_pdl(unary_kernel<T>, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream),
               op, n, (const T*)x, (T)alpha, (T*)out);
    return check_launch("unary");
  });
}

int tg_unary_backward(int dtype, int op, int64_t n, const void* g, const void* x, const void* y,
                      double alpha, void* gx, void* stream) {
  if (n <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    unary_backward_kernel<T><<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
        op, n, (const T*)g, (const T*)x, (const T*)y, (T)alpha, (T*)gx);
    return check_launch("unary_backward");
  });
}

int tg_gelu_forward(int dtype, int64_t n, const void* x, void* y, void* stream) {
  if (n <= 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == TG_F32 && n % 4 == 0 && aligned16(x) && aligned16(y)) {
    launch_pdl(gelu_fwd_vec4_kernel, dim3(grid_for(n / 4, 256)), dim3(256), 0, s,
               n / 4, (const float4*)x,
                                                               (float4*)y);
    return check_launch("gelu_forward");
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    gelu_fwd_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(n, (const T*)x, (T*)y);
    return check_launch("gelu_forward");
  });
}

int tg_gelu_backward(int dtype, int64_t n, const void* g, const void* x, void* gx, void* stream) {
  if (n <= 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == TG_F32 && n % 4 == 0 && aligned16(x) && aligned16(g) && aligned16(gx)) {
    launch_pdl(gelu_bwd_vec4_kernel, dim3(grid_for(n / 4, 256)), dim3(256), 0, s,
               n / 4, (const float4*)g,
                                                               (const float4*)x, (float4*)gx);
    return check_launch("gelu_backward");
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    gelu_bwd_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(n, (const T*)g, (const T*)x, (T*)gx);
    return check_launch("gelu_backward");
  });
}

int tg_relu_backward(int dtype, int64_t n, const void* g, const void* x, void* gx, void* stream) {
  if (n <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    launch_pdl(relu_bwd_kernel<T>, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream),
               n, (const T*)g, (const T*)x, (T*)gx);
    return check_launch("relu_backward");
  });
}

}  // extern "C"

// ---------------------------------------------------------------- casts and strided copies
namespace tg {
namespace {

template <typename S, typename D>
__global__ void cast_kernel(int64_t n, const S* __restrict__ src, D* __restrict__ dst) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = (D)src[i];
}

template <typename S>
int cast_from(int dst_dtype, int64_t n, const S* src, void* dst, cudaStream_t s) {
  const unsigned g = grid_for(n, 256);
  switch (dst_dtype) {
    case TG_F32: cast_kernel<S, float><<<g, 256, 0, s>>>(n, src, (float*)dst); break;
    case TG_F64: cast_kernel<S, double><<<g, 256, 0, s>>>(n, src, (double*)dst); break;
    case TG_I64: cast_kernel<S, long long><<<g, 256, 0, s>>>(n, src, (long long*)dst); break;
    default: return set_error(TG_ERR_ARG, "cast: bad destination dtype %d", dst_dtype);
  }
  return check_launch("cast");
}

struct CopyDims {
  int ndim;
  int64_t shape[kMaxDims], ss[kMaxDims], ds[kMaxDims];
};

template <typename E>
__global__ void strided_copy_kernel(const E* __restrict__ src, E* __restrict__ dst, int64_t n,
                                    CopyDims d) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, os = 0, od = 0;
    for (int k = d.ndim - 1; k >= 0; --k) {
      const int64_t idx = rem % d.shape[k];
      rem /= d.shape[k];
      os += idx * d.ss[k];
      od += idx * d.ds[k];
    }
    dst[od] = src[os];
  }
}

}  // namespace
}  // namespace tg

extern "C" {

int tg_cast(int src_dtype, int dst_dtype, int64_t n, const void* src, void* dst, void* stream) {
  if (n <= 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  switch (src_dtype) {
    case TG_F32: return cast_from<float>(dst_dtype, n, (const float*)src, dst, s);
    case TG_F64: return cast_from<double>(dst_dtype, n, (const double*)src, dst, s);
    case TG_I64: return cast_from<long long>(dst_dtype, n, (const long long*)src, dst, s);
  }
  return set_error(TG_ERR_ARG, "cast: bad source dtype %d", src_dtype);
}

int tg_strided_copy(int elem_bytes, int ndim, const int64_t* shape, const void* src,
                    const int64_t* src_strides, void* dst, const int64_t* dst_strides,
                    void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "strided_copy: ndim %d out of range", ndim);
  CopyDims d{};
  d.ndim = ndim;
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    d.shape[i] = shape[i];
    d.ss[i] = src_strides[i];
    d.ds[i] = dst_strides[i];
    n *= shape[i];
  }
  if (n == 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  const unsigned g = grid_for(n, 256);
  switch (elem_bytes) {
    case 1: strided_copy_kernel<uint8_t><<<g, 256, 0, s>>>((const uint8_t*)src, (uint8_t*)dst, n, d); break;
    case 4: strided_copy_kernel<uint32_t><<<g, 256, 0, s>>>((const uint32_t*)src, (uint32_t*)dst, n, d); break;
    case 8: strided_copy_kernel<uint64_t><<<g, 256, 0, s>>>((const uint64_t*)src, (uint64_t*)dst, n, d); break;
    default: return set_error(TG_ERR_ARG, "strided_copy: element size %d", elem_bytes);
  }
  return check_launch("strided_copy");
}

}  // extern "C"
