// Gradient-norm clipping and the Adam/AdamW update (optim/clip.py:15-31, optim/adam.py:59-94).
//
// Multi-tensor launches carry up to kMaxTensors (pointer, size) pairs in the kernel parameter
// block, so one launch covers a whole parameter group without uploading a pointer table.
// The squared norm is accumulated in float64 per thread in a fixed element order, reduced per
// block, and the block partials are summed in order (deterministic).
#include "common.cuh"

namespace tg {
namespace {

constexpr int kMaxTensors = 64;
constexpr int kNormBlocks = 148 * 8;

struct TensorList {
  int count;
  void* ptr[kMaxTensors];
  int64_t numel[kMaxTensors];
};

struct AdamList {
  int count;
  void* p[kMaxTensors];
  const void* g[kMaxTensors];
  void* m[kMaxTensors];
  void* v[kMaxTensors];
  int64_t numel[kMaxTensors];
  double step_size[kMaxTensors];  // lr / (1 - beta1^step)
  double bc2_sqrt[kMaxTensors];   // sqrt(1 - beta2^step)
};

// Sum of squares in float64. fp32 tensors with 16-byte aligned storage are read as float4
// with four independent accumulators (the scalar tail after them); other tensors element by
// element. The element-to-thread map and the reduction order are fixed (deterministic).
template <typename T>
__global__ void __launch_bounds__(256) sumsq_kernel(TensorList L, double* __restrict__ partial) {
  __shared__ double sh[32];
  double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int t = 0; t < L.count; ++t) {
    const T* x = reinterpret_cast<const T*>(L.ptr[t]);
    int64_t done = 0;
    if (sizeof(T) == 4 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
      const int64_t n4 = L.numel[t] >> 2;
      const float4* x4 = reinterpret_cast<const float4*>(x);
      for (int64_t i = tid; i < n4; i += stride) {
        const float4 v = x4[i];
        a0 += (double)v.x * (double)v.x;
        a1 += (double)v.y * (double)v.y;
        a2 += (double)v.z * (double)v.z;
        a3 += (double)v.w * (double)v.w;
      }
      done = n4 << 2;
    }
    for (int64_t i = done + tid; i < L.numel[t]; i += stride) {
      const double v = (double)x[i];
      a0 += v * v;
    }
  }
  double acc = (a0 + a1) + (a2 + a3);
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

__global__ void norm_final_kernel(const double* __restrict__ partial, int n, double* total) {
  __shared__ double sh[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) total[0] = sqrt(acc);
}

template <typename T>
__global__ void clip_kernel(TensorList L, const double* __restrict__ total, double max_norm,
                            double eps) {
  const double scale = max_norm / (total[0] + eps);
  if (!(scale < 1.0)) return;
  const T f = (T)scale;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int t = 0; t < L.count; ++t) {
    T* x = reinterpret_cast<T*>(L.ptr[t]);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < L.numel[t]; i += stride)
      x[i] = x[i] * f;
  }
}

template <typename T>
__device__ __forceinline__ void adam_elem(T& p, T g, T& m, T& v, T decay, T l2, T b1, T omb1,
                                          T b2, T omb2, T step_size, T bc2_sqrt, T eps) {
  p = p * decay;
  g = g + l2 * p;
  m = m * b1 + omb1 * g;
  v = v * b2 + (omb2 * g) * g;
  const T denom = dev_sqrt<T>(v) / bc2_sqrt + eps;
  p = p - step_size * m / denom;
}

// The factor clip_grad_norm_ applies to every gradient, decided on the device from the total
// norm: (T)(max_norm / (total + eps)) when that is below 1, else no rescale (clip_kernel's
// rule, so a gradient scaled here equals the one clip_kernel would have written).
struct ClipFactor {
  const double* total;  // nullptr: no clip pending
  double max_norm, eps;
};

template <typename T>
__device__ __forceinline__ bool clip_factor(const ClipFactor& c, T& f) {
  if (c.total == nullptr) return false;
  const double scale = c.max_norm / (c.total[0] + c.eps);
  f = (T)scale;
  return scale < 1.0;
}

template <typename T>
__global__ void __launch_bounds__(256)
adam_multi_kernel(AdamList L, T b1, T b2, T eps, T decay, T l2, ClipFactor clip = {}) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const T omb1 = T(1) - b1, omb2 = T(1) - b2;
  T cf = T(1);
  const bool scaled = clip_factor<T>(clip, cf);
  for (int t = 0; t < L.count; ++t) {
    T* p = reinterpret_cast<T*>(L.p[t]);
    const T* g = reinterpret_cast<const T*>(L.g[t]);
    T* m = reinterpret_cast<T*>(L.m[t]);
    T* v = reinterpret_cast<T*>(L.v[t]);
    const T ss = (T)L.step_size[t], bs = (T)L.bc2_sqrt[t];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < L.numel[t]; i += stride) {
      T pi = p[i], mi = m[i], vi = v[i];
      const T gi = scaled ? g[i] * cf : g[i];
      adam_elem<T>(pi, gi, mi, vi, decay, l2, b1, omb1, b2, omb2, ss, bs, eps);
      p[i] = pi;
      m[i] = mi;
      v[i] = vi;
    }
  }
}

// Flat fp32 range with 16-byte vectors. With a clip pending (clip.total set), the gradient
// is read rescaled and the update is the whole of clip_grad_norm_'s rewrite plus AdamW in
// one pass: 28 bytes per parameter instead of 8 + 28.
__global__ void __launch_bounds__(256)
adam_flat_vec4_kernel(int64_t n4, float4* __restrict__ p, const float4* __restrict__ g,
                      float4* __restrict__ m, float4* __restrict__ v, float b1, float b2,
                      float eps, float decay, float l2, float ss, float bs, ClipFactor clip) {
  const float omb1 = 1.f - b1, omb2 = 1.f - b2;
  float cf = 1.f;
  const bool scaled = clip_factor<float>(clip, cf);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 P = p[i], G = g[i], M = m[i], V = v[i];
    if (scaled) G = make_float4(G.x * cf, G.y * cf, G.z * cf, G.w * cf);
    adam_elem<float>(P.x, G.x, M.x, V.x, decay, l2, b1, omb1, b2, omb2, ss, bs, eps);
    adam_elem<float>(P.y, G.y, M.y, V.y, decay, l2, b1, omb1, b2, omb2, ss, bs, eps);
    adam_elem<float>(P.z, G.z, M.z, V.z, decay, l2, b1, omb1, b2, omb2, ss, bs, eps);
    adam_elem<float>(P.w, G.w, M.w, V.w, decay, l2, b1, omb1, b2, omb2, ss, bs, eps);
    p[i] = P; m[i] = M; v[i] = V;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

size_t tg_sumsq_scratch_bytes(int count) {
  const int launches = (count + kMaxTensors - 1) / kMaxTensors;
  return (size_t)(launches > 0 ? launches : 1) * kNormBlocks * sizeof(double);
}

int tg_sumsq_multi(int dtype, int count, void* const* ptrs, const int64_t* numels,
                   double* total_dev, void* scratch, void* stream) {
  TG_CHECK_ARG(count >= 0 && scratch && total_dev, "sumsq_multi: bad arguments");
  cudaStream_t s = as_stream(stream);
  double* partial = reinterpret_cast<double*>(scratch);
  int launches = 0;
  int rc = TG_DISPATCH_FLOAT(dtype, T, [&] {
    for (int base = 0; base < count || (count == 0 && launches == 0); base += kMaxTensors) {
      TensorList L{};
      L.count = count - base < kMaxTensors ? count - base : kMaxTensors;
      if (L.count < 0) L.count = 0;
      for (int i = 0; i < L.count; ++i) {
        L.ptr[i] = ptrs[base + i];
        L.numel[i] = numels[base + i];
      }
      sumsq_kernel<T><<<kNormBlocks, 256, 0, s>>>(L, partial + (size_t)launches * kNormBlocks);
      ++launches;
      if (count == 0) break;
    }
    return check_launch("sumsq_multi", launches);
  });
  if (rc != TG_OK) return rc;
  norm_final_kernel<<<1, 256, 0, s>>>(partial, launches * kNormBlocks, total_dev);
  return check_launch("sumsq_multi(final)");
}

int tg_clip_scale_multi(int dtype, int count, void* const* ptrs, const int64_t* numels,
                        const double* total_dev, double max_norm, double eps, void* scratch,
                        void* stream) {
  (void)scratch;
  cudaStream_t s = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    for (int base = 0; base < count; base += kMaxTensors) {
      TensorList L{};
      L.count = count - base < kMaxTensors ? count - base : kMaxTensors;
      for (int i = 0; i < L.count; ++i) {
        L.ptr[i] = ptrs[base + i];
        L.numel[i] = numels[base + i];
      }
      clip_kernel<T><<<2 * 148 * 4, 256, 0, s>>>(L, total_dev, max_norm, eps);
    }
    return check_launch("clip_scale_multi", (count + kMaxTensors - 1) / kMaxTensors);
  });
}

int tg_adam_update_clipped(int dtype, int64_t n, void* p, const void* g, void* m, void* v,
                           double lr, double beta1, double beta2, double eps,
                           double weight_decay, int64_t step, int decoupled,
                           const double* clip_total_dev, double max_norm, double clip_eps,
                           void* stream);

int tg_adam_update(int dtype, int64_t n, void* p, const void* g, void* m, void* v, double lr,
                   double beta1, double beta2, double eps, double weight_decay, int64_t step,
                   int decoupled, void* stream) {
  return tg_adam_update_clipped(dtype, n, p, g, m, v, lr, beta1, beta2, eps, weight_decay, step,
                                decoupled, nullptr, 0.0, 0.0, stream);
}

int tg_adam_update_clipped(int dtype, int64_t n, void* p, const void* g, void* m, void* v,
                           double lr, double beta1, double beta2, double eps,
                           double weight_decay, int64_t step, int decoupled,
                           const double* clip_total_dev, double max_norm, double clip_eps,
                           void* stream) {
  TG_CHECK_ARG(step >= 1, "adam_update: step must be >= 1");
  const ClipFactor clip{clip_total_dev, max_norm, clip_eps};
  if (n <= 0) return TG_OK;
  cudaStream_t s = as_stream(stream);
  const double ss = lr / (1.0 - pow(beta1, (double)step));
  const double bs = sqrt(1.0 - pow(beta2, (double)step));
  const double decay = (weight_decay != 0.0 && decoupled) ? 1.0 - lr * weight_decay : 1.0;
  const double l2 = (weight_decay != 0.0 && !decoupled) ? weight_decay : 0.0;
  if (dtype == TG_F32 && n % 4 == 0 && aligned16(p) && aligned16(g) && aligned16(m) &&
      aligned16(v)) {
    adam_flat_vec4_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(
        n / 4, (float4*)p, (const float4*)g, (float4*)m, (float4*)v, (float)beta1,
        (float)beta2, (float)eps, (float)decay, (float)l2, (float)ss, (float)bs, clip);
    return check_launch("adam_update");
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    AdamList L{};
    L.count = 1;
    L.p[0] = p; L.g[0] = g; L.m[0] = m; L.v[0] = v; L.numel[0] = n;
    L.step_size[0] = ss; L.bc2_sqrt[0] = bs;
    adam_multi_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(L, (T)beta1, (T)beta2, (T)eps,
                                                          (T)decay, (T)l2, clip);
    return check_launch("adam_update");
  });
}

size_t tg_adam_multi_scratch_bytes(int count) {
  (void)count;
  return 0;
}

int tg_adam_update_multi(int dtype, int count, void* const* p, void* const* g, void* const* m,
                         void* const* v, const int64_t* numels, const int64_t* steps, double lr,
                         double beta1, double beta2, double eps, double weight_decay,
                         int decoupled, void* scratch, void* stream) {
  (void)scratch;
  cudaStream_t s = as_stream(stream);
  const double decay = (weight_decay != 0.0 && decoupled) ? 1.0 - lr * weight_decay : 1.0;
  const double l2 = (weight_decay != 0.0 && !decoupled) ? weight_decay : 0.0;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    for (int base = 0; base < count; base += kMaxTensors) {
      AdamList L{};
      L.count = count - base < kMaxTensors ? count - base : kMaxTensors;
      int64_t total = 0;
      for (int i = 0; i < L.count; ++i) {
        const int k = base + i;
        if (steps[k] < 1) return set_error(TG_ERR_ARG, "adam_update_multi: step must be >= 1");
        L.p[i] = p[k]; L.g[i] = g[k]; L.m[i] = m[k]; L.v[i] = v[k];
        L.numel[i] = numels[k];
        L.step_size[i] = lr / (1.0 - pow(beta1, (double)steps[k]));
        L.bc2_sqrt[i] = sqrt(1.0 - pow(beta2, (double)steps[k]));
        total += numels[k];
      }
      adam_multi_kernel<T><<<grid_for(total, 256), 256, 0, s>>>(L, (T)beta1, (T)beta2, (T)eps,
                                                                (T)decay, (T)l2);
    }
    return check_launch("adam_update_multi", (count + kMaxTensors - 1) / kMaxTensors);
  });
}

}  // extern "C"
