// Embedding gather / scatter-add (ops/layers.py:192-232) and softmax cross-entropy with the
// class axis last (ops/loss.py:23-97, ops/activation.py:48-52).
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"

namespace tg {
namespace {

// ---------------------------------------------------------------- embedding
// Ids outside [0, num) give a zero row and set *bad (when given): device-resident ids are
// validated where they are read, the flag is read back at the next host synchronisation.
template <typename T>
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ w,
                                 T* __restrict__ out, int64_t n, int64_t num, int64_t dim,
                                 int* __restrict__ bad) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t id = ids[r];
    const bool ok = id >= 0 && id < num;
    if (!ok && bad && threadIdx.x == 0) atomicOr(bad, 1);
    const T* src = w + (ok ? id : 0) * dim;
    T* dst = out + r * dim;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) dst[c] = ok ? src[c] : T(0);
  }
}

__global__ void embed_fwd_vec4_kernel(const int64_t* __restrict__ ids, const float4* __restrict__ w,
                                      float4* __restrict__ out, int64_t n, int64_t num,
                                      int64_t dim4, int* __restrict__ bad) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t id = ids[r];
    const bool ok = id >= 0 && id < num;
    if (!ok && bad && threadIdx.x == 0) atomicOr(bad, 1);
    const float4* src = w + (ok ? id : 0) * dim4;
    float4* dst = out + r * dim4;
    for (int64_t c = threadIdx.x; c < dim4; c += blockDim.x)
      dst[c] = ok ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
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

// Sort keys id * n + position (ids clamped into [0, num), an out-of-range id flagged in *bad).
// The keys are unique, so their ascending order is the stable sort by id that the reference
// takes, whatever algorithm sorts them.
__global__ void embed_keys_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t num,
                                  uint64_t* __restrict__ keys, int* __restrict__ bad) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t id = ids[i];
    if (id < 0 || id >= num) {
      if (bad) atomicOr(bad, 1);
      id = 0;
    }
    keys[i] = (uint64_t)id * (uint64_t)n + (uint64_t)i;
  }
}

// The VJP from sorted keys: one warp per sorted position; the warp at the first position of a
// run of equal ids sums that run's gradient rows in ascending position and writes (or adds)
// the id's row. Other warps return at once.
template <typename T>
__global__ void embed_bwd_sorted_kernel(const T* __restrict__ g, const uint64_t* __restrict__ keys,
                                        int64_t n, T* __restrict__ gw, int64_t dim,
                                        int accumulate) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const uint64_t un = (uint64_t)n;
  for (int64_t k = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); k < n;
       k += warps) {
    const uint64_t id = keys[k] / un;
    if (k > 0 && keys[k - 1] / un == id) continue;
    // Run end: the first later key of another id, 32 keys at a time.
    const uint64_t limit = (id + 1) * un;  // keys of this id are below it
    int64_t e = k + 1;
    while (true) {
      const int64_t i = e + lane;
      const bool same = i < n && keys[i] < limit;
      const unsigned m = __ballot_sync(0xffffffffu, same);
      if (m != 0xffffffffu) {
        e += __ffs(~m) - 1;
        break;
      }
      e += 32;
    }
    const uint64_t base = id * un;
    T* dst = gw + (int64_t)id * dim;
    for (int64_t c = lane; c < dim; c += 32) {
      T acc = T(0);
#pragma unroll 4
      for (int64_t i = k; i < e; ++i) acc += g[(int64_t)(keys[i] - base) * dim + c];
      dst[c] = accumulate ? dst[c] + acc : acc;
    }
  }
}

int key_bits(uint64_t max_key) {
  int b = 1;
  while (b < 64 && (max_key >> b)) ++b;
  return b;
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
                         int64_t num, int64_t dim, int* bad_id_dev, void* stream) {
  if (n <= 0 || dim <= 0) return TG_OK;
  TG_CHECK_ARG(num > 0, "embedding: empty table");
  cudaStream_t s = as_stream(stream);
  const unsigned grid = (unsigned)(n < 148 * 16 ? n : 148 * 16);
  if (dtype == TG_F32 && dim % 4 == 0 && aligned16(w) && aligned16(out)) {
    embed_fwd_vec4_kernel<<<grid, 128, 0, s>>>(ids, (const float4*)w, (float4*)out, n, num,
                                               dim / 4, bad_id_dev);
    return check_launch("embedding_forward");
  }
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    embed_fwd_kernel<T><<<grid, 128, 0, s>>>(ids, (const T*)w, (T*)out, n, num, dim, bad_id_dev);
    return check_launch("embedding_forward");
  });
}

size_t tg_embedding_sort_scratch_bytes(int64_t n, int64_t num) {
  if (n <= 0 || num <= 0 || n > INT32_MAX) return 16;
  size_t temp = 0;
  const int bits = key_bits((uint64_t)num * (uint64_t)n - 1);
  cub::DeviceRadixSort::SortKeys(nullptr, temp, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                 (int)n, 0, bits);
  return ((size_t)n * 8 + 255) / 256 * 256 + temp + 256;
}

int tg_embedding_sort(const int64_t* ids, int64_t n, int64_t num, uint64_t* sorted_keys,
                      int* bad_id_dev, void* scratch, size_t scratch_bytes, void* stream) {
  TG_CHECK_ARG(n >= 0 && num > 0 && n <= INT32_MAX, "embedding_sort: bad sizes");
  TG_CHECK_ARG((uint64_t)num <= UINT64_MAX / (uint64_t)(n > 0 ? n : 1),
               "embedding_sort: num * n overflows 64 bits");
  if (n == 0) return TG_OK;
  TG_CHECK_ARG(scratch && scratch_bytes >= tg_embedding_sort_scratch_bytes(n, num),
               "embedding_sort: scratch too small");
  cudaStream_t s = as_stream(stream);
  uint64_t* keys = reinterpret_cast<uint64_t*>(scratch);
  const size_t keys_bytes = ((size_t)n * 8 + 255) / 256 * 256;
  const unsigned grid = (unsigned)((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
  embed_keys_kernel<<<grid, 256, 0, s>>>(ids, n, num, keys, bad_id_dev);
  int r = check_launch("embedding_sort(keys)");
  if (r) return r;
  const int bits = key_bits((uint64_t)num * (uint64_t)n - 1);
  size_t temp = scratch_bytes - keys_bytes;
  TG_CUDA_TRY(cub::DeviceRadixSort::SortKeys((uint8_t*)scratch + keys_bytes, temp, keys,
                                             sorted_keys, (int)n, 0, bits, s));
  return check_launch("embedding_sort(radix)", 0);
}

int tg_embedding_backward_sorted(int dtype, const void* g, const uint64_t* sorted_keys,
                                 int64_t n, void* gw, int64_t num, int64_t dim, int accumulate,
                                 void* stream) {
  cudaStream_t s = as_stream(stream);
  const size_t es = dtype == TG_F64 ? 8 : 4;
  if (!accumulate && num * dim > 0) TG_CUDA_TRY(cudaMemsetAsync(gw, 0, num * dim * es, s));
  if (n <= 0 || dim <= 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    const int64_t blocks = (n + 7) / 8;  // 8 warps per block
    embed_bwd_sorted_kernel<T><<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(
        (const T*)g, sorted_keys, n, (T*)gw, dim, accumulate);
    return check_launch("embedding_backward");
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
