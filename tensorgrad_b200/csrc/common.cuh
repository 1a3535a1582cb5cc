// Shared helpers of the tensorgrad_b200 C-ABI library: status codes, the per-thread error
// message, launch checking, dtype dispatch and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <cmath>
#include <utility>

#include "../../include/tgb200.h"

namespace tg {

// Records a detail message for tg_last_error() (per host thread) and returns `status`.
int set_error(int status, const char* fmt, ...);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch, for chains of short kernels (the recurrent steps): a kernel
// launched with launch_pdl may be scheduled before the kernel ahead of it on the stream has
// finished. Such a kernel calls pdl_trigger() (lets its own successor be scheduled) and then
// pdl_wait() before it touches any global memory: the wait returns once the kernel ahead has
// completed and its writes are visible. A kernel without the attribute waits as usual.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// TG_PDL=0 launches such kernels plainly (for comparison probes); read once per process.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Returns TG_OK, or TG_ERR_CUDA with the launch error recorded under `what`. `kernels` is
// how many kernels the calling entry point just launched (added to tg_launch_count()).
int check_launch(const char* what, int kernels = 1);

#define TG_CHECK_ARG(cond, ...)                              \
  do {                                                       \
    if (!(cond)) return ::tg::set_error(TG_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define TG_CUDA_TRY(expr)                                                          \
  do {                                                                             \
    cudaError_t _e = (expr);                                                       \
    if (_e != cudaSuccess)                                                         \
      return ::tg::set_error(TG_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

// Dispatch a templated body on the element type code.
#define TG_DISPATCH_FLOAT(dtype, T, ...)                                  \
  [&]() -> int {                                                          \
    if ((dtype) == TG_F32) { using T = float; return __VA_ARGS__(); }    \
    if ((dtype) == TG_F64) { using T = double; return __VA_ARGS__(); }   \
    return ::tg::set_error(TG_ERR_ARG, "unsupported dtype code %d", (int)(dtype)); \
  }()

inline unsigned grid_for(int64_t n, int threads, int64_t cap = 148 * 32) {
  int64_t b = (n + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > cap) b = cap;
  return (unsigned)b;
}

// ---------------------------------------------------------------- device helpers
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; every thread receives the result. `sh` holds >= 32 elements.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  T r = (threadIdx.x < nw) ? sh[threadIdx.x] : T(0);
  if (wid == 0) r = warp_sum(r);
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  return sh[0];
}

template <typename T>
__device__ __forceinline__ T block_max(T v, T* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  T r = (threadIdx.x < nw) ? sh[threadIdx.x] : T(-INFINITY);
  if (wid == 0) r = warp_max(r);
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  return sh[0];
}

template <typename T> __device__ __forceinline__ T dev_exp(T x);
template <> __device__ __forceinline__ float dev_exp<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double dev_exp<double>(double x) { return exp(x); }
template <typename T> __device__ __forceinline__ T dev_log(T x);
template <> __device__ __forceinline__ float dev_log<float>(float x) { return logf(x); }
template <> __device__ __forceinline__ double dev_log<double>(double x) { return log(x); }
template <typename T> __device__ __forceinline__ T dev_tanh(T x);
template <> __device__ __forceinline__ float dev_tanh<float>(float x) { return tanhf(x); }
template <> __device__ __forceinline__ double dev_tanh<double>(double x) { return tanh(x); }
template <typename T> __device__ __forceinline__ T dev_sqrt(T x);
template <> __device__ __forceinline__ float dev_sqrt<float>(float x) { return sqrtf(x); }
template <> __device__ __forceinline__ double dev_sqrt<double>(double x) { return sqrt(x); }

}  // namespace tg
