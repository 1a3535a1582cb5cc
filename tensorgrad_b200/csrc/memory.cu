// Device and pinned host memory, and events, for the host package (no framework allocator).
//
// Device buffers come from the CUDA stream-ordered allocator: each device's default memory
// pool has its release threshold raised to "never", so freed blocks stay in the pool and a
// later allocation of the step reuses them without a cudaMalloc (the same effect as a caching
// allocator, kept by the driver, with frees ordered on the stream that used the buffer).
// Page-locked host buffers are cudaHostAlloc'd; events are timing-free CUDA events.
#include <mutex>

#include "common.cuh"

namespace tg {
namespace {

constexpr int kMaxDevices = 64;
std::once_flag g_pool_once[kMaxDevices];

int retain_pool(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return set_error(TG_ERR_UNSUPPORTED, "device %d", dev);
  int rc = TG_OK;
  std::call_once(g_pool_once[dev], [&] {
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) != cudaSuccess) {
      rc = set_error(TG_ERR_CUDA, "no default memory pool on device %d", dev);
      return;
    }
    uint64_t keep = UINT64_MAX;
    if (cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess)
      rc = set_error(TG_ERR_CUDA, "memory pool release threshold on device %d", dev);
  });
  return rc;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int tg_malloc(void** ptr, size_t bytes, void* stream) {
  TG_CHECK_ARG(ptr != nullptr, "tg_malloc: NULL result pointer");
  *ptr = nullptr;
  if (bytes == 0) bytes = 16;
  int dev = 0;
  TG_CUDA_TRY(cudaGetDevice(&dev));
  const int rc = retain_pool(dev);
  if (rc != TG_OK) return rc;
  const cudaError_t e = cudaMallocAsync(ptr, bytes, as_stream(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(e == cudaErrorMemoryAllocation ? TG_ERR_OOM : TG_ERR_CUDA,
                     "tg_malloc(%zu bytes): %s", bytes, cudaGetErrorString(e));
  }
  return TG_OK;
}

int tg_free(void* ptr, void* stream) {
  if (!ptr) return TG_OK;
  TG_CUDA_TRY(cudaFreeAsync(ptr, as_stream(stream)));
  return TG_OK;
}

int tg_pool_stats(int device, uint64_t* reserved_bytes, uint64_t* used_bytes) {
  cudaMemPool_t pool;
  TG_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
  uint64_t r = 0, u = 0;
  TG_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &r));
  TG_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, &u));
  if (reserved_bytes) *reserved_bytes = r;
  if (used_bytes) *used_bytes = u;
  return TG_OK;
}

int tg_pool_peak(int device, int reset, uint64_t* used_high_bytes) {
  cudaMemPool_t pool;
  TG_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
  uint64_t high = 0;
  TG_CUDA_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &high));
  if (used_high_bytes) *used_high_bytes = high;
  if (reset) {
    uint64_t zero = 0;  // the watermark can only be reset to zero (then tracks from now)
    TG_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &zero));
  }
  return TG_OK;
}

int tg_host_alloc(void** ptr, size_t bytes) {
  TG_CHECK_ARG(ptr != nullptr, "tg_host_alloc: NULL result pointer");
  *ptr = nullptr;
  TG_CUDA_TRY(cudaHostAlloc(ptr, bytes ? bytes : 16, cudaHostAllocDefault));
  return TG_OK;
}

int tg_host_free(void* ptr) {
  if (!ptr) return TG_OK;
  TG_CUDA_TRY(cudaFreeHost(ptr));
  return TG_OK;
}

int tg_set_device(int device) {
  TG_CUDA_TRY(cudaSetDevice(device));
  return TG_OK;
}

int tg_get_device(int* device) {
  TG_CUDA_TRY(cudaGetDevice(device));
  return TG_OK;
}

int tg_device_count(int* count) {
  *count = 0;
  const cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *count = 0;
  }
  return TG_OK;
}

int tg_event_create(void** event) {
  cudaEvent_t e;
  TG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  *event = e;
  return TG_OK;
}

int tg_event_record(void* event, void* stream) {
  TG_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(event), as_stream(stream)));
  return TG_OK;
}

// 1 when every piece of work recorded before the event has completed, 0 if not yet.
int tg_event_query(void* event) {
  const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
  if (e == cudaSuccess) return 1;
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    return 0;
  }
  return -set_error(TG_ERR_CUDA, "event query: %s", cudaGetErrorString(e));
}

int tg_event_destroy(void* event) {
  if (event) TG_CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return TG_OK;
}

}  // extern "C"
