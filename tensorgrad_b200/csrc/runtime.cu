// Status reporting, device queries and memory movement of the C ABI.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"

namespace tg {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

static unsigned long long g_launches = 0;

int check_launch(const char* what, int kernels) {
  __atomic_fetch_add(&g_launches, (unsigned long long)kernels, __ATOMIC_RELAXED);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TG_OK;
}

}  // namespace tg

extern "C" {

int tg_version(void) { return 100; }

uint64_t tg_launch_count(void) { return __atomic_load_n(&tg::g_launches, __ATOMIC_RELAXED); }

const char* tg_status_string(int status) {
  switch (status) {
    case TG_OK: return "ok";
    case TG_ERR_ARG: return "invalid argument";
    case TG_ERR_CUDA: return "CUDA error";
    case TG_ERR_UNSUPPORTED: return "unsupported";
    case TG_ERR_INDEX: return "index out of range";
    case TG_ERR_TIMEOUT: return "timed out";
    case TG_ERR_OOM: return "out of device memory";
    case TG_ERR_COMM: return "collective failed";
  }
  return "unknown status";
}

int tg_last_error(char* buf, size_t len) {
  if (!buf || !len) return TG_ERR_ARG;
  strncpy(buf, tg::g_last_error, len - 1);
  buf[len - 1] = 0;
  return TG_OK;
}

int tg_device_info(int device, int* sm_count, int* cc_major, int* cc_minor) {
  TG_CUDA_TRY(cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, device));
  TG_CUDA_TRY(cudaDeviceGetAttribute(cc_major, cudaDevAttrComputeCapabilityMajor, device));
  TG_CUDA_TRY(cudaDeviceGetAttribute(cc_minor, cudaDevAttrComputeCapabilityMinor, device));
  return TG_OK;
}

int tg_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return TG_OK;
  TG_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, tg::as_stream(stream)));
  return TG_OK;
}

int tg_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return TG_OK;
  TG_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, tg::as_stream(stream)));
  return TG_OK;
}

int tg_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return TG_OK;
  TG_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, tg::as_stream(stream)));
  return TG_OK;
}

int tg_memset_zero(void* dst, size_t bytes, void* stream) {
  if (!bytes) return TG_OK;
  TG_CUDA_TRY(cudaMemsetAsync(dst, 0, bytes, tg::as_stream(stream)));
  return TG_OK;
}

int tg_stream_synchronize(void* stream) {
  TG_CUDA_TRY(cudaStreamSynchronize(tg::as_stream(stream)));
  return TG_OK;
}

}  // extern "C"
