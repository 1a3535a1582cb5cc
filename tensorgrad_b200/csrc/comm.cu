// Gradient all-reduce across the GPUs of one box through NCCL, with failure detection.
//
// The reference is single-process; data-parallel training adds one exchange step per step: the
// average of every gradient over the ranks. This file binds NCCL at run time (dlopen of the
// library path the host gives, so the process shares one NCCL with any framework it loaded)
// and wraps it for that step:
//   * communicators are created nonblocking (ncclConfig_t.blocking = 0) and their set-up is
//     polled against a deadline, so a rank that never joins ends in TG_ERR_TIMEOUT instead of
//     a hang;
//   * every collective runs on the communicator's own stream, ordered after the compute
//     stream's work by an event, so the exchange overlaps the rest of the backward pass; the
//     compute stream waits for it (tg_comm_join) without a host synchronisation;
//   * tg_comm_wait polls the communicator's stream and its asynchronous error state on the host
//     with a deadline; on an error or an expired deadline it aborts the communicator (which
//     ends NCCL's kernels) and returns TG_ERR_COMM or TG_ERR_TIMEOUT.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "common.cuh"

namespace tg {
namespace {

struct Nccl {
  void* handle = nullptr;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommFinalize) finalize = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclGetVersion) get_version = nullptr;
};

Nccl g_nccl;
std::mutex g_nccl_mutex;

template <typename F>
bool bind(void* h, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

int need_nccl() {
  if (!g_nccl.handle)
    return set_error(TG_ERR_UNSUPPORTED, "NCCL is not loaded (call tg_comm_load first)");
  return TG_OK;
}

double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

void pause_us(long us) {
  timespec ts{0, us * 1000};
  nanosleep(&ts, nullptr);
}

struct Comm {
  ncclComm_t comm = nullptr;
  cudaStream_t stream = nullptr;  // the collectives' stream
  cudaEvent_t ready = nullptr;    // compute stream -> collective stream
  cudaEvent_t done = nullptr;     // collective stream -> compute stream
  int rank = 0, nranks = 1;
  bool aborted = false;
};

// Aborts and records why; the communicator cannot be used afterwards.
int fail(Comm* c, int status, const char* what, const char* detail) {
  if (!c->aborted && c->comm) {
    g_nccl.abort(c->comm);
    c->aborted = true;
  }
  return set_error(status, "%s (rank %d of %d): %s; the communicator was aborted", what, c->rank,
                   c->nranks, detail);
}

// Polls the communicator's asynchronous state until it leaves ncclInProgress.
int settle(Comm* c, double deadline, const char* what) {
  while (true) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = g_nccl.get_async_error(c->comm, &st);
    if (q != ncclSuccess && q != ncclInProgress)
      return fail(c, TG_ERR_COMM, what, g_nccl.error_string(q));
    if (st == ncclSuccess) return TG_OK;
    if (st != ncclInProgress) return fail(c, TG_ERR_COMM, what, g_nccl.error_string(st));
    if (now_s() > deadline) return fail(c, TG_ERR_TIMEOUT, what, "deadline passed");
    pause_us(50);
  }
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

int tg_comm_load(const char* library_path) {
  std::lock_guard<std::mutex> lock(g_nccl_mutex);
  if (g_nccl.handle) return TG_OK;
  const char* path = (library_path && library_path[0]) ? library_path : "libnccl.so.2";
  // An NCCL this process already loaded is used as is (one NCCL per process).
  void* h = dlopen(path, RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) return set_error(TG_ERR_UNSUPPORTED, "cannot load NCCL from %s: %s", path, dlerror());
  Nccl n;
  n.handle = h;
  if (!bind(h, "ncclGetUniqueId", n.get_unique_id) ||
      !bind(h, "ncclCommInitRankConfig", n.init_rank_config) ||
      !bind(h, "ncclCommGetAsyncError", n.get_async_error) ||
      !bind(h, "ncclAllReduce", n.all_reduce) || !bind(h, "ncclCommAbort", n.abort) ||
      !bind(h, "ncclCommFinalize", n.finalize) || !bind(h, "ncclCommDestroy", n.destroy) ||
      !bind(h, "ncclGetErrorString", n.error_string) ||
      !bind(h, "ncclGetVersion", n.get_version))
    return set_error(TG_ERR_UNSUPPORTED, "NCCL at %s lacks a needed entry point", path);
  g_nccl = n;
  return TG_OK;
}

int tg_comm_nccl_version(int* version) {
  int rc = need_nccl();
  if (rc) return rc;
  const ncclResult_t r = g_nccl.get_version(version);
  return r == ncclSuccess ? TG_OK : set_error(TG_ERR_COMM, "ncclGetVersion failed");
}

/* Writes the 128-byte NCCL unique id (rank 0 makes it; every rank then passes it in). */
int tg_comm_unique_id(void* out, size_t len) {
  int rc = need_nccl();
  if (rc) return rc;
  TG_CHECK_ARG(out && len >= sizeof(ncclUniqueId), "tg_comm_unique_id: buffer < %zu bytes",
               sizeof(ncclUniqueId));
  ncclUniqueId id;
  const ncclResult_t r = g_nccl.get_unique_id(&id);
  if (r != ncclSuccess) return set_error(TG_ERR_COMM, "ncclGetUniqueId: %s", g_nccl.error_string(r));
  memcpy(out, &id, sizeof(id));
  return TG_OK;
}

int tg_comm_init(int nranks, int rank, const void* unique_id, double timeout_s, void** out) {
  int rc = need_nccl();
  if (rc) return rc;
  TG_CHECK_ARG(out && unique_id && nranks >= 1 && rank >= 0 && rank < nranks && timeout_s > 0,
               "tg_comm_init: bad arguments");
  *out = nullptr;
  Comm* c = new Comm();
  c->rank = rank;
  c->nranks = nranks;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ready, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    delete c;
    return set_error(TG_ERR_CUDA, "tg_comm_init: stream/event creation failed");
  }
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;  // set-up and calls return at once; completion is polled
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  const ncclResult_t r = g_nccl.init_rank_config(&c->comm, nranks, id, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    const int st = set_error(TG_ERR_COMM, "ncclCommInitRankConfig: %s", g_nccl.error_string(r));
    if (c->comm) g_nccl.abort(c->comm);
    delete c;
    return st;
  }
  rc = settle(c, now_s() + timeout_s, "communicator set-up");
  if (rc != TG_OK) {  // aborted by settle()
    cudaEventDestroy(c->ready);
    cudaEventDestroy(c->done);
    cudaStreamDestroy(c->stream);
    delete c;
    return rc;
  }
  *out = c;
  return TG_OK;
}

/* In-place sum (average = 0) or average (average != 0) of `count` elements of `buf` over the
 * ranks, on the communicator's stream after the work queued so far on `stream`. */
int tg_comm_all_reduce(void* comm, void* buf, size_t count, int dtype, int average,
                       void* stream, double timeout_s) {
  Comm* c = static_cast<Comm*>(comm);
  TG_CHECK_ARG(c && !c->aborted, "tg_comm_all_reduce: no usable communicator");
  TG_CHECK_ARG(dtype == TG_F32 || dtype == TG_F64, "tg_comm_all_reduce: dtype %d", dtype);
  if (count == 0) return TG_OK;
  TG_CUDA_TRY(cudaEventRecord(c->ready, as_stream(stream)));
  TG_CUDA_TRY(cudaStreamWaitEvent(c->stream, c->ready, 0));
  const ncclResult_t r =
      g_nccl.all_reduce(buf, buf, count, dtype == TG_F32 ? ncclFloat32 : ncclFloat64,
                        average ? ncclAvg : ncclSum, c->comm, c->stream);
  if (r != ncclSuccess && r != ncclInProgress)
    return fail(c, TG_ERR_COMM, "ncclAllReduce", g_nccl.error_string(r));
  if (r == ncclInProgress) return settle(c, now_s() + timeout_s, "ncclAllReduce enqueue");
  return TG_OK;
}

/* `stream` waits (on the device) for every collective issued so far. */
int tg_comm_join(void* comm, void* stream) {
  Comm* c = static_cast<Comm*>(comm);
  TG_CHECK_ARG(c != nullptr, "tg_comm_join: NULL communicator");
  TG_CUDA_TRY(cudaEventRecord(c->done, c->stream));
  TG_CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), c->done, 0));
  return TG_OK;
}

/* Host-side watch: returns once every collective issued so far has completed, or, when the
 * communicator reports an error or `timeout_s` passes first, aborts it and returns
 * TG_ERR_COMM / TG_ERR_TIMEOUT. */
int tg_comm_wait(void* comm, double timeout_s) {
  Comm* c = static_cast<Comm*>(comm);
  TG_CHECK_ARG(c != nullptr, "tg_comm_wait: NULL communicator");
  if (c->aborted) return set_error(TG_ERR_COMM, "tg_comm_wait: communicator was aborted");
  const double deadline = now_s() + timeout_s;
  while (true) {
    const cudaError_t q = cudaStreamQuery(c->stream);
    if (q == cudaSuccess) return TG_OK;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      return fail(c, TG_ERR_CUDA, "collective stream", cudaGetErrorString(q));
    }
    ncclResult_t st = ncclSuccess;
    g_nccl.get_async_error(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress)
      return fail(c, TG_ERR_COMM, "collective", g_nccl.error_string(st));
    if (now_s() > deadline) return fail(c, TG_ERR_TIMEOUT, "collective", "deadline passed");
    pause_us(20);
  }
}

int tg_comm_abort(void* comm) {
  Comm* c = static_cast<Comm*>(comm);
  if (c && !c->aborted && c->comm) {
    g_nccl.abort(c->comm);
    c->aborted = true;
  }
  return TG_OK;
}

/* Finalises (bounded by timeout_s, else aborts) and frees the communicator. */
int tg_comm_destroy(void* comm, double timeout_s) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) return TG_OK;
  int rc = TG_OK;
  if (!c->aborted && c->comm) {
    const ncclResult_t r = g_nccl.finalize(c->comm);
    if (r == ncclSuccess || r == ncclInProgress)
      rc = settle(c, now_s() + timeout_s, "communicator finalize");
    else
      rc = fail(c, TG_ERR_COMM, "ncclCommFinalize", g_nccl.error_string(r));
    if (!c->aborted) g_nccl.destroy(c->comm);
  }
  cudaEventDestroy(c->ready);
  cudaEventDestroy(c->done);
  cudaStreamDestroy(c->stream);
  delete c;
  return rc;
}

}  // extern "C"
