// GEMM entry points and the linear layer's forward/VJP built on them.
#include <stdlib.h>

#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "reduce.cuh"

namespace tg {
namespace {

template <typename T>
GemmArgs<T> make_args(int ta, int tb, int64_t m, int64_t n, int64_t k, double alpha,
                      const void* a, int64_t lda, int64_t sa, const void* b, int64_t ldb,
                      int64_t sb, double beta, void* c, int64_t ldc, int64_t sc,
                      const void* bias, int64_t batch) {
  GemmArgs<T> p;
  p.m = m; p.n = n; p.k = k;
  p.a = (const T*)a; p.lda = lda; p.stride_a = sa;
  p.b = (const T*)b; p.ldb = ldb; p.stride_b = sb;
  p.c = (T*)c; p.ldc = ldc; p.stride_c = sc;
  p.bias = (const T*)bias;
  p.alpha = (T)alpha; p.beta = (T)beta;
  p.trans_a = ta; p.trans_b = tb;
  p.batch = batch;
  return p;
}

int check_gemm(int ta, int tb, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
               int64_t ldc) {
  TG_CHECK_ARG(m >= 0 && n >= 0 && k >= 0, "gemm: negative size");
  TG_CHECK_ARG(lda >= (ta ? m : k) || m == 0 || k == 0, "gemm: lda too small");
  TG_CHECK_ARG(ldb >= (tb ? k : n) || n == 0 || k == 0, "gemm: ldb too small");
  TG_CHECK_ARG(ldc >= n || m == 0, "gemm: ldc too small");
  return TG_OK;
}

// Forcing the SIMT path for fp32 (set TG_GEMM=simt) is a debugging switch for users.
bool force_simt() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM");
    v = (e && e[0] == 's') ? 1 : 0;
  }
  return v == 1;
}

// Live timing of tensor-core GEMM launches: when enabled, each launch is bracketed by two
// CUDA events on its own stream; tg_gemm_profile_read() sums the elapsed times.
struct ProfileRec {
  cudaEvent_t start, stop;
  double flops;
};
std::vector<ProfileRec> g_prof;
std::vector<cudaEvent_t> g_event_pool;
bool g_prof_on = false;

cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

// Largest split-K workspace the linear VJP asks its caller for.
constexpr size_t kLinearWorkspaceCap = size_t(128) << 20;

// Process-wide matmul precision of the fp32 tensor-core path (tg_set_matmul_precision).
int g_precision = 0;

// sum_{i < m} min(cap, i + 1): the entries of a causal (lower-triangular) band.
double tri_count(double m, double cap) {
  if (m <= cap) return m * (m + 1) / 2;
  return cap * (cap + 1) / 2 + (m - cap) * cap;
}

// Algorithmic FLOPs of one product: 2mnk per batch entry, counting only the causal half
// of the attention products (scores i >= j; reductions over k <= i or k >= i).
template <typename T>
double algorithmic_flops(const GemmArgs<T>& p) {
  const double m = (double)p.m, n = (double)p.n, k = (double)p.k, b = (double)p.batch;
  switch (p.kmode) {
    case GEMM_K_SKIP_UPPER: return 2.0 * b * k * tri_count(m, n);
    case GEMM_K_UP_TO_ROW: return 2.0 * b * n * tri_count(m, k);
    case GEMM_K_FROM_ROW: return 2.0 * b * n * (m * k - tri_count(m, k) + (m < k ? m : k));
    default: return 2.0 * b * m * n * k;
  }
}

// The tensor-core kernel, bracketed by profiling events when profiling is on.
int tc_timed(const GemmArgs<float>& p, cudaStream_t s) {
  ProfileRec rec{};
  if (g_prof_on) {
    rec = {take_event(), take_event(), algorithmic_flops(p)};
    cudaEventRecord(rec.start, s);
  }
  const int rc = gemm_tc_f32(p, s);
  if (g_prof_on) {
    if (rc == TG_OK) {
      cudaEventRecord(rec.stop, s);
      g_prof.push_back(rec);
    } else {
      g_event_pool.push_back(rec.start);
      g_event_pool.push_back(rec.stop);
    }
  }
  return rc;
}

template <typename T>
int gemm_dispatch(GemmArgs<T> p, bool allow_tc, cudaStream_t s) {
  if (p.m == 0 || p.n == 0) return TG_OK;
  p.precision = g_precision;
  if (p.k == 0) {
    // C = beta * C (+ bias): run the SIMT kernel, whose k loop is empty.
    return gemm_simt<T>(p, s);
  }
  if constexpr (sizeof(T) == 4) {
    if (allow_tc && !force_simt()) {
      const int rc = tc_timed(p, s);
      if (rc != TG_ERR_UNSUPPORTED) return rc;
    }
  }
  return gemm_simt<T>(p, s);
}

}  // namespace

int gemm_tc_profiled(const GemmArgs<float>& p, cudaStream_t stream) {
  return tc_timed(p, stream);
}

template <typename T>
int gemm_run(const GemmArgs<T>& p, cudaStream_t stream) {
  return gemm_dispatch<T>(p, true, stream);
}
template int gemm_run<float>(const GemmArgs<float>&, cudaStream_t);
template int gemm_run<double>(const GemmArgs<double>&, cudaStream_t);

}  // namespace tg

using namespace tg;

extern "C" {

int tg_gemm(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, double alpha,
            const void* a, int64_t lda, const void* b, int64_t ldb, double beta, void* c,
            int64_t ldc, const void* bias, void* stream) {
  const int rc = check_gemm(trans_a, trans_b, m, n, k, lda, ldb, ldc);
  if (rc) return rc;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    auto p = make_args<T>(trans_a, trans_b, m, n, k, alpha, a, lda, 0, b, ldb, 0, beta, c, ldc,
                          0, bias, 1);
    return gemm_dispatch<T>(p, true, as_stream(stream));
  });
}

int tg_gemm_simt(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                 double alpha, const void* a, int64_t lda, const void* b, int64_t ldb,
                 double beta, void* c, int64_t ldc, const void* bias, void* stream) {
  const int rc = check_gemm(trans_a, trans_b, m, n, k, lda, ldb, ldc);
  if (rc) return rc;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    auto p = make_args<T>(trans_a, trans_b, m, n, k, alpha, a, lda, 0, b, ldb, 0, beta, c, ldc,
                          0, bias, 1);
    return gemm_dispatch<T>(p, false, as_stream(stream));
  });
}

int tg_gemm_batched(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                    double alpha, const void* a, int64_t lda, int64_t stride_a, const void* b,
                    int64_t ldb, int64_t stride_b, double beta, void* c, int64_t ldc,
                    int64_t stride_c, int64_t batch, void* stream) {
  const int rc = check_gemm(trans_a, trans_b, m, n, k, lda, ldb, ldc);
  if (rc) return rc;
  TG_CHECK_ARG(batch >= 0 && batch <= 65535, "gemm_batched: batch %lld out of range",
               (long long)batch);
  if (batch == 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    auto p = make_args<T>(trans_a, trans_b, m, n, k, alpha, a, lda, stride_a, b, ldb, stride_b,
                          beta, c, ldc, stride_c, nullptr, batch);
    return gemm_dispatch<T>(p, true, as_stream(stream));
  });
}

int tg_set_matmul_precision(int precision) {
  TG_CHECK_ARG(precision == 0 || precision == 1, "matmul precision %d (0 = fp32, 1 = tf32)",
               precision);
  g_precision = precision;
  return TG_OK;
}

int tg_gemm_profile(int enable) {
  g_prof_on = enable != 0;
  return TG_OK;
}

int tg_gemm_profile_read(double* total_ms, int64_t* launches, double* flops) {
  double ms = 0.0, fl = 0.0;
  for (auto& r : g_prof) {
    TG_CUDA_TRY(cudaEventSynchronize(r.stop));
    float t = 0.f;
    TG_CUDA_TRY(cudaEventElapsedTime(&t, r.start, r.stop));
    ms += t;
    fl += r.flops;
    g_event_pool.push_back(r.start);
    g_event_pool.push_back(r.stop);
  }
  if (total_ms) *total_ms = ms;
  if (launches) *launches = (int64_t)g_prof.size();
  if (flops) *flops = fl;
  g_prof.clear();
  return TG_OK;
}

int tg_linear_forward(int dtype, const void* x, const void* w, const void* bias, void* y,
                      int64_t rows, int64_t in_features, int64_t out_features, void* stream) {
  return tg_gemm(dtype, 0, 1, rows, out_features, in_features, 1.0, x, in_features, w,
                 in_features, 0.0, y, out_features, bias, stream);
}

size_t tg_linear_backward_scratch_bytes(int dtype, int64_t rows, int64_t in_features,
                                        int64_t out_features, unsigned need) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  size_t bytes = (need & 4) ? (tg_colsum_scratch_bytes(dtype, rows, out_features) + 255) / 256 * 256
                            : 0;
  if (dtype == TG_F32) {
    int64_t mn = 0;
    if (need & 1) mn = rows * in_features;
    if ((need & 2) && out_features * in_features > mn) mn = out_features * in_features;
    size_t ws = (size_t)mn * es * 4;  // room for four split-K partials
    if (ws > kLinearWorkspaceCap) ws = kLinearWorkspaceCap;
    bytes += ws;
  }
  return bytes ? bytes : 16;
}

int tg_linear_backward(int dtype, const void* g, const void* x, const void* w, void* gx, void* gw,
                       void* gb, int64_t rows, int64_t in_features, int64_t out_features,
                       unsigned need, double beta_gw, void* scratch, void* stream) {
  int rc = check_gemm(0, 0, rows, in_features, out_features, out_features, in_features,
                      in_features);
  if (rc) return rc;
  TG_CHECK_ARG(!((need & 4) && gb) || scratch, "linear_backward: scratch is NULL");
  // Split-K partials (tensor-core products) live after the column-sum partials.
  const size_t cs = (need & 4) ? (tg_colsum_scratch_bytes(dtype, rows, out_features) + 255) / 256 * 256
                               : 0;
  const size_t total = scratch ? tg_linear_backward_scratch_bytes(dtype, rows, in_features,
                                                                  out_features, need) : 0;
  float* ws = (scratch && total > cs + 16) ? reinterpret_cast<float*>((uint8_t*)scratch + cs)
                                           : nullptr;
  const size_t ws_bytes = ws ? total - cs : 0;
  cudaStream_t s = as_stream(stream);
  rc = TG_DISPATCH_FLOAT(dtype, T, [&] {
    if ((need & 1) && gx) {
      // gx[rows, in] = g[rows, out] @ w[out, in]
      auto p = make_args<T>(0, 0, rows, in_features, out_features, 1.0, g, out_features, 0, w,
                            in_features, 0, 0.0, gx, in_features, 0, nullptr, 1);
      p.workspace = ws;
      p.workspace_bytes = ws_bytes;
      const int r = gemm_dispatch<T>(p, true, s);
      if (r) return r;
    }
    if ((need & 2) && gw) {
      // gw[out, in] = g^T @ x: A = g stored rows x out (k x m), B = x stored rows x in (k x n)
      auto p = make_args<T>(1, 0, out_features, in_features, rows, 1.0, g, out_features, 0, x,
                            in_features, 0, beta_gw, gw, in_features, 0, nullptr, 1);
      p.workspace = ws;
      p.workspace_bytes = ws_bytes;
      const int r = gemm_dispatch<T>(p, true, s);
      if (r) return r;
    }
    return (int)TG_OK;
  });
  if (rc) return rc;
  if ((need & 4) && gb) rc = tg_colsum(dtype, g, gb, rows, out_features, 0, scratch, stream);
  return rc;
}

}  // extern "C"
