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
unsigned long long g_fallbacks = 0;  // fp32 products the tensor-core kernel could not take

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


// Scratch of tg_linear_backward: column-sum partials (cs), split-K partials (ws, fp32 only)
// and, for fp32 with out_features not a multiple of 4, a copy of the gradient with rows padded
// to a multiple of 4 elements (gpad), which the tensor maps need.
struct LinearBwdScratch {
  size_t cs = 0, ws = 0, gpad = 0, total = 0;
};

LinearBwdScratch linear_bwd_scratch(int dtype, int64_t rows, int64_t in_features,
                                    int64_t out_features, unsigned need) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  LinearBwdScratch L;
  if (need & 4) L.cs = (tg_colsum_scratch_bytes(dtype, rows, out_features) + 255) / 256 * 256;
  if (dtype == TG_F32) {
    int64_t mn = 0;
    if (need & 1) mn = rows * in_features;
    if ((need & 2) && out_features * in_features > mn) mn = out_features * in_features;
    size_t ws = (size_t)mn * es * 4;  // room for four split-K partials
    if (ws > kLinearWorkspaceCap) ws = kLinearWorkspaceCap;
    L.ws = (ws + 255) / 256 * 256;
    if ((out_features % 4) && (need & 3))
      L.gpad = ((size_t)rows * (size_t)((out_features + 3) / 4 * 4) * es + 255) / 256 * 256;
  }
  L.total = L.cs + L.ws + L.gpad;
  return L;
}

// Split-K partials for a linear forward whose output has too few tiles to fill the SMs while
// its reduction is long (e.g. a classifier head over a wide flattened input): room for up to
// about two splits per SM. Zero when the product already fills the GPU or is not fp32.
size_t linear_fwd_workspace(int dtype, int64_t rows, int64_t in_features, int64_t out_features) {
  if (dtype != TG_F32 || rows <= 0 || out_features <= 0 || in_features < 1024) return 0;
  const int64_t tiles = ((rows + 127) / 128) * ((out_features + 63) / 64);
  if (tiles >= 74) return 0;
  const int64_t splits = (296 + tiles - 1) / tiles;
  return ((size_t)splits * (size_t)rows * (size_t)out_features * sizeof(float) + 255) / 256 * 256;
}

// dst (rows x cols, row stride ldd) = src (row stride lds).
template <typename T>
__global__ void copy_rows_kernel(const T* __restrict__ src, int64_t lds, T* __restrict__ dst,
                                 int64_t ldd, int64_t rows, int64_t cols) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) dst[r * ldd + c] = src[r * lds + c];
}
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
  if (gemm_smallk_applies(p)) return gemm_smallk<T>(p, s);
  if constexpr (sizeof(T) == 4) {
    if (allow_tc && !force_simt()) {
      const int rc = tc_timed(p, s);
      if (rc != TG_ERR_UNSUPPORTED) return rc;
      // Not a tensor-core shape (an operand off a 16-byte boundary, a stride not a multiple
      // of 4 floats): counted, so that tests can require none on the training steps.
      __atomic_fetch_add(&g_fallbacks, 1ull, __ATOMIC_RELAXED);
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

uint64_t tg_gemm_fallback_count(void) {
  return __atomic_load_n(&g_fallbacks, __ATOMIC_RELAXED);
}

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

size_t tg_linear_forward_scratch_bytes(int dtype, int64_t rows, int64_t in_features,
                                       int64_t out_features) {
  const size_t ws = linear_fwd_workspace(dtype, rows, in_features, out_features);
  return ws ? ws : 16;
}

int tg_linear_forward(int dtype, const void* x, const void* w, const void* bias, void* y,
                      int64_t rows, int64_t in_features, int64_t out_features, void* scratch,
                      void* stream) {
  const size_t ws = scratch ? linear_fwd_workspace(dtype, rows, in_features, out_features) : 0;
  if (ws == 0)
    return tg_gemm(dtype, 0, 1, rows, out_features, in_features, 1.0, x, in_features, w,
                   in_features, 0.0, y, out_features, bias, stream);
  int rc = check_gemm(0, 1, rows, out_features, in_features, in_features, in_features,
                      out_features);
  if (rc) return rc;
  auto p = make_args<float>(0, 1, rows, out_features, in_features, 1.0, x, in_features, 0, w,
                            in_features, 0, 0.0, y, out_features, 0, bias, 1);
  p.workspace = reinterpret_cast<float*>(scratch);
  p.workspace_bytes = ws;
  return gemm_dispatch<float>(p, true, as_stream(stream));
}

size_t tg_linear_backward_scratch_bytes(int dtype, int64_t rows, int64_t in_features,
                                        int64_t out_features, unsigned need) {
  const LinearBwdScratch L = linear_bwd_scratch(dtype, rows, in_features, out_features, need);
  return L.total ? L.total : 16;
}

int tg_linear_backward(int dtype, const void* g, const void* x, const void* w, void* gx, void* gw,
                       void* gb, int64_t rows, int64_t in_features, int64_t out_features,
                       unsigned need, double beta_gw, void* scratch, void* stream) {
  int rc = check_gemm(0, 0, rows, in_features, out_features, out_features, in_features,
                      in_features);
  if (rc) return rc;
  TG_CHECK_ARG(!((need & 4) && gb) || scratch, "linear_backward: scratch is NULL");
  // Scratch: column-sum partials, then split-K partials (tensor-core products), then the
  // gradient re-laid with 16-byte rows when out_features is not a multiple of 4.
  const LinearBwdScratch L = scratch ? linear_bwd_scratch(dtype, rows, in_features,
                                                          out_features, need)
                                     : LinearBwdScratch{};
  uint8_t* base = (uint8_t*)scratch;
  float* ws = L.ws ? reinterpret_cast<float*>(base + L.cs) : nullptr;
  cudaStream_t s = as_stream(stream);
  rc = TG_DISPATCH_FLOAT(dtype, T, [&] {
    const T* gk = (const T*)g;
    int64_t ldg = out_features;
    if (L.gpad && (((need & 1) && gx) || ((need & 2) && gw))) {
      ldg = (out_features + 3) / 4 * 4;
      T* gp = reinterpret_cast<T*>(base + L.cs + L.ws);
      copy_rows_kernel<T><<<dim3(1, (unsigned)(rows < 65535 ? rows : 65535)), 128, 0, s>>>(
          (const T*)g, out_features, gp, ldg, rows, out_features);
      const int r = check_launch("linear_backward(relayout)");
      if (r) return r;
      gk = gp;
    }
    if ((need & 1) && gx) {
      // gx[rows, in] = g[rows, out] @ w[out, in]
      auto p = make_args<T>(0, 0, rows, in_features, out_features, 1.0, gk, ldg, 0, w,
                            in_features, 0, 0.0, gx, in_features, 0, nullptr, 1);
      p.workspace = ws;
      p.workspace_bytes = L.ws;
      const int r = gemm_dispatch<T>(p, true, s);
      if (r) return r;
    }
    if ((need & 2) && gw) {
      // gw[out, in] = g^T @ x: A = g stored rows x out (k x m), B = x stored rows x in (k x n)
      auto p = make_args<T>(1, 0, out_features, in_features, rows, 1.0, gk, ldg, 0, x,
                            in_features, 0, beta_gw, gw, in_features, 0, nullptr, 1);
      p.workspace = ws;
      p.workspace_bytes = L.ws;
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
