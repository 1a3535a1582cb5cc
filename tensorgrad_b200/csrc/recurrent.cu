// Elman RNN, LSTM and GRU over a whole sequence with backpropagation through time
// (ops/recurrent.py).
//
// One C-ABI call runs a whole sequence, so the host loop over time steps is C++, not Python:
//   forward : the input projection of every step as one GEMM (bias in its epilogue), then per
//             step one recurrent GEMM (tcgen05 3xTF32 for fp32) and one gate kernel that
//             applies the nonlinearities and writes the states in the reference's layout;
//   backward: per step (reverse time) one gate-VJP kernel, which also folds in the output
//             gradient of that step and carries the cell gradient, and one GEMM
//             dh = dz W_hh (split over CTAs when it has few tiles); then one GEMM per weight
//             over all steps and column sums for the biases.
// Gate order and formulas are the reference's (PyTorch's): LSTM (i, f, g, o), GRU (r, u, n)
// with n = tanh(a_n + r * (h W_hn^T + b_hn)).
#include "common.cuh"
#include "gemm.cuh"
#include "reduce.cuh"

namespace tg {
namespace {

constexpr int kThreads = 256;

inline size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// The reference's overflow-free logistic (ops/elementwise.py:230-237).
template <typename T>
__device__ __forceinline__ T sigm(T x) {
  const T z = dev_exp<T>(-fabs(x));
  return x >= T(0) ? T(1) / (T(1) + z) : z / (T(1) + z);
}

template <typename T>
__global__ void add_vec_kernel(const T* __restrict__ a, const T* __restrict__ b,
                               T* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = a[i] + b[i];
}

template <typename T>
__global__ void pad_cols_kernel(const T* __restrict__ x, T* __restrict__ xp, int64_t rows,
                                int64_t cols, int64_t ld) {
  const int64_t total = rows * ld;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / ld, c = i - r * ld;
    xp[i] = c < cols ? x[r * cols + c] : T(0);
  }
}

// ------------------------------------------------------------------ LSTM cells
// z (B, 4H) holds x W_ih^T + b + h W_hh^T; it is overwritten with the gates (i, f, g, o).
// out_t is (B, 2, H): hidden, then cell state.
template <typename T>
__global__ void __launch_bounds__(kThreads)
lstm_cell_fwd(T* __restrict__ z, const T* __restrict__ rec, const T* __restrict__ c_prev,
              int64_t c_ld, T* __restrict__ out_t, T* __restrict__ tanh_c, int64_t B, int64_t H) {
  const int64_t total = B * H;
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / H, j = idx - b * H;
    T* zr = z + b * 4 * H;
    const T* rr = rec + b * 4 * H;
    const T i = sigm(zr[j] + rr[j]), f = sigm(zr[H + j] + rr[H + j]);
    const T g = dev_tanh<T>(zr[2 * H + j] + rr[2 * H + j]);
    const T o = sigm(zr[3 * H + j] + rr[3 * H + j]);
    zr[j] = i;
    zr[H + j] = f;
    zr[2 * H + j] = g;
    zr[3 * H + j] = o;
    const T c = f * c_prev[b * c_ld + j] + i * g;
    const T tc = dev_tanh<T>(c);
    out_t[(b * 2 + 1) * H + j] = c;
    out_t[(b * 2) * H + j] = o * tc;
    tanh_c[idx] = tc;
  }
}

// One reverse step: dh = dh_carry + g_h, dc = dc_carry + g_c + dh o (1 - tanh(c)^2); the
// gate gradients go to dz (B, 4H); dc_carry becomes dc * f. `first` marks the last time step
// (the carries start at zero and are not read).
template <typename T>
__global__ void __launch_bounds__(kThreads)
lstm_cell_bwd(const T* __restrict__ gates, const T* __restrict__ tanh_c,
              const T* __restrict__ c_prev, int64_t c_ld, const T* __restrict__ g_t,
              const T* __restrict__ dh_carry, T* __restrict__ dc_carry, T* __restrict__ dz,
              int64_t B, int64_t H, int first) {
  const int64_t total = B * H;
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / H, j = idx - b * H;
    const T* a = gates + b * 4 * H;
    const T i = a[j], f = a[H + j], gg = a[2 * H + j], o = a[3 * H + j];
    const T tc = tanh_c[idx];
    T dh = g_t[(b * 2) * H + j];
    T dc = g_t[(b * 2 + 1) * H + j];
    if (!first) {
      dh = dh_carry[idx] + dh;
      dc = dc_carry[idx] + dc;
    }
    dc = dc + dh * o * (T(1) - tc * tc);
    T* d = dz + b * 4 * H;
    d[j] = dc * gg * (i * (T(1) - i));
    d[H + j] = dc * c_prev[b * c_ld + j] * (f * (T(1) - f));
    d[2 * H + j] = dc * i * (T(1) - gg * gg);
    d[3 * H + j] = dh * tc * (o * (T(1) - o));
    dc_carry[idx] = dc * f;
  }
}

// ------------------------------------------------------------------ GRU cells
// a (B, 3H) = x W_ih^T + b_ih, overwritten with (r, u, n); hw (B, 3H) = h W_hh^T + b_hh.
template <typename T>
__global__ void __launch_bounds__(kThreads)
gru_cell_fwd(T* __restrict__ a, const T* __restrict__ hw, const T* __restrict__ h_prev,
             T* __restrict__ hn_t, T* __restrict__ out_t, int64_t B, int64_t H) {
  const int64_t total = B * H;
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / H, j = idx - b * H;
    T* ar = a + b * 3 * H;
    const T* hr = hw + b * 3 * H;
    const T r = sigm(ar[j] + hr[j]);
    const T u = sigm(ar[H + j] + hr[H + j]);
    const T bn = hr[2 * H + j];
    const T n = dev_tanh<T>(ar[2 * H + j] + r * bn);
    ar[j] = r;
    ar[H + j] = u;
    ar[2 * H + j] = n;
    hn_t[idx] = bn;
    out_t[idx] = (h_prev[idx] - n) * u + n;
  }
}

// One reverse step: dh = dh_buf + g_t; dz_ih = (dr, du, dn), dz_hh = (dr, du, dn r);
// dh_buf becomes dh u (the recurrent product is added by the GEMM that follows).
template <typename T>
__global__ void __launch_bounds__(kThreads)
gru_cell_bwd(const T* __restrict__ gates, const T* __restrict__ hn_t,
             const T* __restrict__ h_prev, const T* __restrict__ g_t, T* __restrict__ dh_buf,
             T* __restrict__ dz_ih, T* __restrict__ dz_hh, int64_t B, int64_t H, int first) {
  const int64_t total = B * H;
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = idx / H, j = idx - b * H;
    const T* a = gates + b * 3 * H;
    const T r = a[j], u = a[H + j], n = a[2 * H + j];
    const T dh = first ? g_t[idx] : dh_buf[idx] + g_t[idx];
    const T dn = dh * (T(1) - u) * (T(1) - n * n);
    const T du = dh * (h_prev[idx] - n) * (u * (T(1) - u));
    const T dr = dn * hn_t[idx] * (r * (T(1) - r));
    T* di = dz_ih + b * 3 * H;
    T* dr_ = dz_hh + b * 3 * H;
    di[j] = dr;
    di[H + j] = du;
    di[2 * H + j] = dn;
    dr_[j] = dr;
    dr_[H + j] = du;
    dr_[2 * H + j] = dn * r;
    dh_buf[idx] = dh * u;
  }
}

// ------------------------------------------------------------------ Elman cells
// z (B, H) holds x W_ih^T + b_ih and becomes the state act(z + h W_hh^T + b_hh).
template <typename T>
__global__ void __launch_bounds__(kThreads)
rnn_cell_fwd(T* __restrict__ z, const T* __restrict__ rec, int64_t n, int relu) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const T v = z[idx] + rec[idx];
    z[idx] = relu ? (v > T(0) ? v : T(0)) : dev_tanh<T>(v);
  }
}

// One reverse step: dh = g_t (+ the carry dz_{t+1} W_hh), dz_t = dh act'(h_t) with
// act' = 1 - h^2 (tanh) or [h > 0] (relu).
template <typename T>
__global__ void __launch_bounds__(kThreads)
rnn_cell_bwd(const T* __restrict__ h_t, const T* __restrict__ g_t, const T* __restrict__ carry,
             T* __restrict__ dz_t, int64_t n, int relu, int first) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const T dh = first ? g_t[idx] : carry[idx] + g_t[idx];
    const T h = h_t[idx];
    dz_t[idx] = relu ? (h > T(0) ? dh : T(0)) : dh * (T(1) - h * h);
  }
}

template <typename T>
GemmArgs<T> gemm_args(int ta, int tb, int64_t m, int64_t n, int64_t k, const T* a, int64_t lda,
                      const T* b, int64_t ldb, T* c, int64_t ldc, const T* bias, T beta) {
  GemmArgs<T> p{};
  p.m = m; p.n = n; p.k = k;
  p.a = a; p.lda = lda; p.b = b; p.ldb = ldb; p.c = c; p.ldc = ldc;
  p.bias = bias; p.alpha = T(1); p.beta = beta;
  p.trans_a = ta; p.trans_b = tb; p.batch = 1;
  return p;
}

// Split-K partials of the per-step recurrent GEMMs and of the weight gradients.
constexpr size_t kWorkspaceFloats = 4u << 20;  // 16 MiB

struct RnnBwdLayout {
  size_t dz, dz2, carry, carry2, xpad, colsum, ws, total;
};

RnnBwdLayout rnn_bwd_layout(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H, int gates,
                            bool two_dz) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const int64_t rows = T_ * B, G = gates * H;
  RnnBwdLayout L{};
  L.dz = align256((size_t)(rows * G) * es);
  L.dz2 = two_dz ? L.dz : 0;
  L.carry = align256((size_t)(B * H) * es);
  L.carry2 = L.carry;
  L.xpad = (I % 4) ? align256((size_t)(rows * ((I + 3) / 4 * 4)) * es) : 0;
  L.colsum = align256((size_t)colsum_chunks(rows, G) * (size_t)G * es);
  L.ws = dtype == TG_F32 ? kWorkspaceFloats * sizeof(float) : 0;
  L.total = L.dz + L.dz2 + L.carry + L.carry2 + L.xpad + L.colsum + L.ws;
  return L;
}

// Forward scratch: the summed biases (LSTM) or h W_hn + b_hn (GRU), then (fp32) a split-K
// workspace for the per-step recurrent products, whose outputs (batch x gates) have few tiles.
size_t fwd_ws_offset(int dtype, size_t head) { return dtype == TG_F32 ? align256(head) : 0; }
size_t fwd_ws_bytes(int dtype) { return dtype == TG_F32 ? kWorkspaceFloats * sizeof(float) : 0; }

int check_rnn(int64_t T_, int64_t B, int64_t I, int64_t H) {
  TG_CHECK_ARG(T_ > 0 && B > 0 && I > 0 && H > 0, "rnn: empty sequence or sizes");
  return TG_OK;
}

// Weight gradients shared by both cells: dW_ih = dz^T x, dW_hh = dz_hh^T h_prev with
// h_prev = (h0, h_1 .. h_{T-1}) (rows of `hs` at row stride hs_ld), db = column sums, and
// dx = dz W_ih.
template <typename T>
int rnn_weight_grads(int64_t T_, int64_t B, int64_t I, int64_t H, int gates, const T* dz,
                     const T* dz_hh, const T* x, const T* h0, const T* hs, int64_t hs_ld,
                     const T* w_ih, T* dx, T* dw_ih, T* dw_hh, T* db_ih, T* db_hh,
                     const RnnBwdLayout& L, uint8_t* base, cudaStream_t st) {
  const int64_t rows = T_ * B, G = gates * H;
  uint8_t* p = base + L.dz + L.dz2 + L.carry + L.carry2;
  T* xpad = reinterpret_cast<T*>(p);
  p += L.xpad;
  void* cs = p;
  p += L.colsum;
  float* ws = reinterpret_cast<float*>(p);
  int r;
  if (dw_ih) {
    const T* xb = x;
    int64_t ldx = I;
    if (I % 4) {
      ldx = (I + 3) / 4 * 4;
      pad_cols_kernel<T><<<grid_for(rows * ldx, kThreads), kThreads, 0, st>>>(x, xpad, rows, I,
                                                                              ldx);
      if ((r = check_launch("rnn backward(pad x)"))) return r;
      xb = xpad;
    }
    auto q = gemm_args<T>(1, 0, G, I, rows, dz, G, xb, ldx, dw_ih, I, nullptr, T(0));
    if (L.ws) { q.workspace = ws; q.workspace_bytes = L.ws; }
    if ((r = gemm_run<T>(q, st))) return r;
  }
  if (dw_hh) {
    T beta = T(0);
    if (T_ > 1) {
      auto q = gemm_args<T>(1, 0, G, H, (T_ - 1) * B, dz_hh + B * G, G, hs, hs_ld, dw_hh, H,
                            nullptr, T(0));
      if (L.ws) { q.workspace = ws; q.workspace_bytes = L.ws; }
      if ((r = gemm_run<T>(q, st))) return r;
      beta = T(1);
    }
    auto q = gemm_args<T>(1, 0, G, H, B, dz_hh, G, h0, H, dw_hh, H, nullptr, beta);
    if ((r = gemm_run<T>(q, st))) return r;
  }
  if (db_ih) {
    if ((r = colsum<T>(dz, db_ih, rows, G, 0, cs, st))) return r;
  }
  if (db_hh) {
    if ((r = colsum<T>(dz_hh, db_hh, rows, G, 0, cs, st))) return r;
  }
  if (dx) {
    auto q = gemm_args<T>(0, 0, rows, I, G, dz, G, w_ih, I, dx, I, nullptr, T(0));
    if ((r = gemm_run<T>(q, st))) return r;
  }
  return TG_OK;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

// Scratch of the LSTM forward: the summed biases (4H), the step's recurrent product
// h W_hh^T (B x 4H, written with beta = 0 so the GEMM stores whole tiles through TMA; the
// cell kernel adds the input projection), then the GEMM's split workspace.
static size_t lstm_fwd_head(size_t es, int64_t B, int64_t H) {
  return align256((size_t)(4 * H) * es) + align256((size_t)(B * 4 * H) * es);
}

size_t tg_lstm_forward_scratch_bytes(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H) {
  (void)T_; (void)I;
  const size_t es = dtype == TG_F64 ? 8 : 4;
  const size_t head = lstm_fwd_head(es, B, H);
  return head + fwd_ws_bytes(dtype);  // head is a multiple of 256 bytes
}

int tg_lstm_forward(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H, const void* x,
                    const void* h0, const void* c0, const void* w_ih, const void* w_hh,
                    const void* b_ih, const void* b_hh, void* acts, void* out, void* tanh_c,
                    void* scratch, void* stream) {
  int rc = check_rnn(T_, B, I, H);
  if (rc) return rc;
  TG_CHECK_ARG((b_ih == nullptr) == (b_hh == nullptr), "lstm: pass both biases or neither");
  TG_CHECK_ARG(scratch, "lstm: scratch required");
  cudaStream_t st = as_stream(stream);
  const int64_t G = 4 * H;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* bsum = nullptr;
    int r;
    if (b_ih) {
      bsum = reinterpret_cast<T*>(scratch);
      add_vec_kernel<T><<<grid_for(G, kThreads), kThreads, 0, st>>>((const T*)b_ih,
                                                                    (const T*)b_hh, bsum, G);
      if ((r = check_launch("lstm(bias)"))) return r;
    }
    T* z = (T*)acts;
    T* o = (T*)out;
    auto proj = gemm_args<T>(0, 1, T_ * B, G, I, (const T*)x, I, (const T*)w_ih, I, z, G, bsum,
                             T(0));
    if ((r = gemm_run<T>(proj, st))) return r;
    for (int64_t t = 0; t < T_; ++t) {
      const T* h_prev = t == 0 ? (const T*)h0 : o + (t - 1) * B * 2 * H;
      const int64_t h_ld = t == 0 ? H : 2 * H;
      const T* c_prev = t == 0 ? (const T*)c0 : o + (t - 1) * B * 2 * H + H;
      const int64_t c_ld = t == 0 ? H : 2 * H;
      T* zt = z + t * B * G;
      T* rb = reinterpret_cast<T*>((uint8_t*)scratch + align256((size_t)G * sizeof(T)));
      auto rec = gemm_args<T>(0, 1, B, G, H, h_prev, h_ld, (const T*)w_hh, H, rb, G, nullptr,
                              T(0));
      if (fwd_ws_bytes(dtype)) {
        rec.workspace = reinterpret_cast<float*>(
            (uint8_t*)scratch + fwd_ws_offset(dtype, lstm_fwd_head(sizeof(T), B, H)));
        rec.workspace_bytes = fwd_ws_bytes(dtype);
      }
      if ((r = gemm_run<T>(rec, st))) return r;
      launch_pdl(lstm_cell_fwd<T>, dim3(grid_for(B * H, kThreads)), dim3(kThreads), 0, st, zt,
                 rb, c_prev, c_ld, o + t * B * 2 * H, (T*)tanh_c + t * B * H, B, H);
      if ((r = check_launch("lstm(cell)"))) return r;
    }
    return (int)TG_OK;
  });
}

size_t tg_lstm_backward_scratch_bytes(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H) {
  return rnn_bwd_layout(dtype, T_, B, I, H, 4, false).total;
}

int tg_lstm_backward(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H, const void* g,
                     const void* x, const void* h0, const void* c0, const void* w_ih,
                     const void* w_hh, const void* acts, const void* out, const void* tanh_c,
                     void* dx, void* dh0, void* dc0, void* dw_ih, void* dw_hh, void* db_ih,
                     void* db_hh, void* scratch, void* stream) {
  int rc = check_rnn(T_, B, I, H);
  if (rc) return rc;
  TG_CHECK_ARG(scratch && g, "lstm backward: scratch and g required");
  cudaStream_t st = as_stream(stream);
  const int64_t G = 4 * H;
  const RnnBwdLayout L = rnn_bwd_layout(dtype, T_, B, I, H, 4, false);
  uint8_t* base = (uint8_t*)scratch;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* dz = reinterpret_cast<T*>(base);
    T* dh = reinterpret_cast<T*>(base + L.dz + L.dz2);
    T* dc = reinterpret_cast<T*>(base + L.dz + L.dz2 + L.carry);
    float* ws = reinterpret_cast<float*>(base + L.total - L.ws);
    const T* o = (const T*)out;
    int r;
    for (int64_t t = T_ - 1; t >= 0; --t) {
      const T* c_prev = t == 0 ? (const T*)c0 : o + (t - 1) * B * 2 * H + H;
      const int64_t c_ld = t == 0 ? H : 2 * H;
      T* dzt = dz + t * B * G;
      launch_pdl(lstm_cell_bwd<T>, dim3(grid_for(B * H, kThreads)), dim3(kThreads), 0, st,
          (const T*)acts + t * B * G, (const T*)tanh_c + t * B * H, c_prev, c_ld,
          (const T*)g + t * B * 2 * H, dh, dc, dzt, B, H, t == T_ - 1);
      if ((r = check_launch("lstm backward(cell)"))) return r;
      if (t > 0 || dh0) {
        T* dst = t > 0 ? dh : (T*)dh0;
        auto q = gemm_args<T>(0, 0, B, H, G, dzt, G, (const T*)w_hh, H, dst, H, nullptr, T(0));
        if (L.ws) { q.workspace = ws; q.workspace_bytes = L.ws; }
        if ((r = gemm_run<T>(q, st))) return r;
      }
    }
    if (dc0) {
      TG_CUDA_TRY(cudaMemcpyAsync(dc0, dc, (size_t)(B * H) * sizeof(T), cudaMemcpyDeviceToDevice, st));
    }
    return rnn_weight_grads<T>(T_, B, I, H, 4, dz, dz, (const T*)x, (const T*)h0, o, 2 * H,
                               (const T*)w_ih, (T*)dx, (T*)dw_ih, (T*)dw_hh, (T*)db_ih,
                               (T*)db_hh, L, base, st);
  });
}

size_t tg_gru_forward_scratch_bytes(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H) {
  (void)T_; (void)I;
  const size_t es = dtype == TG_F64 ? 8 : 4;
  return align256((size_t)(B * 3 * H) * es) + fwd_ws_bytes(dtype);
}

int tg_gru_forward(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H, const void* x,
                   const void* h0, const void* w_ih, const void* w_hh, const void* b_ih,
                   const void* b_hh, void* acts, void* hn, void* out, void* scratch,
                   void* stream) {
  int rc = check_rnn(T_, B, I, H);
  if (rc) return rc;
  TG_CHECK_ARG((b_ih == nullptr) == (b_hh == nullptr), "gru: pass both biases or neither");
  TG_CHECK_ARG(scratch, "gru: scratch required");
  cudaStream_t st = as_stream(stream);
  const int64_t G = 3 * H;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* hw = reinterpret_cast<T*>(scratch);
    T* a = (T*)acts;
    T* o = (T*)out;
    int r;
    auto proj = gemm_args<T>(0, 1, T_ * B, G, I, (const T*)x, I, (const T*)w_ih, I, a, G,
                             (const T*)b_ih, T(0));
    if ((r = gemm_run<T>(proj, st))) return r;
    for (int64_t t = 0; t < T_; ++t) {
      const T* h_prev = t == 0 ? (const T*)h0 : o + (t - 1) * B * H;
      auto rec = gemm_args<T>(0, 1, B, G, H, h_prev, H, (const T*)w_hh, H, hw, G,
                              (const T*)b_hh, T(0));
      if (fwd_ws_bytes(dtype)) {
        rec.workspace = reinterpret_cast<float*>(
            (uint8_t*)scratch + fwd_ws_offset(dtype, align256((size_t)(B * G) * sizeof(T))));
        rec.workspace_bytes = fwd_ws_bytes(dtype);
      }
      if ((r = gemm_run<T>(rec, st))) return r;
      launch_pdl(gru_cell_fwd<T>, dim3(grid_for(B * H, kThreads)), dim3(kThreads), 0, st,
          a + t * B * G, hw, h_prev, (T*)hn + t * B * H, o + t * B * H, B, H);
      if ((r = check_launch("gru(cell)"))) return r;
    }
    return (int)TG_OK;
  });
}

size_t tg_gru_backward_scratch_bytes(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H) {
  return rnn_bwd_layout(dtype, T_, B, I, H, 3, true).total;
}

int tg_gru_backward(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H, const void* g,
                    const void* x, const void* h0, const void* w_ih, const void* w_hh,
                    const void* acts, const void* hn, const void* out, void* dx, void* dh0,
                    void* dw_ih, void* dw_hh, void* db_ih, void* db_hh, void* scratch,
                    void* stream) {
  int rc = check_rnn(T_, B, I, H);
  if (rc) return rc;
  TG_CHECK_ARG(scratch && g, "gru backward: scratch and g required");
  cudaStream_t st = as_stream(stream);
  const int64_t G = 3 * H;
  const RnnBwdLayout L = rnn_bwd_layout(dtype, T_, B, I, H, 3, true);
  uint8_t* base = (uint8_t*)scratch;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* dz_ih = reinterpret_cast<T*>(base);
    T* dz_hh = reinterpret_cast<T*>(base + L.dz);
    T* dh = reinterpret_cast<T*>(base + L.dz + L.dz2);
    float* ws = reinterpret_cast<float*>(base + L.total - L.ws);
    const T* o = (const T*)out;
    int r;
    for (int64_t t = T_ - 1; t >= 0; --t) {
      const T* h_prev = t == 0 ? (const T*)h0 : o + (t - 1) * B * H;
      launch_pdl(gru_cell_bwd<T>, dim3(grid_for(B * H, kThreads)), dim3(kThreads), 0, st,
          (const T*)acts + t * B * G, (const T*)hn + t * B * H, h_prev, (const T*)g + t * B * H,
          dh, dz_ih + t * B * G, dz_hh + t * B * G, B, H, t == T_ - 1);
      if ((r = check_launch("gru backward(cell)"))) return r;
      if (t > 0 || dh0) {
        auto q = gemm_args<T>(0, 0, B, H, G, dz_hh + t * B * G, G, (const T*)w_hh, H, dh, H,
                              nullptr, T(1));
        if (L.ws) { q.workspace = ws; q.workspace_bytes = L.ws; }
        if ((r = gemm_run<T>(q, st))) return r;
      }
    }
    if (dh0) {
      TG_CUDA_TRY(cudaMemcpyAsync(dh0, dh, (size_t)(B * H) * sizeof(T), cudaMemcpyDeviceToDevice, st));
    }
    return rnn_weight_grads<T>(T_, B, I, H, 3, dz_ih, dz_hh, (const T*)x, (const T*)h0, o, H,
                               (const T*)w_ih, (T*)dx, (T*)dw_ih, (T*)dw_hh, (T*)db_ih,
                               (T*)db_hh, L, base, st);
  });
}

size_t tg_rnn_forward_scratch_bytes(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H) {
  (void)T_; (void)I;
  const size_t es = dtype == TG_F64 ? 8 : 4;
  return align256((size_t)(B * H) * es) + fwd_ws_bytes(dtype);
}

int tg_rnn_forward(int dtype, int relu, int64_t T_, int64_t B, int64_t I, int64_t H,
                   const void* x, const void* h0, const void* w_ih, const void* w_hh,
                   const void* b_ih, const void* b_hh, void* out, void* scratch, void* stream) {
  int rc = check_rnn(T_, B, I, H);
  if (rc) return rc;
  TG_CHECK_ARG((b_ih == nullptr) == (b_hh == nullptr), "rnn: pass both biases or neither");
  TG_CHECK_ARG(scratch, "rnn: scratch required");
  cudaStream_t st = as_stream(stream);
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* hw = reinterpret_cast<T*>(scratch);
    T* o = (T*)out;
    int r;
    auto proj = gemm_args<T>(0, 1, T_ * B, H, I, (const T*)x, I, (const T*)w_ih, I, o, H,
                             (const T*)b_ih, T(0));
    if ((r = gemm_run<T>(proj, st))) return r;
    for (int64_t t = 0; t < T_; ++t) {
      const T* h_prev = t == 0 ? (const T*)h0 : o + (t - 1) * B * H;
      auto rec = gemm_args<T>(0, 1, B, H, H, h_prev, H, (const T*)w_hh, H, hw, H,
                              (const T*)b_hh, T(0));
      if (fwd_ws_bytes(dtype)) {
        rec.workspace = reinterpret_cast<float*>(
            (uint8_t*)scratch + fwd_ws_offset(dtype, align256((size_t)(B * H) * sizeof(T))));
        rec.workspace_bytes = fwd_ws_bytes(dtype);
      }
      if ((r = gemm_run<T>(rec, st))) return r;
      launch_pdl(rnn_cell_fwd<T>, dim3(grid_for(B * H, kThreads)), dim3(kThreads), 0, st,
                 o + t * B * H, (const T*)hw, B * H, relu);
      if ((r = check_launch("rnn(cell)"))) return r;
    }
    return (int)TG_OK;
  });
}

size_t tg_rnn_backward_scratch_bytes(int dtype, int64_t T_, int64_t B, int64_t I, int64_t H) {
  return rnn_bwd_layout(dtype, T_, B, I, H, 1, false).total;
}

int tg_rnn_backward(int dtype, int relu, int64_t T_, int64_t B, int64_t I, int64_t H,
                    const void* g, const void* x, const void* h0, const void* w_ih,
                    const void* w_hh, const void* out, void* dx, void* dh0, void* dw_ih,
                    void* dw_hh, void* db_ih, void* db_hh, void* scratch, void* stream) {
  int rc = check_rnn(T_, B, I, H);
  if (rc) return rc;
  TG_CHECK_ARG(scratch && g, "rnn backward: scratch and g required");
  cudaStream_t st = as_stream(stream);
  const RnnBwdLayout L = rnn_bwd_layout(dtype, T_, B, I, H, 1, false);
  uint8_t* base = (uint8_t*)scratch;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    T* dz = reinterpret_cast<T*>(base);
    T* carry = reinterpret_cast<T*>(base + L.dz + L.dz2);
    float* ws = reinterpret_cast<float*>(base + L.total - L.ws);
    const T* o = (const T*)out;
    int r;
    for (int64_t t = T_ - 1; t >= 0; --t) {
      launch_pdl(rnn_cell_bwd<T>, dim3(grid_for(B * H, kThreads)), dim3(kThreads), 0, st,
                 o + t * B * H, (const T*)g + t * B * H, (const T*)carry, dz + t * B * H,
                 B * H, relu, t == T_ - 1);
      if ((r = check_launch("rnn backward(cell)"))) return r;
      if (t > 0 || dh0) {
        auto q = gemm_args<T>(0, 0, B, H, H, dz + t * B * H, H, (const T*)w_hh, H, carry, H,
                              nullptr, T(0));
        if (L.ws) { q.workspace = ws; q.workspace_bytes = L.ws; }
        if ((r = gemm_run<T>(q, st))) return r;
      }
    }
    if (dh0) {
      TG_CUDA_TRY(cudaMemcpyAsync(dh0, carry, (size_t)(B * H) * sizeof(T),
                                  cudaMemcpyDeviceToDevice, st));
    }
    return rnn_weight_grads<T>(T_, B, I, H, 1, dz, dz, (const T*)x, (const T*)h0, o, H,
                               (const T*)w_ih, (T*)dx, (T*)dw_ih, (T*)dw_hh, (T*)db_ih,
                               (T*)db_hh, L, base, st);
  });
}

}  // extern "C"
