/*
 * tgb200.h -- C ABI of libtgb200.so, the sm_100a kernels behind tensorgrad_b200.
 *
 * The reference tensorgrad computes every op of the training step with NumPy/OpenBLAS inside
 * its Python VJP closures; it has no FFI of its own. This header is the boundary that
 * replaces those NumPy bodies: each entry point names the reference function (file:line in
 * the tensorgrad 0.2.0 project) whose arithmetic it performs. Signatures use plain device
 * pointers, element counts and a CUDA stream passed as `void*` (NULL = legacy default
 * stream); no framework types cross the boundary. Every call is asynchronous on `stream`
 * unless stated otherwise, and returns a status code (TG_OK = 0). tg_last_error() gives the
 * detail of the last failure on the calling host thread.
 *
 * Layouts: all matrices are row-major. `dtype` is TG_F32 or TG_F64 (the float64 build mode);
 * integer ids/targets are int64.
 */
#ifndef TGB200_H
#define TGB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status and dtypes */
enum tg_status {
  TG_OK = 0,
  TG_ERR_ARG = 1,         /* invalid argument (maps to ValueError in the host wrappers) */
  TG_ERR_CUDA = 2,        /* a CUDA runtime/launch error */
  TG_ERR_UNSUPPORTED = 3, /* shape/dtype combination not supported */
  TG_ERR_INDEX = 4,       /* id/target out of range (maps to IndexError) */
  TG_ERR_TIMEOUT = 5,     /* a bounded device-side wait, or a collective, ran out of time */
  TG_ERR_OOM = 6,         /* device memory exhausted */
  TG_ERR_COMM = 7         /* a collective failed (the communicator reported an error) */
};
enum tg_dtype { TG_F32 = 0, TG_F64 = 1, TG_I64 = 2 /* casts only */ };

/* Library version (major * 10000 + minor * 100 + patch). */
int tg_version(void);
/* Static text for a status code. */
const char* tg_status_string(int status);
/* Copies the detail message of the calling thread's last failure into buf (NUL-terminated). */
int tg_last_error(char* buf, size_t len);
/* SM count and compute capability of `device`. */
int tg_device_info(int device, int* sm_count, int* cc_major, int* cc_minor);

/* ------------------------------------------------------------------ memory and devices
 * The reference keeps every array in host NumPy memory (no allocator of its own). Device
 * buffers here come from the stream-ordered allocator: tg_malloc / tg_free order the
 * allocation and the release on `stream`, and each device's pool keeps freed memory for reuse
 * (no cudaMalloc once a step's working set has been seen). tg_host_alloc gives page-locked
 * host memory (uploads from it run as asynchronous DMA). Events are timing-free. */
int tg_malloc(void** ptr, size_t bytes, void* stream);
int tg_free(void* ptr, void* stream);
int tg_pool_stats(int device, uint64_t* reserved_bytes, uint64_t* used_bytes);
/* High-water mark of the pool's bytes in use since the last reset (then reset when `reset`
 * is nonzero): the device counterpart of the host peak the reference's gradient-checkpointing
 * tests take with tracemalloc (tests/test_checkpoint.py:116-131). */
int tg_pool_peak(int device, int reset, uint64_t* used_high_bytes);
int tg_host_alloc(void** ptr, size_t bytes);
int tg_host_free(void* ptr);
int tg_set_device(int device);
int tg_get_device(int* device);
/* Visible CUDA devices (0 when there is no driver or device; never an error). */
int tg_device_count(int* count);
int tg_event_create(void** event);
int tg_event_record(void* event, void* stream);
/* 1 once the work before the event has completed, 0 if not yet, < 0 on error. */
int tg_event_query(void* event);
int tg_event_destroy(void* event);

/* ------------------------------------------------------------------ memory movement
 * The reference keeps every array in host memory; these move tensor storage and inputs
 * (token ids, targets, upstream gradients) between host and device. */
int tg_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int tg_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int tg_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int tg_memset_zero(void* dst, size_t bytes, void* stream);
int tg_stream_synchronize(void* stream);

/* ------------------------------------------------------------------ GEMM
 * C[m,n] = alpha * op(A)[m,k] @ op(B)[k,n] + beta * C (+ bias[n]); BLAS-like, row-major.
 *   trans_a = 0: A is m x k (lda >= k);  trans_a = 1: A is stored k x m (lda >= m).
 *   trans_b = 0: B is k x n (ldb >= n);  trans_b = 1: B is stored n x k (ldb >= k).
 * beta = 0 never reads C. fp32 runs on the tcgen05 tensor cores with a 3xTF32 split
 * (fp32-level accuracy) when strides are 16-byte aligned, otherwise on the SIMT path;
 * fp64 runs on the SIMT path. Replaces the `@` products of ops/layers.py:34-49 and
 * ops/linalg.py:16-63. */
int tg_gemm(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, double alpha,
            const void* a, int64_t lda, const void* b, int64_t ldb, double beta, void* c,
            int64_t ldc, const void* bias, void* stream);
/* Precision of the fp32 tensor-core GEMMs issued through tg_gemm / tg_linear_*: 0 (default)
 * = fp32-accurate 3xTF32; 1 = plain TF32 (one MMA per product, ~2^-11 relative error; fast,
 * outside the 1e-4 parity bar). Process-wide; no reference counterpart. */
int tg_set_matmul_precision(int precision);
/* Same, forcing the SIMT (CUDA-core) kernel: the accuracy reference for tg_gemm. */
int tg_gemm_simt(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                 double alpha, const void* a, int64_t lda, const void* b, int64_t ldb,
                 double beta, void* c, int64_t ldc, const void* bias, void* stream);
/* Live timing of the tensor-core GEMM (measurement support, no reference counterpart):
 * tg_gemm_profile(1) brackets every following tensor-core launch with CUDA events on its
 * stream; tg_gemm_profile_read() waits for them and returns the summed device time (ms),
 * the launch count and the algorithmic FLOPs (2 m n k per launch), then clears the record. */
int tg_gemm_profile(int enable);
int tg_gemm_profile_read(double* total_ms, int64_t* launches, double* flops);
/* Kernels launched by this library since load (every entry point counts its own). */
uint64_t tg_launch_count(void);
/* fp32 products since load that the tensor-core kernel could not take (an operand or a
 * stride off a 16-byte boundary) and that ran on the CUDA-core kernel instead. Reductions of
 * at most 8 always run on the CUDA cores (a memory-bound outer product) and are not counted. */
uint64_t tg_gemm_fallback_count(void);
/* Reads (and with reset != 0 clears) the tensor-core GEMM's device status word: TG_OK, or
 * TG_ERR_TIMEOUT when a bounded pipeline wait gave up. Synchronous. */
int tg_gemm_tc_status(int reset);
/* The same record for the fused attention kernels (forward; P and dS of the backward). */
int tg_attention_tc_status(int reset);
/* Test support for those bounded waits (no reference counterpart): budget_cycles sets the
 * cycle budget of every wait in the fused attention kernels (<= 0 restores the default,
 * about two seconds); withhold_loads != 0 makes the forward's producer issue no load, so its
 * first wait on a load runs out, TG_ERR_TIMEOUT is recorded and the kernel drains and
 * returns with nothing in flight. Synchronous. */
int tg_attention_set_wait_test(int64_t budget_cycles, int withhold_loads);
/* Test support (no reference counterpart): y[i] = the fp32 exponential the fused attention
 * kernels compute on the FMA pipe for part of their softmax numerators (range reduction plus
 * a fitted polynomial; see csrc/expfma.cuh), so a test can bound its error. */
int tg_test_exp_fma(int64_t n, const float* x, float* y, void* stream);
/* Strided-batched GEMM: `batch` products at element offsets i*stride_{a,b,c}. */
int tg_gemm_batched(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                    double alpha, const void* a, int64_t lda, int64_t stride_a, const void* b,
                    int64_t ldb, int64_t stride_b, double beta, void* c, int64_t ldc,
                    int64_t stride_c, int64_t batch, void* stream);

/* linear (ops/layers.py:22-62): y[rows,out] = x[rows,in] @ w[out,in]^T + bias. `scratch`
 * (tg_linear_forward_scratch_bytes, may be NULL) holds split-K partials for outputs with few
 * tiles and a long reduction; the partials are summed in a fixed order (deterministic). */
size_t tg_linear_forward_scratch_bytes(int dtype, int64_t rows, int64_t in_features,
                                       int64_t out_features);
int tg_linear_forward(int dtype, const void* x, const void* w, const void* bias, void* y,
                      int64_t rows, int64_t in_features, int64_t out_features, void* scratch,
                      void* stream);
/* linear VJP (ops/layers.py:43-49): gx = g @ w, gw = g^T @ x (+ beta_gw * gw), gb = colsum(g).
 * need bit 0 = gx, bit 1 = gw, bit 2 = gb (unset bits skip the launch). beta_gw = 1
 * accumulates into an existing gw (tied weights). `scratch` holds
 * tg_linear_backward_scratch_bytes(dtype, rows, in, out, need) bytes: the column-sum partials
 * and a workspace that lets the fp32 products split their reduction over more CTAs (e.g. the
 * vocabulary-wide head, whose 192 output tiles would leave the second wave of 148 SMs mostly
 * idle). It may be NULL when bit 2 is clear; the products then run unsplit. */
size_t tg_linear_backward_scratch_bytes(int dtype, int64_t rows, int64_t in_features,
                                        int64_t out_features, unsigned need);
int tg_linear_backward(int dtype, const void* g, const void* x, const void* w, void* gx, void* gw,
                       void* gb, int64_t rows, int64_t in_features, int64_t out_features,
                       unsigned need, double beta_gw, void* scratch, void* stream);

/* ------------------------------------------------------------------ reductions
 * out[c] = (accumulate ? out[c] : 0) + sum_r x[r, c]: the bias-gradient / unbroadcast
 * column sum (ops/_util.py:49-63, ops/layers.py:49). Deterministic two-pass reduction
 * through `scratch` (tg_colsum_scratch_bytes bytes). */
size_t tg_colsum_scratch_bytes(int dtype, int64_t rows, int64_t cols);
int tg_colsum(int dtype, const void* x, void* out, int64_t rows, int64_t cols, int accumulate,
              void* scratch, void* stream);
/* General sum of a contiguous tensor of shape in_shape[ndim] down to keep-mask axes
 * (keep[i] = 1 keeps axis i, 0 sums it); out is contiguous over the kept axes.
 * The adjoint of broadcasting (ops/_util.py:49-63) and reduce.sum (ops/reduce.py). */
int tg_reduce_sum(int dtype, int ndim, const int64_t* in_shape, const int* keep, const void* x,
                  void* out, void* stream);
/* out[0] = sum of all n elements (float64 accumulation; deterministic). reduce.sum / mean
 * over all axes (ops/reduce.py). `scratch` holds tg_sum_all_scratch_bytes() bytes. */
size_t tg_sum_all_scratch_bytes(void);
int tg_sum_all(int dtype, const void* x, void* out, int64_t n, void* scratch, void* stream);

/* ------------------------------------------------------------------ elementwise
 * Broadcast binary op: out (contiguous, shape[ndim]) = a op b, with a/b read through element
 * strides (0 on broadcast axes). ops/elementwise.py:43-121. op: */
enum tg_binary_op { TG_ADD = 0, TG_SUB = 1, TG_MUL = 2, TG_DIV = 3, TG_POW = 4,
                    TG_EQ = 5 /* 1 where a == b, else 0 (the extrema's tie masks) */ };
int tg_binary(int dtype, int op, int ndim, const int64_t* shape, const void* a,
              const int64_t* a_strides, const void* b, const int64_t* b_strides, void* out,
              void* stream);
/* out = alpha * x + beta * y over n contiguous elements (y may be NULL when beta = 0). */
int tg_axpby(int dtype, int64_t n, double alpha, const void* x, double beta, const void* y,
             void* out, void* stream);
/* out = alpha * x * (*scale_dev) (scale read on the device; used for upstream scalars). */
int tg_scale_by_device_scalar(int dtype, int64_t n, const void* x, const void* scale_dev,
                              double alpha, void* out, void* stream);
/* Unary ops: out = f(x). ops/elementwise.py:133-268. */
enum tg_unary_op {
  TG_NEG = 0, TG_EXP = 1, TG_LOG = 2, TG_SQRT = 3, TG_TANH = 4, TG_SIGMOID = 5, TG_RELU = 6,
  TG_SQUARE = 7, TG_FILL = 8 /* out = alpha */, TG_POWS = 9 /* out = x ** alpha */,
  TG_ABS = 10, TG_FINITE_OR_ZERO = 11 /* x where finite, else 0 (softmax's row shift) */,
  TG_LOG1P = 12 /* log(1 + x), accurate for small x (binary cross entropy's softplus) */
};
int tg_unary(int dtype, int op, int64_t n, const void* x, double alpha, void* out, void* stream);
/* out = cond ? a : b with broadcasting (ops/shape.py:290-328, where / masked_fill): `cond`
 * read as != 0, of cond_dtype -1 (one byte per element, NumPy bool), TG_F32, TG_F64 or
 * TG_I64; every operand addressed by its own element strides over the output shape (0 on
 * broadcast axes). */
int tg_where(int dtype, int cond_dtype, int ndim, const int64_t* shape, const void* cond,
             const int64_t* cond_strides, const void* a, const int64_t* a_strides,
             const void* b, const int64_t* b_strides, void* out, void* stream);
/* out (bytes) = a op b with broadcasting, op 0..5 = ==, !=, <, <=, >, >= (Tensor's
 * comparison operators, tensor.py); strides as tg_where's. */
int tg_compare(int dtype, int op, int ndim, const int64_t* shape, const void* a,
               const int64_t* a_strides, const void* b, const int64_t* b_strides, uint8_t* out,
               void* stream);
/* Keep-axis maximum (is_min = 0) or minimum of x over the axes with keep[i] == 0
 * (ops/reduce.py:70-105); a NaN anywhere in a reduced set gives NaN, as np.max does. */
int tg_reduce_extremum(int dtype, int is_min, int ndim, const int64_t* in_shape,
                       const int* keep, const void* x, void* out, void* stream);
/* Tensor.all / any (tensor.py:418-429): one byte per kept element, whether every (any)
 * element of its reduced set is nonzero; x of in_dtype -1 (bytes), TG_F32, TG_F64 or
 * TG_I64. An empty set gives 1 for all and 0 for any. */
int tg_reduce_truth(int in_dtype, int is_all, int ndim, const int64_t* in_shape,
                    const int* keep, const void* x, uint8_t* out, void* stream);
/* Tensor.argmax (tensor.py:431-435): int64 index within the reduced set (row-major over the
 * reduced axes) of its first maximum, a NaN counting as the maximum. */
int tg_argmax(int dtype, int ndim, const int64_t* in_shape, const int* keep, const void* x,
              int64_t* out, void* stream);
/* dtype conversion of n elements (ops/elementwise.py:323-343 astype). */
int tg_cast(int src_dtype, int dst_dtype, int64_t n, const void* src, void* dst, void* stream);
/* dst[idx . dst_strides] = src[idx . src_strides] for every index of shape[ndim] (element
 * strides, elem_bytes in {1, 4, 8}): permute/transpose, slicing, broadcast materialisation and
 * the scatter of getitem's VJP (ops/shape.py:45-235). */
int tg_strided_copy(int elem_bytes, int ndim, const int64_t* shape, const void* src,
                    const int64_t* src_strides, void* dst, const int64_t* dst_strides,
                    void* stream);
/* GELU, tanh approximation (ops/elementwise.py:275-320). */
int tg_gelu_forward(int dtype, int64_t n, const void* x, void* y, void* stream);
int tg_gelu_backward(int dtype, int64_t n, const void* g, const void* x, void* gx, void* stream);
/* ReLU VJP g * (x > 0) (ops/elementwise.py:261-262). */
int tg_relu_backward(int dtype, int64_t n, const void* g, const void* x, void* gx, void* stream);
/* Unary VJPs from the saved input x or output y: op = TG_EXP (g*y), TG_LOG (g/x),
 * TG_SQRT (g/(2y)), TG_TANH (g(1-y^2)), TG_SIGMOID (g y (1-y)), TG_POWS (g a x^(a-1)). */
int tg_unary_backward(int dtype, int op, int64_t n, const void* g, const void* x, const void* y,
                      double alpha, void* gx, void* stream);

/* Inverted dropout (ops/layers.py:235-259; attention weights, ops/attention.py:59-68) with
 * the reference's keep-mask (_random.py:53-70) generated on the device: y[i] = x[i] * m,
 * m = scale if 16-bit word (first_element + i) of the PCG64 stream is >= threshold, else 0.
 * pcg_state = {state_hi, state_lo, inc_hi, inc_lo}: NumPy's PCG64 state before the mask's
 * first draw; word e is bits [16 (e % 4), 16 (e % 4) + 16) of the stream's 64-bit output
 * e / 4 (0-based), exactly as keep_mask views random_raw(). The same call with the same
 * state on the upstream gradient is the VJP. The caller advances its generator past the
 * ceil(n_total / 4) outputs the whole mask consumes. threshold = round(p * 65536). */
int tg_dropout_pcg64(int dtype, int64_t n, const void* x, void* y, const uint64_t* pcg_state,
                     int64_t first_element, uint32_t threshold, double scale, void* stream);

/* ------------------------------------------------------------------ layer norm
 * ops/layers.py:65-141. Per row of `cols`: mean, rstd = 1/sqrt(var + eps) (biased var),
 * y = (x - mean) * rstd * w + b; w/b may be NULL. mean/rstd[rows] are saved for backward. */
int tg_layer_norm_forward(int dtype, const void* x, const void* w, const void* b, void* y,
                          void* mean, void* rstd, int64_t rows, int64_t cols, double eps,
                          void* stream);
/* gx = rstd (gh - mean(gh) - xhat mean(gh xhat)), gh = g w; gw = sum_rows g xhat;
 * gb = sum_rows g. need bit 0 = gx, bit 1 = gw, bit 2 = gb. `scratch` holds
 * tg_layer_norm_scratch_bytes bytes when gw or gb is needed. */
size_t tg_layer_norm_scratch_bytes(int dtype, int64_t rows, int64_t cols);
int tg_layer_norm_backward(int dtype, const void* g, const void* x, const void* w,
                           const void* mean, const void* rstd, void* gx, void* gw, void* gb,
                           int64_t rows, int64_t cols, unsigned need, void* scratch,
                           void* stream);

/* Same as tg_layer_norm_backward, but allocation-free: for callers that cannot allocate
 * device memory (a C or FFI host without a CUDA allocator of its own, or a latency-critical
 * path where a cudaMalloc, which may synchronise the device, is not acceptable). No
 * counterpart in the reference, which allocates its NumPy temporaries freely. The weight/
 * bias partial sums use a file-scope device array of 4 MiB per device instead of `scratch`;
 * a call whose partials need more (tg_layer_norm_scratch_bytes(dtype, rows, cols) > 4 MiB)
 * returns TG_ERR_ARG. The array's device address is looked up on every call made outside
 * stream capture and cached per device; a call on a capturing stream uses the cached
 * address, so a device's first call should come before any stream capture. All calls on a
 * device share its array, so calls that overlap on that GPU (e.g. on two streams) race; each
 * call overwrites every partial it reads, so no clearing is needed between calls. */
int tg_layer_norm_backward_noalloc(int dtype, const void* g, const void* x, const void* w,
                                   const void* mean, const void* rstd, void* gx, void* gw,
                                   void* gb, int64_t rows, int64_t cols, unsigned need,
                                   void* stream);

/* ------------------------------------------------------------------ embedding
 * ops/layers.py:209-232. out[i, :] = w[ids[i], :]. Ids outside [0, num) give a zero row and
 * set *bad_id_dev (int32, may be NULL) to 1: host ids are checked by the caller before the
 * call, as the reference checks them; device-resident ids are checked here and the flag is
 * read back at the caller's next synchronisation. */
int tg_embedding_forward(int dtype, const int64_t* ids, const void* w, void* out, int64_t n,
                         int64_t num, int64_t dim, int* bad_id_dev, void* stream);
/* Scatter-add of gradient rows into gw[num, dim] in the reference's order
 * (ops/layers.py:192-206: stable sort of ids, then a sum per run of equal ids):
 * `order` is the stable argsort of ids, `seg_start[nseg + 1]` the run boundaries in it and
 * `seg_id[nseg]` the id of each run. accumulate = 0 zero-fills gw first. */
int tg_embedding_backward(int dtype, const void* g, const int64_t* order,
                          const int64_t* seg_start, const int64_t* seg_id, int64_t nseg,
                          void* gw, int64_t num, int64_t dim, int accumulate, void* stream);
/* The same order computed on the device, for device-resident ids: tg_embedding_sort writes
 * sorted_keys[n] = the ascending keys id * n + position (unique keys, so this is the stable
 * sort by id; an id outside [0, num) is counted as 0 and sets *bad_id_dev). `scratch`:
 * tg_embedding_sort_scratch_bytes(n, num). tg_embedding_backward_sorted then sums each run of
 * equal ids in ascending position into its row of gw. */
size_t tg_embedding_sort_scratch_bytes(int64_t n, int64_t num);
int tg_embedding_sort(const int64_t* ids, int64_t n, int64_t num, uint64_t* sorted_keys,
                      int* bad_id_dev, void* scratch, size_t scratch_bytes, void* stream);
int tg_embedding_backward_sorted(int dtype, const void* g, const uint64_t* sorted_keys,
                                 int64_t n, void* gw, int64_t num, int64_t dim, int accumulate,
                                 void* stream);

/* ------------------------------------------------------------------ cross entropy
 * ops/loss.py:23-97 with ops/activation.py:48-52 (class axis last). Per row: lse = log sum
 * exp(x), loss_row = lse - x[t] (0 where t == ignore_index). Targets are validated: a target
 * outside [0, classes) that is not ignore_index sets *bad_target_dev (int32) to 1.
 * Per-row losses go to row_loss[rows] (the result itself for reduction 2 = none);
 * reduction 0 = mean over valid rows and 1 = sum write out[0], summed in float64 in row
 * order. n_valid_dev (int64[1], may be NULL for none) receives the valid-row count. */
int tg_cross_entropy_forward(int dtype, const void* logits, const int64_t* targets, void* lse,
                             void* row_loss, void* out, int64_t rows, int64_t classes,
                             int64_t ignore_index, int reduction, int64_t* n_valid_dev,
                             int* bad_target_dev, void* stream);
/* grad = (softmax(x) - onehot(t)) * valid * g_dev[0 or row] / (mean ? n_valid : 1). */
int tg_cross_entropy_backward(int dtype, const void* logits, const int64_t* targets,
                              const void* lse, const void* g_dev, const int64_t* n_valid_dev,
                              void* grad, int64_t rows, int64_t classes, int64_t ignore_index,
                              int reduction, void* stream);

/* ------------------------------------------------------------------ attention
 * Fused causal/non-causal softmax attention (ops/attention.py:71-116, 163-272) as a flash-
 * style kernel: the forward stores O and the row log-sum-exp instead of P; the backward
 * recomputes P. Tensors are (B, H, T, D) viewed through element strides
 * (batch, head, token); the last axis is contiguous. For packed QKV, q/k/v point into one
 * (B, T, 3*H*D) buffer at offsets 0, H*D, 2*H*D with token stride 3*H*D. Causal: key j is
 * visible to query i iff j <= i + (tk - tq). lse is (B, H, tq) contiguous. */
typedef struct tg_attn_shape {
  int64_t batch, heads, tq, tk, head_dim;
  int64_t q_sb, q_sh, q_st; /* strides of q (elements) */
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  int64_t o_sb, o_sh, o_st; /* strides of o / dO (same layout) */
  int causal;
} tg_attn_shape;
/* fp32 with head_dim % 4 == 0 (and, when causal, tq == tk) runs on the tensor cores: batched
 * 3xTF32 tcgen05 GEMMs for the score and value products, causal tiles above the diagonal
 * skipped, softmax in warp-per-row kernels; the scores live in `scratch` for the call only.
 * Other shapes and float64 use flash-style CUDA-core kernels (O and lse only, no scores).
 * `scratch` holds tg_attention_forward_scratch_bytes bytes. */
size_t tg_attention_forward_scratch_bytes(int dtype, const tg_attn_shape* s);
int tg_attention_forward(int dtype, const tg_attn_shape* s, const void* q, const void* k,
                         const void* v, void* o, void* lse, void* scratch, void* stream);
/* dq/dk/dv use the strides of q/k/v; P is recomputed from lse.
 * `scratch` holds tg_attention_backward_scratch_bytes bytes. */
size_t tg_attention_backward_scratch_bytes(int dtype, const tg_attn_shape* s);
int tg_attention_backward(int dtype, const tg_attn_shape* s, const void* q, const void* k,
                          const void* v, const void* o, const void* lse, const void* dout,
                          void* dq, void* dk, void* dv, void* scratch, void* stream);

/* Attention with dropout on the attention weights (ops/attention.py:59-116 with dropout_p >
 * 0 in training): the reference's keep-mask over the whole (B, H, tq, tk) probability array
 * (element ((b H + h) tq + i) tk + j uses 16-bit word of that index of the PCG64 stream whose
 * state before the draw is pcg_state, as tg_dropout_pcg64), regenerated by the VJP rather
 * than stored. Weights W = P * (keep ? keep_scale : 0); O = W V; the VJP is the reference's
 * attention_backward with the mask applied to dW = dO V^T. fp32 and float64; the products
 * are the library's batched GEMMs, the probabilities live in `scratch`
 * (tg_attention_dropout_scratch_bytes, the same for both directions) for the call. */
size_t tg_attention_dropout_scratch_bytes(int dtype, const tg_attn_shape* s);
int tg_attention_forward_dropout(int dtype, const tg_attn_shape* s, const void* q, const void* k,
                                 const void* v, void* o, void* lse, const uint64_t* pcg_state,
                                 uint32_t threshold, double keep_scale, void* scratch,
                                 void* stream);
int tg_attention_backward_dropout(int dtype, const tg_attn_shape* s, const void* q,
                                  const void* k, const void* v, const void* dout, void* dq,
                                  void* dk, void* dv, const uint64_t* pcg_state,
                                  uint32_t threshold, double keep_scale, void* scratch,
                                  void* stream);

/* ------------------------------------------------------------------ convolution / pooling
 * conv2d (ops/conv.py:128-177): cross-correlation of x (n, c, h, w) with w (c_out, c, kh, kw)
 * by an im2col patch matrix `cols` stored patch-major: `rows` x `ld` from
 * tg_conv2d_cols_shape (row kk = channel*kh*kw + i*kw + j, zero rows beyond c*kh*kw; column
 * m = image*oh*ow + pixel; ld >= n*oh*ow, both multiples of 4 so the rows suit the TMA). Then
 * one GEMM per direction: y = cols^T W^T (+ b) written straight to NCHW by the GEMM
 * epilogue; dW = G cols^T with the reduction running over images and pixels of the NCHW
 * gradient; dcols = W^T G per image, folded back onto dx by col2im (a gather,
 * deterministic). `cols` is written by the forward call and read by the backward call (the
 * reference keeps its patch matrix for the weight gradient too, ops/conv.py:91-98,
 * 114-116). Zero padding (ph, pw), strides (sh, sw). */
typedef struct tg_conv_shape {
  int64_t n, c, h, w;      /* input */
  int64_t c_out, kh, kw;   /* filters */
  int64_t sh, sw, ph, pw;  /* stride, zero padding */
  int64_t oh, ow;          /* output: (h + 2 ph - kh) / sh + 1, likewise ow */
} tg_conv_shape;
int tg_conv2d_cols_shape(const tg_conv_shape* s, int64_t* rows, int64_t* ld);
size_t tg_conv2d_forward_scratch_bytes(int dtype, const tg_conv_shape* s);
int tg_conv2d_forward(int dtype, const tg_conv_shape* s, const void* x, const void* w,
                      const void* b, void* y, void* cols, void* scratch, void* stream);
/* The patch matrix alone (what tg_conv2d_forward writes to `cols`): the weight-gradient
 * product as an op of its own, for the differentiable VJPs of conv2d (ops/conv.py:215-250). */
int tg_conv2d_im2col(int dtype, const tg_conv_shape* s, const void* x, void* cols,
                     void* stream);
/* g: (n, c_out, oh, ow). gx / gw / gb may be NULL (not needed). */
size_t tg_conv2d_backward_scratch_bytes(int dtype, const tg_conv_shape* s, int need_gx);
int tg_conv2d_backward(int dtype, const tg_conv_shape* s, const void* g, const void* cols,
                       const void* w, void* gx, void* gw, void* gb, void* scratch, void* stream);

/* Training-mode batch norm over (n, c, hw) (ops/layers.py:144-189; BatchNorm1d/2d): per
 * channel the biased batch mean/variance, y = (x - mean) * rstd * w + b with rstd =
 * 1/sqrt(var + eps); mean and rstd (c) are saved for the VJP; running_mean / running_var (c,
 * may be NULL) become (1 - momentum) r + momentum * stat with the unbiased variance
 * var * m / (m - 1), m = n*hw. w / b may be NULL (no affine). Statistics accumulate in
 * float64. `scratch`: tg_batch_norm_scratch_bytes. */
size_t tg_batch_norm_scratch_bytes(int dtype, int64_t n, int64_t c, int64_t hw);
int tg_batch_norm_forward(int dtype, int64_t n, int64_t c, int64_t hw, const void* x,
                          const void* w, const void* b, void* y, void* mean, void* rstd,
                          void* running_mean, void* running_var, double momentum, double eps,
                          void* scratch, void* stream);
/* The VJP of the composite the reference records: with xhat = (x - mean) rstd,
 * gb = sum g, gw = sum g xhat, gx = rstd w (g - gb/m - xhat gw/m). Any of gx/gw/gb NULL. */
int tg_batch_norm_backward(int dtype, int64_t n, int64_t c, int64_t hw, const void* g,
                           const void* x, const void* w, const void* mean, const void* rstd,
                           void* gx, void* gw, void* gb, void* scratch, void* stream);

/* max_pool2d (ops/conv.py:300-357): -inf padding (ph <= kh/2, pw <= kw/2), first maximum of
 * each window in row-major order wins, a NaN counts as the maximum. The winning cell's
 * window offset (i*kw + j, kh*kw <= 256) is stored in `argmax` (n, c, oh, ow bytes) for the
 * VJP, which sums g into every input cell over the windows that chose it. The struct's
 * c_out is ignored. */
int tg_max_pool2d_forward(int dtype, const tg_conv_shape* s, const void* x, void* y,
                          uint8_t* argmax, void* stream);
int tg_max_pool2d_backward(int dtype, const tg_conv_shape* s, const void* g,
                           const uint8_t* argmax, void* gx, void* stream);
/* The adjoint of the backward: out (n, c, oh, ow) = u (n, c, h, w) at each window's recorded
 * winner (0 for a winner in the padding); the VJP of the VJP (ops/conv.py:340-356). */
int tg_max_pool2d_gather(int dtype, const tg_conv_shape* s, const void* u,
                         const uint8_t* argmax, void* out, void* stream);

/* ------------------------------------------------------------------ recurrent layers
 * ops/recurrent.py:223-437: a whole time-major sequence x (T, B, I) per call; gate order and
 * formulas are the reference's (PyTorch's). W_ih (G*H, I), W_hh (G*H, H), biases (G*H) may
 * both be NULL (not one). Forward: one GEMM projects every step, then per step one
 * recurrent GEMM and one gate kernel. Backward (BPTT): per step in reverse one gate-VJP
 * kernel and one GEMM dh = dz W_hh, then one GEMM per weight and column sums for the biases.
 *
 * LSTM (G = 4, gates i, f, g, o): out (T, B, 2, H) holds h_t and c_t of every step; acts
 * (T, B, 4H) receives the activated gates and tanh_c (T, B, H) tanh(c_t), both kept for the
 * VJP. g is the gradient of out (T, B, 2, H). dx, dh0, dc0, dw_ih, dw_hh, db_ih, db_hh may be
 * NULL (not needed). */
size_t tg_lstm_forward_scratch_bytes(int dtype, int64_t T, int64_t B, int64_t I, int64_t H);
int tg_lstm_forward(int dtype, int64_t T, int64_t B, int64_t I, int64_t H, const void* x,
                    const void* h0, const void* c0, const void* w_ih, const void* w_hh,
                    const void* b_ih, const void* b_hh, void* acts, void* out, void* tanh_c,
                    void* scratch, void* stream);
size_t tg_lstm_backward_scratch_bytes(int dtype, int64_t T, int64_t B, int64_t I, int64_t H);
int tg_lstm_backward(int dtype, int64_t T, int64_t B, int64_t I, int64_t H, const void* g,
                     const void* x, const void* h0, const void* c0, const void* w_ih,
                     const void* w_hh, const void* acts, const void* out, const void* tanh_c,
                     void* dx, void* dh0, void* dc0, void* dw_ih, void* dw_hh, void* db_ih,
                     void* db_hh, void* scratch, void* stream);
/* GRU (G = 3, gates r, u, n; n = tanh(a_n + r (h W_hn^T + b_hn)), h_t = (h - n) u + n):
 * out (T, B, H); acts (T, B, 3H) receives (r, u, n) and hn (T, B, H) the h W_hn^T + b_hn
 * term. g is the gradient of out. */
size_t tg_gru_forward_scratch_bytes(int dtype, int64_t T, int64_t B, int64_t I, int64_t H);
int tg_gru_forward(int dtype, int64_t T, int64_t B, int64_t I, int64_t H, const void* x,
                   const void* h0, const void* w_ih, const void* w_hh, const void* b_ih,
                   const void* b_hh, void* acts, void* hn, void* out, void* scratch,
                   void* stream);
size_t tg_gru_backward_scratch_bytes(int dtype, int64_t T, int64_t B, int64_t I, int64_t H);
int tg_gru_backward(int dtype, int64_t T, int64_t B, int64_t I, int64_t H, const void* g,
                    const void* x, const void* h0, const void* w_ih, const void* w_hh,
                    const void* acts, const void* hn, const void* out, void* dx, void* dh0,
                    void* dw_ih, void* dw_hh, void* db_ih, void* db_hh, void* scratch,
                    void* stream);

/* Elman RNN (ops/recurrent.py:140-219; G = 1): h_t = act(x_t W_ih^T + b_ih + h_{t-1} W_hh^T
 * + b_hh), act = tanh (relu = 0) or max(., 0) (relu = 1); out (T, B, H) holds h_1 .. h_T,
 * which is all the VJP needs. g is the gradient of out. */
size_t tg_rnn_forward_scratch_bytes(int dtype, int64_t T, int64_t B, int64_t I, int64_t H);
int tg_rnn_forward(int dtype, int relu, int64_t T, int64_t B, int64_t I, int64_t H,
                   const void* x, const void* h0, const void* w_ih, const void* w_hh,
                   const void* b_ih, const void* b_hh, void* out, void* scratch, void* stream);
size_t tg_rnn_backward_scratch_bytes(int dtype, int64_t T, int64_t B, int64_t I, int64_t H);
int tg_rnn_backward(int dtype, int relu, int64_t T, int64_t B, int64_t I, int64_t H,
                    const void* g, const void* x, const void* h0, const void* w_ih,
                    const void* w_hh, const void* out, void* dx, void* dh0, void* dw_ih,
                    void* dw_hh, void* db_ih, void* db_hh, void* scratch, void* stream);

/* ------------------------------------------------------------------ data-parallel exchange
 * The averaged gradient all-reduce of batch-sharded training (no reference counterpart: the
 * reference is single-process), through NCCL loaded at run time from `library_path` (NULL:
 * "libnccl.so.2"; an NCCL the process already loaded is reused). Communicators are created
 * nonblocking; tg_comm_init polls their set-up against `timeout_s` (TG_ERR_TIMEOUT if a rank
 * never joins). Collectives run on the communicator's own stream after the work queued on
 * `stream`; tg_comm_join makes `stream` wait for them on the device; tg_comm_wait watches them
 * from the host and, on an asynchronous NCCL error or when `timeout_s` passes, aborts the
 * communicator and returns TG_ERR_COMM or TG_ERR_TIMEOUT (an aborted communicator stays
 * unusable). tg_comm_destroy finalises within `timeout_s`, else aborts. */
int tg_comm_load(const char* library_path);
int tg_comm_nccl_version(int* version);
int tg_comm_unique_id(void* out, size_t len);
int tg_comm_init(int nranks, int rank, const void* unique_id, double timeout_s, void** comm);
int tg_comm_all_reduce(void* comm, void* buf, size_t count, int dtype, int average, void* stream,
                       double timeout_s);
int tg_comm_join(void* comm, void* stream);
int tg_comm_wait(void* comm, double timeout_s);
int tg_comm_abort(void* comm);
int tg_comm_destroy(void* comm, double timeout_s);

/* ------------------------------------------------------------------ optimiser
 * optim/clip.py:15-31: total = sqrt(sum over tensors of sum(g^2)) accumulated in float64.
 * ptrs/numels are HOST arrays of `count` device pointers / sizes. The result (float64) is
 * written to total_dev[0]. `scratch` holds tg_sumsq_scratch_bytes(count) bytes. */
size_t tg_sumsq_scratch_bytes(int count);
int tg_sumsq_multi(int dtype, int count, void* const* ptrs, const int64_t* numels,
                   double* total_dev, void* scratch, void* stream);
/* If max_norm / (sqrt(total_sq... total_dev[0]) + eps) < 1, scale every tensor by that
 * factor rounded to the tensor dtype (the reference casts the scale to g.dtype). */
int tg_clip_scale_multi(int dtype, int count, void* const* ptrs, const int64_t* numels,
                        const double* total_dev, double max_norm, double eps, void* scratch,
                        void* stream);
/* AdamW/Adam update of one flat range (optim/adam.py:59-94) in the reference's order:
 * p *= 1 - lr*wd (decoupled); m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
 * p -= (lr/bc1) m / (sqrt(v)/sqrt(bc2) + eps), with bc_i = 1 - b_i^step.
 * decoupled = 0 gives Adam's L2 form (g += wd p). */
int tg_adam_update(int dtype, int64_t n, void* p, const void* g, void* m, void* v, double lr,
                   double beta1, double beta2, double eps, double weight_decay, int64_t step,
                   int decoupled, void* stream);
/* clip_grad_norm_ and AdamW fused (optim/clip.py:15-31 then optim/adam.py:59-94): the same
 * update, with the gradient read as g * (g's dtype)(max_norm / (total + clip_eps)) when that
 * factor is below 1, total = clip_total_dev[0] (tg_sumsq_multi's result). g itself is left
 * as it was (the host applies tg_clip_scale_multi later if the clipped gradient is read), so
 * one pass moves 28 bytes per fp32 parameter instead of the rewrite's 8 plus the update's 28.
 * clip_total_dev = NULL is tg_adam_update. */
int tg_adam_update_clipped(int dtype, int64_t n, void* p, const void* g, void* m, void* v,
                           double lr, double beta1, double beta2, double eps,
                           double weight_decay, int64_t step, int decoupled,
                           const double* clip_total_dev, double max_norm, double clip_eps,
                           void* stream);
/* Multi-tensor variant: one launch over `count` ranges (HOST pointer/size/step arrays). */
size_t tg_adam_multi_scratch_bytes(int count);
int tg_adam_update_multi(int dtype, int count, void* const* p, void* const* g, void* const* m,
                         void* const* v, const int64_t* numels, const int64_t* steps, double lr,
                         double beta1, double beta2, double eps, double weight_decay,
                         int decoupled, void* scratch, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TGB200_H */
