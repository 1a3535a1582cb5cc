// Deterministic reductions: column sums (bias gradients, the adjoint of broadcasting over
// leading axes), general keep-axis sums, and full sums.
#include "common.cuh"
#include "reduce.cuh"

namespace tg {
namespace {

constexpr int kColTile = 32;   // columns per block (one warp wide)
constexpr int kRowLanes = 8;   // row groups per block

// Pass 1 (fp32, 16-byte vectors): block (cx, chunk) sums rows [chunk*rpc, ...) of 128
// columns (a float4 per lane) into partial[chunk][c]; each row group keeps 4 rows in flight.
constexpr int kVecCols = 4 * kColTile;

__global__ void __launch_bounds__(kColTile * kRowLanes)
colsum_partial_vec4(const float* __restrict__ x, float* __restrict__ partial, int64_t rows,
                    int64_t cols, int64_t rows_per_chunk) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  __shared__ float4 sh[kRowLanes][kColTile];
  const int64_t c4 = (int64_t)blockIdx.x * kColTile + threadIdx.x;  // float4 column index
  const int64_t n4 = cols >> 2;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  int64_t r1 = r0 + rows_per_chunk;
  if (r1 > rows) r1 = rows;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c4 < n4) {
    const float4* xc = reinterpret_cast<const float4*>(x) + c4;
    int64_t r = r0 + threadIdx.y;
    for (; r + 3 * kRowLanes < r1; r += 4 * kRowLanes) {
      const float4 a = xc[r * n4], b = xc[(r + kRowLanes) * n4];
      const float4 c = xc[(r + 2 * kRowLanes) * n4], d = xc[(r + 3 * kRowLanes) * n4];
      acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
      acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
      acc.x += c.x; acc.y += c.y; acc.z += c.z; acc.w += c.w;
      acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
    }
    for (; r < r1; r += kRowLanes) {
      const float4 a = xc[r * n4];
      acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
    }
  }
  sh[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && c4 < n4) {
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kRowLanes; ++i) {
      const float4 v = sh[i][threadIdx.x];
      t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
    }
    reinterpret_cast<float4*>(partial + (int64_t)blockIdx.y * cols)[c4] = t;
  }
}

// Pass 1: block (cx, chunk) sums rows [chunk*rpc, ...) of 32 columns into partial[chunk][c].
template <typename T>
__global__ void __launch_bounds__(kColTile * kRowLanes)
colsum_partial_kernel(const T* __restrict__ x, T* __restrict__ partial, int64_t rows,
                      int64_t cols, int64_t rows_per_chunk) {
  __shared__ T sh[kRowLanes][kColTile + 1];
  const int64_t c = (int64_t)blockIdx.x * kColTile + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  int64_t r1 = r0 + rows_per_chunk;
  if (r1 > rows) r1 = rows;
  T acc = T(0);
  if (c < cols)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += kRowLanes) acc += x[r * cols + c];
  sh[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    T s = T(0);
#pragma unroll
    for (int i = 0; i < kRowLanes; ++i) s += sh[i][threadIdx.x];
    partial[(int64_t)blockIdx.y * cols + c] = s;
  }
}

// out[c] (+)= sum over chunks of partial[chunk][c]. Blocks of 32 columns x 8 chunk lanes:
// lane y sums chunks y, y+8, ... (loads batched by the unrolled loop), then the 8 lane sums
// are added in lane order. The order is fixed by the shape: deterministic.
template <typename T>
__global__ void __launch_bounds__(256)
colsum_final_kernel(const T* __restrict__ partial, T* __restrict__ out, int64_t cols,
                    int64_t chunks, int accumulate) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  __shared__ T sh[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int64_t c0 = (int64_t)blockIdx.x * 32; c0 < cols; c0 += (int64_t)gridDim.x * 32) {
    const int64_t c = c0 + tx;
    T s = T(0);
    if (c < cols) {
#pragma unroll 4
      for (int64_t i = ty; i < chunks; i += 8) s += partial[i * cols + c];
    }
    sh[ty][tx] = s;
    __syncthreads();
    if (ty == 0 && c < cols) {
      T t = sh[0][tx];
#pragma unroll
      for (int k = 1; k < 8; ++k) t += sh[k][tx];
      out[c] = accumulate ? out[c] + t : t;
    }
    __syncthreads();
  }
}

// One block per output element of a keep-axis reduction; threads stride the reduced space.
template <typename T>
__global__ void reduce_keep_kernel(const T* __restrict__ x, T* __restrict__ out, ReduceDims d) {
  __shared__ T sh[32];
  for (int64_t o = blockIdx.x; o < d.out_count; o += gridDim.x) {
    int64_t base = 0, rem = o;
    for (int i = d.n_keep - 1; i >= 0; --i) {
      base += (rem % d.keep_size[i]) * d.keep_stride[i];
      rem /= d.keep_size[i];
    }
    T acc = T(0);
    for (int64_t r = threadIdx.x; r < d.red_count; r += blockDim.x) {
      int64_t off = base, rr = r;
      for (int i = d.n_red - 1; i >= 0; --i) {
        off += (rr % d.red_size[i]) * d.red_stride[i];
        rr /= d.red_size[i];
      }
      acc += x[off];
    }
    acc = block_sum(acc, sh);
    if (threadIdx.x == 0) out[o] = acc;
    __syncthreads();
  }
}

template <typename T>
__global__ void sum_partial_kernel(const T* __restrict__ x, double* __restrict__ partial,
                                   int64_t n) {
  __shared__ double sh[32];
  double acc = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    acc += (double)x[i];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

template <typename T>
__global__ void sum_final_kernel(const double* __restrict__ partial, int nparts, T* out) {
  __shared__ double sh[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) out[0] = (T)acc;
}

}  // namespace

int64_t colsum_chunks(int64_t rows, int64_t cols) {
  // Enough blocks for about four per SM; at least 32 rows per chunk.
  const int64_t col_blocks = (cols + kVecCols - 1) / kVecCols;
  int64_t chunks = (4 * 148 + col_blocks - 1) / col_blocks;
  const int64_t max_chunks = (rows + 31) / 32;
  if (chunks > max_chunks) chunks = max_chunks;
  if (chunks < 1) chunks = 1;
  return chunks;
}

template <typename T>
int colsum(const T* x, T* out, int64_t rows, int64_t cols, int accumulate, void* scratch,
           cudaStream_t stream) {
  if (cols == 0) return TG_OK;
  if (rows == 0) {
    if (!accumulate) TG_CUDA_TRY(cudaMemsetAsync(out, 0, cols * sizeof(T), stream));
    return TG_OK;
  }
  const int64_t chunks = colsum_chunks(rows, cols);
  const int64_t rpc = (rows + chunks - 1) / chunks;
  T* partial = reinterpret_cast<T*>(scratch);
  if (sizeof(T) == 4 && cols % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(scratch) & 15) == 0) {
    dim3 grid((unsigned)((cols + kVecCols - 1) / kVecCols), (unsigned)chunks);
    launch_pdl(colsum_partial_vec4, dim3(grid), dim3(kColTile, kRowLanes), 0, stream,
        reinterpret_cast<const float*>(x), reinterpret_cast<float*>(partial), rows, cols, rpc);
  } else {
    dim3 grid((unsigned)((cols + kColTile - 1) / kColTile), (unsigned)chunks);
    colsum_partial_kernel<T><<<grid, dim3(kColTile, kRowLanes), 0, stream>>>(x, partial, rows,
                                                                            cols, rpc);
  }
  const int64_t col_tiles = (cols + 31) / 32;
  launch_pdl(colsum_final_kernel<T>, dim3((unsigned)(col_tiles < 4096 ? col_tiles : 4096)),
             dim3(256), 0, stream, partial, out, cols, chunks, accumulate);
  return check_launch("colsum", 2);
}
template int colsum<float>(const float*, float*, int64_t, int64_t, int, void*, cudaStream_t);
template int colsum<double>(const double*, double*, int64_t, int64_t, int, void*, cudaStream_t);

}  // namespace tg

extern "C" {

size_t tg_colsum_scratch_bytes(int dtype, int64_t rows, int64_t cols) {
  const size_t es = dtype == TG_F64 ? 8 : 4;
  return (size_t)tg::colsum_chunks(rows, cols) * (size_t)cols * es;
}

int tg_colsum(int dtype, const void* x, void* out, int64_t rows, int64_t cols, int accumulate,
              void* scratch, void* stream) {
  TG_CHECK_ARG(rows >= 0 && cols >= 0, "colsum: negative size");
  TG_CHECK_ARG(scratch || rows == 0 || cols == 0, "colsum: scratch is NULL");
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    return tg::colsum<T>((const T*)x, (T*)out, rows, cols, accumulate, scratch,
                         tg::as_stream(stream));
  });
}

int tg_reduce_sum(int dtype, int ndim, const int64_t* in_shape, const int* keep, const void* x,
                  void* out, void* stream) {
  TG_CHECK_ARG(ndim >= 0 && ndim <= tg::kMaxDims, "reduce_sum: ndim %d out of range", ndim);
  tg::ReduceDims d{};
  int64_t stride = 1;
  int64_t strides[tg::kMaxDims];
  for (int i = ndim - 1; i >= 0; --i) {
    strides[i] = stride;
    stride *= in_shape[i];
  }
  d.out_count = 1;
  d.red_count = 1;
  for (int i = 0; i < ndim; ++i) {
    if (keep[i]) {
      d.keep_size[d.n_keep] = in_shape[i];
      d.keep_stride[d.n_keep++] = strides[i];
      d.out_count *= in_shape[i];
    } else {
      d.red_size[d.n_red] = in_shape[i];
      d.red_stride[d.n_red++] = strides[i];
      d.red_count *= in_shape[i];
    }
  }
  if (d.out_count == 0) return TG_OK;
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    cudaStream_t s = tg::as_stream(stream);
    if (d.red_count == 0) {
      TG_CUDA_TRY(cudaMemsetAsync(out, 0, d.out_count * sizeof(T), s));
      return (int)TG_OK;
    }
    unsigned grid = (unsigned)(d.out_count < 148 * 16 ? d.out_count : 148 * 16);
    tg::reduce_keep_kernel<T><<<grid, 256, 0, s>>>((const T*)x, (T*)out, d);
    return tg::check_launch("reduce_sum");
  });
}

size_t tg_sum_all_scratch_bytes(void) { return 1024 * sizeof(double); }

int tg_sum_all(int dtype, const void* x, void* out, int64_t n, void* scratch, void* stream) {
  TG_CHECK_ARG(n >= 0 && scratch, "sum_all: bad size or NULL scratch");
  return TG_DISPATCH_FLOAT(dtype, T, [&] {
    cudaStream_t s = tg::as_stream(stream);
    const int parts = (int)tg::grid_for(n, 256, 1024);
    double* partial = reinterpret_cast<double*>(scratch);
    tg::sum_partial_kernel<T><<<parts, 256, 0, s>>>((const T*)x, partial, n);
    tg::sum_final_kernel<T><<<1, 256, 0, s>>>(partial, parts, (T*)out);
    return tg::check_launch("sum_all", 2);
  });
}

}  // extern "C"
