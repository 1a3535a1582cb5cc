// fp32 GEMM on the sm_100a tensor cores: tcgen05.mma kind::tf32 with a 3xTF32 split.
//
// C[m,n] = alpha * op(A) op(B) + beta * C (+ bias[n]) for row-major fp32 operands.
//
// Accuracy. TF32 keeps 10 explicit mantissa bits, far from the float64 reference at a
// relative 1e-4. Each operand x is split in shared memory into hi = x with the low 13
// mantissa bits cleared (exactly representable in TF32, so the tensor core's own input
// conversion is exact) and lo = x - hi (exact in fp32), and the tile product is accumulated
// as hi*hi + hi*lo + lo*hi in fp32 in TMEM. The dropped lo*lo term and the TF32 truncation
// of lo are ~2^-20 relative, close to fp32 rounding.
//
// Pipeline (one 128 x BN output tile per CTA, BN = 64 or 128, 256 threads; batched products
// index the third tensor-map dimension with blockIdx.z):
//   warp 0, lane 0 : TMA producer -- 128B-swizzled A/B tiles (BK = 32 fp32 = one swizzle
//                    row) into a STAGES-deep ring, completion on full[s].
//   warps 2..7     : split the stage into hi (in place) and lo (its own buffer), fence the
//                    generic-proxy writes for the async proxy, arrive on split[s]; warps 4..7
//                    then run the epilogue (TMEM lanes 32*(warp-4) .. +31 via tcgen05.ld).
//   warp 1, lane 0 : MMA issuer -- 3 x (BK/8) tcgen05.mma per stage, tcgen05.commit frees
//                    the stage (empty[s]); a final commit signals the accumulator.
// Operands may be K-major (rows hold K) or MN-major (rows hold M or N); both are native
// UMMA layouts for TF32, so no transposes are materialised. No TMA multicast is used.
//
// Every mbarrier wait is bounded (clock64 budget). On expiry the kernel records
// TG_ERR_TIMEOUT in a device status word, stops issuing work, drains what it started
// (bounded again), frees its TMEM and returns; tg_gemm_tc_status() reads the word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace tg {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;                       // fp32 elements per 128-byte swizzle row
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 2 GHz

__device__ int g_status = 0;

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false when the CTA is aborting (budget spent here or, when
// `respect_abort`, elsewhere in the CTA). Drains after an abort pass respect_abort = false:
// they still give up after their own budget.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                         bool respect_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (respect_abort && *abort_flag) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      *abort_flag = 1;
      atomicExch(&g_status, (int)TG_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 3-D tiled load (x innermost, z = batch); no multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor with sm_100 version bits.
//   start: byte address; lbo/sbo: leading/stride byte offsets; layout: 2 = SWIZZLE_128B
//   (16-byte atoms, 8-row period), 1 = SWIZZLE_128B_BASE32B (32-byte atoms, 4-row period).
__device__ __forceinline__ uint64_t smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((start >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  d |= (uint64_t)layout << 61;
  return d;
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, majors, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

struct TcArgs {
  int64_t m, n, k;
  float* c;
  int64_t ldc, stride_c;  // row stride and batch stride of C (elements)
  const float* bias;
  float alpha, beta;
  int kmode;              // GemmKMode: reduction range / tile skipping per output tile
};

// Split threads: warps 2..7.
constexpr int kSplitThreads = 192;

template <int BN>
struct Layout {
  static constexpr uint32_t A_BYTES = BM * BK * 4;  // 16 KB
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE = 2 * A_BYTES + 2 * B_BYTES;  // hi + lo of A and B
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

// Descriptor of k-step kk (8 tf32 along K) of a stage tile.
//  K-major: rows of 32 K values (128 B), 128-byte swizzle; the step starts 32 B into each
//           row; the next 8-row group is 1024 B on.
//  MN-major: the tile is 32-wide MN chunks of BK K-rows (128 B each, 4 KB per chunk). TF32
//           MN-major operands use the 128-byte swizzle with 32-byte atoms (4-row period):
//           the step starts 8 rows (1024 B) on, the next 4-row group is 512 B on (SBO) and the
//           next 32-wide MN chunk 4 KB on (LBO).
template <bool MN>
__device__ __forceinline__ uint64_t tile_desc(uint32_t tile_base, int kk) {
  if (MN) return smem_desc(tile_base + kk * 1024, /*lbo*/ 32 * BK * 4, /*sbo*/ 512, 1);
  return smem_desc(tile_base + kk * 32, /*lbo (unused)*/ 16, /*sbo*/ 1024, 2);
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(256, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               TcArgs args) {
  using L = Layout<BN>;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int bz = (int)blockIdx.z;
  // Causal attention products: a tile strictly above the diagonal is skipped outright
  // (kSkipUpper), and reductions over a triangular operand stop at (kUpToRow) or start
  // from (kFromRow) the tile's first output row. Uniform per CTA, so before any sync.
  if (args.kmode == GEMM_K_SKIP_UPPER && n0 > m0 + BM - 1) return;
  const int nk_all = (int)((args.k + BK - 1) / BK);
  int kb0 = 0, kb1 = nk_all;
  if (args.kmode == GEMM_K_UP_TO_ROW) {
    const int64_t kend = m0 + BM < args.k ? m0 + BM : args.k;
    kb1 = (int)((kend + BK - 1) / BK);
  } else if (args.kmode == GEMM_K_FROM_ROW) {
    kb0 = (int)(m0 / BK);
  }
  const int nk = kb1 > kb0 ? kb1 - kb0 : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE);
  uint64_t* split = full + STAGES;
  uint64_t* empty = split + STAGES;
  uint64_t* accum = empty + STAGES;
  uint64_t* drain = accum + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&split[s], kSplitThreads);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (; it < nk; ++it) {
        const int s = it % STAGES, round = it / STAGES;
        if (round > 0 && !wait_bar(&empty[s], (round - 1) & 1, abort_flag)) break;
        uint8_t* st = smem + s * L::STAGE;
        uint8_t* a_hi = st;
        uint8_t* b_hi = st + 2 * L::A_BYTES;
        mbar_arrive_expect_tx(&full[s], L::A_BYTES + L::B_BYTES);
        const int k0 = (kb0 + it) * BK;
        if (A_MN) {
#pragma unroll
          for (int c = 0; c < BM / 32; ++c)
            tma_load_3d(a_hi + c * 32 * BK * 4, &tmA, &full[s], (int)m0 + 32 * c, k0, bz);
        } else {
          tma_load_3d(a_hi, &tmA, &full[s], k0, (int)m0, bz);
        }
        if (B_MN) {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
            tma_load_3d(b_hi + c * 32 * BK * 4, &tmB, &full[s], (int)n0 + 32 * c, k0, bz);
        } else {
          tma_load_3d(b_hi, &tmB, &full[s], k0, (int)n0, bz);
        }
      }
      if (*abort_flag) {
        // Let the copies already issued land before the CTA's shared memory goes away.
        for (int j = it - STAGES; j < it; ++j) {
          if (j < 0) continue;
          wait_bar(&full[j % STAGES], (j / STAGES) & 1, abort_flag, false);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BM, BN, A_MN, B_MN);
      bool ok = true;
      for (int it = 0; it < nk; ++it) {
        const int s = it % STAGES, round = it / STAGES;
        if (!wait_bar(&split[s], round & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * L::STAGE);
        const uint32_t a_hi = st, a_lo = st + L::A_BYTES;
        const uint32_t b_hi = st + 2 * L::A_BYTES, b_lo = b_hi + L::B_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t ah = tile_desc<A_MN>(a_hi, kk), al = tile_desc<A_MN>(a_lo, kk);
          const uint64_t bh = tile_desc<B_MN>(b_hi, kk), bl = tile_desc<B_MN>(b_lo, kk);
          mma_tf32(tmem, al, bh, idesc, (it | kk) != 0);
          mma_tf32(tmem, ah, bl, idesc, 1);
          mma_tf32(tmem, ah, bh, idesc, 1);
        }
        mma_commit(&empty[s]);
      }
      if (ok) {
        mma_commit(accum);  // with nk == 0 this fires at once; the epilogue then uses 0
      } else {
        mma_commit(drain);
        wait_bar(drain, 0, abort_flag, false);  // MMAs already issued finish before dealloc
      }
    }
  }
  if (warp >= 2) {
    const int t = threadIdx.x - 64;
    for (int it = 0; it < nk; ++it) {
      const int s = it % STAGES, round = it / STAGES;
      if (!wait_bar(&full[s], round & 1, abort_flag)) break;
      uint8_t* st = smem + s * L::STAGE;
      float4* a_hi = reinterpret_cast<float4*>(st);
      float4* a_lo = reinterpret_cast<float4*>(st + L::A_BYTES);
      float4* b_hi = reinterpret_cast<float4*>(st + 2 * L::A_BYTES);
      float4* b_lo = reinterpret_cast<float4*>(st + 2 * L::A_BYTES + L::B_BYTES);
      auto split4 = [](float4* hi, float4* lo, int i) {
        const float4 x = hi[i];
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u); l.x = x.x - h.x;
        h.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u); l.y = x.y - h.y;
        h.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u); l.z = x.z - h.z;
        h.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u); l.w = x.w - h.w;
        hi[i] = h;
        lo[i] = l;
      };
#pragma unroll 4
      for (int i = t; i < (int)(L::A_BYTES / 16); i += kSplitThreads) split4(a_hi, a_lo, i);
#pragma unroll 4
      for (int i = t; i < (int)(L::B_BYTES / 16); i += kSplitThreads) split4(b_hi, b_lo, i);
      fence_proxy_async_smem();
      mbar_arrive(&split[s]);
    }
  }
  if (warp >= 4) {
    // Epilogue: TMEM lane r = 32 * (warp - 4) + lane holds output row m0 + r.
    // tcgen05.ld is warp-collective: decide per warp.
    const bool have = __all_sync(0xffffffffu, wait_bar(accum, 0, abort_flag));
    tc_fence_after();
    if (have) {
      const int ew = warp - 4;
      const int64_t row = m0 + 32 * ew + lane;
      float* crow = args.c + (int64_t)bz * args.stride_c + row * args.ldc;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(32 * ew) << 16) + (uint32_t)(cc * 32), r);
        if (row < args.m) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int64_t col = n0 + cc * 32 + j;
            if (col < args.n) {
              float v = nk ? args.alpha * __uint_as_float(r[j]) : 0.f;
              if (args.beta != 0.f) v += args.beta * crow[col];
              if (args.bias) v += args.bias[col];
              crow[col] = v;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 3-D fp32 map: `batch` row-major matrices of `rows` x `inner` (row stride `ld`, batch
// stride `bstride` elements); boxes of box_inner x box_rows x 1.
static int make_map(CUtensorMap* map, const float* ptr, int64_t inner, int64_t rows, int64_t ld,
                    int64_t batch, int64_t bstride, uint32_t box_inner, uint32_t box_rows,
                    CUtensorMapSwizzle swizzle) {
  EncodeFn enc = get_encode();
  if (!enc) return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(batch > 1 ? bstride : rows * ld) * 4};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: tensor map encode failed (%d)", (int)r);
  return TG_OK;
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
static int launch(const GemmArgs<float>& p, cudaStream_t stream) {
  using L = Layout<BN>;
  CUtensorMap ta, tb;
  int rc;
  // A: K-major = m rows of k; MN-major = k rows of m. Likewise B with n.
  constexpr CUtensorMapSwizzle kSwK = CU_TENSOR_MAP_SWIZZLE_128B;
  constexpr CUtensorMapSwizzle kSwMN = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  if (A_MN) rc = make_map(&ta, p.a, p.m, p.k, p.lda, p.batch, p.stride_a, 32, BK, kSwMN);
  else rc = make_map(&ta, p.a, p.k, p.m, p.lda, p.batch, p.stride_a, BK, BM, kSwK);
  if (rc != TG_OK) return rc;
  if (B_MN) rc = make_map(&tb, p.b, p.n, p.k, p.ldb, p.batch, p.stride_b, 32, BK, kSwMN);
  else rc = make_map(&tb, p.b, p.k, p.n, p.ldb, p.batch, p.stride_b, BK, BN, kSwK);
  if (rc != TG_OK) return rc;
  const size_t smem = STAGES * L::STAGE + 1024 + 256;
  static bool configured = false;
  if (!configured) {
    TG_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES, A_MN, B_MN>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured = true;
  }
  TcArgs a{p.m, p.n, p.k, p.c, p.ldc, p.stride_c, p.bias, p.alpha, p.beta, p.kmode};
  dim3 grid((unsigned)((p.n + BN - 1) / BN), (unsigned)((p.m + BM - 1) / BM), (unsigned)p.batch);
  gemm_tc_kernel<BN, STAGES, A_MN, B_MN><<<grid, 256, smem, stream>>>(ta, tb, a);
  return check_launch("gemm_tc");
}

template <int BN, int ST>
static int launch_any(const GemmArgs<float>& p, bool a_mn, bool b_mn, cudaStream_t stream) {
  if (!a_mn && !b_mn) return launch<BN, ST, false, false>(p, stream);
  if (!a_mn && b_mn) return launch<BN, ST, false, true>(p, stream);
  if (a_mn && !b_mn) return launch<BN, ST, true, false>(p, stream);
  return launch<BN, ST, true, true>(p, stream);
}

}  // namespace tc

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int gemm_tc_f32(const GemmArgs<float>& p, cudaStream_t stream) {
  if (p.batch < 1 || p.batch > 65535 || p.m <= 0 || p.n <= 0 || p.k <= 0)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: batch/empty shape");
  if (!aligned16(p.a) || !aligned16(p.b) || (p.lda % 4) || (p.ldb % 4))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: operands not 16-byte aligned");
  if (p.batch > 1 && ((p.stride_a % 4) || (p.stride_b % 4)))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: batch strides not 16-byte aligned");
  if (p.m > INT32_MAX || p.n > INT32_MAX || p.k > INT32_MAX)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: dimension beyond int32");
  const bool a_mn = p.trans_a != 0;   // A stored k x m
  const bool b_mn = p.trans_b == 0;   // B stored k x n
  if (p.n <= 64) return tc::launch_any<64, 4>(p, a_mn, b_mn, stream);
  return tc::launch_any<128, 3>(p, a_mn, b_mn, stream);
}

}  // namespace tg

extern "C" int tg_gemm_tc_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tg::tc::g_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(tg::tc::g_status, &z, sizeof(int));
  }
  return v;
}
