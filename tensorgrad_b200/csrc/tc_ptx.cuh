// Shared sm_100a plumbing of the tensor-core kernels (the GEMM and the fused attention
// forward): PTX wrappers for mbarriers, TMA, tensor memory and tcgen05.mma, the bounded wait,
// UMMA descriptors, and the host side of tensor maps. Included by one translation unit each;
// every definition has internal linkage (each unit keeps its own status word and map cache).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <functional>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace tg {
namespace tc {
namespace {

constexpr int BM = 128;
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 2 GHz

__device__ int g_status = 0;  // this unit's timeout record
// Cycle budget of every bounded wait in this unit (kTimeoutCycles unless a test shortened it
// to make a wait run out on purpose; read only once a wait has to spin).
__device__ long long g_wait_budget = kTimeoutCycles;

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
  const long long t0 = clock64(), budget = *(volatile long long*)&g_wait_budget;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (respect_abort && *abort_flag) return false;
    if (clock64() - t0 > budget) {
      *abort_flag = 1;
      atomicExch(&g_status, (int)TG_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- CTA-pair (cluster of 2) helpers for the cta_group::2 variant
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// The same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Arrival on a barrier of another CTA of the cluster with the default semantics (release
// at CTA scope): enough for hand-offs that tcgen05 fences order, e.g. an accumulator
// released after tcgen05.ld.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait with cluster-scope acquire (for barriers that the peer CTA arrives on).
__device__ __forceinline__ bool wait_bar_cluster(uint64_t* bar, uint32_t parity,
                                                 volatile int* abort_flag,
                                                 bool respect_abort = true) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64(), budget = *(volatile long long*)&g_wait_budget;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (respect_abort && *abort_flag) return false;
    if (clock64() - t0 > budget) {
      *abort_flag = 1;
      atomicExch(&g_status, (int)TG_ERR_TIMEOUT);
      return false;
    }
  }
}

// 4-D tiled load (x innermost, y rows, h head, b outer batch); no multicast.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int h, int b) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(h), "r"(b)
      : "memory");
}

// 5-D form: an MN-major operand whose MN dimension is split as (32, chunk), so one copy brings
// several 32-wide chunks ([chunk][k][32] in shared memory, the layout of one copy per chunk).
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int c, int h, int b) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(c), "r"(h),
      "r"(b)
      : "memory");
}

// TMA store of a shared-memory box (bulk-group completion) and its group bookkeeping.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x,
                                             int y, int h, int b) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(h), "r"(b)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed store groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

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

// Pair allocation: the same warp of both CTAs of the pair executes it.
__device__ __forceinline__ void tmem_alloc2(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 256-row MMA across the CTA pair: A rows 0..127 and B columns 0..N/2-1 come from the
// issuing (even) CTA's shared memory, A rows 128..255 and B columns N/2..N-1 from the same
// offsets in the odd CTA; each CTA's TMEM receives its 128 rows.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this offset in both CTAs of the pair once the pair's MMAs issued
// so far have completed.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
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

// A from tensor memory (128 lanes = rows, 8 columns = the k-step's 8 tf32 values per row).
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 8 consecutive 32-bit columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
// One 32-bit column of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v)
               : "memory");
}
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  return v;
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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
//   start: byte address; lbo/sbo: leading/stride byte offsets; layout: 4 = SWIZZLE_64B
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

// 4-D fp32 map: `nb` outer entries of `heads` row-major matrices of `rows` x `inner` (row
// stride `ld`, head stride `hstride`, outer stride `bstride` elements); boxes of
// box_inner x box_rows. Dimensions of extent 1 get a harmless stride (the encoder still
// wants a multiple of 16 bytes).
struct MapKey {
  const void* ptr;
  int64_t v[8];
  int dev;
  bool operator==(const MapKey& o) const {
    if (ptr != o.ptr || dev != o.dev) return false;
    for (int i = 0; i < 8; ++i)
      if (v[i] != o.v[i]) return false;
    return true;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.ptr) ^ (size_t)k.dev * 0x9E3779B97F4A7C15ull;
    for (int i = 0; i < 8; ++i) h = (h ^ (size_t)k.v[i]) * 0x100000001B3ull;
    return h;
  }
};

// Encoded maps by value (a map holds only an address, extents, strides and the box, so a
// cached entry is valid whenever the same values recur, e.g. the recurrent products of every
// time step of every training step). Host-side cost of an encode is then paid once.
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_map_cache;
static std::mutex g_map_mutex;
constexpr size_t kMapCacheCap = 1 << 14;

static int make_map_uncached(CUtensorMap* map, const float* ptr, int64_t inner, int64_t rows,
                             int64_t ld, int64_t heads, int64_t hstride, int64_t nb,
                             int64_t bstride, uint32_t box_inner, uint32_t box_rows,
                             CUtensorMapSwizzle swizzle);

static int make_map_chunked_uncached(CUtensorMap* map, const float* ptr, int64_t inner,
                                     int64_t rows, int64_t ld, int64_t heads, int64_t hstride,
                                     int64_t nb, int64_t bstride, uint32_t box_rows,
                                     uint32_t box_chunks, CUtensorMapSwizzle swizzle);

// chunks > 0: the MN-major 5-D map (inner split as 32 x inner / 32; inner % 32 == 0), boxes of
// 32 x box_rows x chunks; otherwise the 4-D map with boxes of box_inner x box_rows.
static int make_map(CUtensorMap* map, const float* ptr, int64_t inner, int64_t rows, int64_t ld,
                    int64_t heads, int64_t hstride, int64_t nb, int64_t bstride,
                    uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle,
                    uint32_t chunks = 0) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{ptr, {inner, rows, ld, heads, hstride, nb, bstride,
                   ((int64_t)box_inner << 32) | ((int64_t)chunks << 20) |
                       ((int64_t)box_rows << 8) | (int64_t)swizzle},
             dev};
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) {
      *map = it->second;
      return TG_OK;
    }
  }
  const int rc = chunks ? make_map_chunked_uncached(map, ptr, inner, rows, ld, heads, hstride,
                                                     nb, bstride, box_rows, chunks, swizzle)
                      : make_map_uncached(map, ptr, inner, rows, ld, heads, hstride, nb,
                                          bstride, box_inner, box_rows, swizzle);
  if (rc == TG_OK) {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    if (g_map_cache.size() >= kMapCacheCap) g_map_cache.clear();
    g_map_cache.emplace(key, *map);
  }
  return rc;
}

static int make_map_uncached(CUtensorMap* map, const float* ptr, int64_t inner, int64_t rows,
                             int64_t ld, int64_t heads, int64_t hstride, int64_t nb,
                             int64_t bstride, uint32_t box_inner, uint32_t box_rows,
                             CUtensorMapSwizzle swizzle) {
  EncodeFn enc = get_encode();
  if (!enc) return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: cuTensorMapEncodeTiled unavailable");
  const int64_t hs = heads > 1 ? hstride : rows * ld;
  const int64_t bs = nb > 1 ? bstride : (heads > 1 ? heads * hstride : rows * ld);
  if (hs <= 0 || bs <= 0 || (hs % 4) || (bs % 4))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: head/batch strides not 16-byte multiples");
  cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)nb};
  cuuint64_t strides[3] = {(cuuint64_t)ld * 4, (cuuint64_t)hs * 4, (cuuint64_t)bs * 4};
  cuuint32_t box[4] = {box_inner, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: tensor map encode failed (%d)", (int)r);
  return TG_OK;
}

static int make_map_chunked_uncached(CUtensorMap* map, const float* ptr, int64_t inner,
                                     int64_t rows, int64_t ld, int64_t heads, int64_t hstride,
                                     int64_t nb, int64_t bstride, uint32_t box_rows,
                                     uint32_t box_chunks, CUtensorMapSwizzle swizzle) {
  EncodeFn enc = get_encode();
  if (!enc) return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: cuTensorMapEncodeTiled unavailable");
  if (inner % 32) return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: chunked map needs inner % 32");
  const int64_t hs = heads > 1 ? hstride : rows * ld;
  const int64_t bs = nb > 1 ? bstride : (heads > 1 ? heads * hstride : rows * ld);
  if (hs <= 0 || bs <= 0 || (hs % 4) || (bs % 4))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: head/batch strides not 16-byte multiples");
  // (32 along MN, rows along K, chunks of 32 along MN, head, batch): a box of box_chunks
  // chunks lands as [chunk][row][32], the same bytes as one 32-wide box per chunk.
  cuuint64_t dims[5] = {32, (cuuint64_t)rows, (cuuint64_t)(inner / 32), (cuuint64_t)heads,
                        (cuuint64_t)nb};
  cuuint64_t strides[4] = {(cuuint64_t)ld * 4, 32 * 4, (cuuint64_t)hs * 4, (cuuint64_t)bs * 4};
  cuuint32_t box[5] = {32, box_rows, box_chunks, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: chunked tensor map encode failed (%d)",
                     (int)r);
  return TG_OK;
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace
}  // namespace tc
}  // namespace tg
