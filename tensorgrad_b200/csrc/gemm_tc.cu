// fp32 GEMM on the sm_100a tensor cores: tcgen05.mma kind::tf32 with a 3xTF32 split.
//
// C[m,n] = alpha * op(A) op(B) + beta * C (+ bias[n]) for row-major fp32 operands, batched
// over the third tensor-map dimension.
//
// Accuracy. TF32 keeps 10 explicit mantissa bits, far from the float64 reference at a
// relative 1e-4. The tensor core reads an fp32 operand as TF32 by truncating its low 13
// mantissa bits (measured: tests/test_gpu_kernels.py records the conversion), so the raw
// operand x already is hi = trunc(x); the kernel writes lo = x - hi (exact in fp32) next to
// it in shared memory and accumulates lo*hi + hi*lo + hi*hi in fp32 in TMEM. The dropped
// lo*lo term and the truncation of lo are ~2^-20 relative.
//
// Persistent, warp-specialised (one CTA of 512 threads per SM, tiles of 128 x BN,
// BN = 64/128/256; k-blocks of BK = 32 fp32 (128-byte rows) for tiles up to 128 wide, 16
// (64-byte rows) for 256-wide and pair tiles):
//   warp 0 (lane 0)  : TMA producer over every (tile, k-block) of this CTA into a raw ring
//                      of 4 to 8 slots.
//   warps 4..11      : write lo for each k-block into a 2- or 3-slot lo ring (A's hi and lo
//                      into TMEM when A is K-major and the tile at most 128 wide), fence the
//                      generic-proxy writes for the async proxy, arrive on split[l].
//   warp 1 (lane 0)  : MMA issuer: 3 x (BK/8) tcgen05.mma per k-block into one of two TMEM
//                      accumulators; tcgen05.commit frees the raw and lo slots and, after a
//                      tile's last k-block, hands the accumulator to the epilogue.
//   warps 12..15     : epilogue: tcgen05.ld of TMEM lanes 32*(warp%4).., alpha/beta/bias,
//                      16-byte stores; then the accumulator is released to the MMA warp.
// So a tile's epilogue overlaps the next tile's loads and MMAs. K-major operands use the
// 64- or 128-byte swizzle (by row length); MN-major TF32 operands the 128-byte swizzle with
// 32-byte atoms, the only swizzle UMMA accepts for them. No TMA multicast is used.
//
// Every mbarrier wait is bounded (clock64 budget). On expiry the kernel records
// TG_ERR_TIMEOUT in a device status word, stops issuing work, drains what it started
// (bounded again), frees its TMEM and returns; tg_gemm_tc_status() reads the word.
#include <stdlib.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "tc_ptx.cuh"

namespace tg {
namespace tc {

struct TcArgs {
  int64_t m, n, k;
  float* c;
  int64_t ldc, stride_c;  // row stride and batch stride of C (elements)
  const float* bias;
  float alpha, beta;
  int kmode;              // GemmKMode: reduction range / tile skipping per output tile
  int raw;                // 1: plain TF32 (no split; the tensor core truncates the fp32 bits)
  int m_tiles, n_tiles, batch;
  int a_fold;             // > 0: A's k index folds over its third map dimension
  int a_bcast, b_bcast;   // 1: the operand is shared by every batch entry (map depth 1)
  int64_t c_hw;           // > 0: NCHW output (see GemmArgs::c_hw)
  int splits, kb_per_split;
  float* ws;              // splits > 1: partial sums, [splits][m][n]
  int heads;              // batch entry bz = outer * heads + head
  int64_t stride_ch;      // head stride of C
  int epi;                // GemmEpilogue
  const float* rv0;       // softmax epilogues: lse (P) or delta (dS) per row
  const float* rv1;
  float* aux;             // GEMM_EPI_SOFTMAX_DS: P in (same layout as C)
  int tma_c;              // 1: whole tiles go out through shared memory and TMA stores (tmC),
                          //    the dS epilogue's P through TMA loads (tmX)
  // Stream-K tail (sk_tiles > 0). The first sk_first tiles (whole rounds of the units) go
  // round-robin as whole tiles; the k-blocks of the last sk_tiles tiles (sk_nk each) are cut
  // into one contiguous range per unit, sk_q long plus one for the first sk_r units. A tile
  // cut between units is a set of pieces: each writes its fp32 partial to a slot of sk_ws
  // ([2 * units][BM][BN], slot 2u for the first piece of unit u's range, 2u + 1 for its last)
  // and counts itself in sk_cnt ([sk_tiles][4], per epilogue warp); the piece that completes
  // the count sums all partials in piece order and writes the tile. No piece waits for another.
  // 1: the MN-major operand has the chunked 5-D map (one copy per k-block instead of one per
  // 32-wide chunk).
  int a_chunked, b_chunked;
  // 1: column tiles vary fastest (few column tiles, many row tiles): the column tiles of a
  // row band run side by side and share its A rows through the L2.
  int n_fast;
  int sk_first, sk_tiles, sk_nk;
  int64_t sk_q, sk_r;
  float* sk_ws;
  int* sk_cnt;
};

constexpr int kThreads = 512;
constexpr int kSplitWarp0 = 4, kSplitThreads = 256;  // warps 4..11
// Split warps per k-block: one group of 8 warps (two per TMEM lane quarter).
constexpr int kSplitGroups = 2, kGroupThreads = kSplitThreads / kSplitGroups;
constexpr int kEpiWarp0 = 12;                        // warps 12..15
// Epilogue staging: per epilogue warp two 32 x 32 fp32 boxes (128-byte swizzle), one TMA
// store (or load) each.
constexpr uint32_t kEpiBox = 32 * 32 * 4;
constexpr uint32_t kEpiBytes = 4 * 2 * kEpiBox;

// PAIR: a CTA of a cta_group::2 pair holds its 128 rows of A and half of the BN columns of B.
//
// Two rings. The raw ring holds what the TMA brings (A then B of one k-block per slot) and a
// slot stays busy until the k-block's MMAs complete; the lo ring holds what the split warps
// write (A's lo, unless A goes to tensor memory, then B's lo) and is only needed from the
// split to the MMAs. A k-block's trip through the raw ring is dominated by the TMA latency
// (about 1.5 us under load), so the raw ring gets the depth and the lo ring two or three
// slots.
template <int BN, bool PAIR = false, bool ATM = false>
struct Layout {
  // k-block depth: 32 fp32 (128-byte rows, 128-byte swizzle) for single-CTA tiles up to 128
  // wide, whose time per k-block is mostly a fixed cost; 16 (64-byte rows) otherwise.
  static constexpr int BK = (!PAIR && BN <= 128) ? 32 : 16;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr uint32_t A_BYTES = BM * BK * 4;
  static constexpr uint32_t B_BYTES = B_ROWS * BK * 4;
  static constexpr uint32_t RAW = A_BYTES + B_BYTES;               // raw slot: A, then B
  static constexpr uint32_t LO = (ATM ? 0 : A_BYTES) + B_BYTES;    // lo slot: A lo, B lo
  // Two accumulators (the epilogue of one tile overlaps the next tile's k-blocks), except
  // for 256-wide tiles with A in tensor memory, where one accumulator leaves TMEM room for A.
  static constexpr int NACC = (ATM && BN > 192) ? 1 : 2;
  static constexpr uint32_t ACC_COLS = NACC * BN;
  // ATM (A in tensor memory): A's hi and lo of each lo slot go to TMEM columns after the
  // accumulators (2 * BK per slot).
  // tcgen05.alloc takes a power of two from 32 to 512 columns.
  static constexpr uint32_t TMEM_COLS =
      ATM ? 512 : (ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                       : ACC_COLS <= 256 ? 256 : 512);
  static_assert(ACC_COLS <= 512, "accumulators exceed tensor memory");
  // Slot counts: the lo ring 2 (3 when its slots are small), bounded by TMEM with ATM; the
  // raw ring whatever fits in 193 KB beside it (at most 8).
  static constexpr int LO_TMEM_CAP = ATM ? (int)((512 - ACC_COLS) / (2 * BK)) : 8;
  static constexpr int LST0 = 3;
  static constexpr int LST = LST0 < LO_TMEM_CAP ? LST0 : LO_TMEM_CAP;
  static constexpr int RST0 = (int)((193 * 1024 - LST * LO) / RAW);
  static constexpr int RST = RST0 < 8 ? RST0 : 8;
  static constexpr uint32_t RINGS = RST * RAW + LST * LO;
};

// Descriptor of k-step kk (8 tf32 along K) of a stage tile with KB k values per row.
//  K-major : rows of KB K values; KB = 16: 64-byte rows, 64-byte swizzle, the next 8-row
//            group 512 B on; KB = 32: 128-byte rows, 128-byte swizzle, the next 8-row group
//            1024 B on. The step starts 32 B further into each row.
//  MN-major: 32-wide MN chunks of KB K-rows (128 B each), 128-byte swizzle with 32-byte
//            atoms: the step starts 8 rows (1024 B) on, the next 4-row group is 512 B on
//            (SBO), the next MN chunk KB * 128 B on (LBO).
template <bool MN, int KB>
__device__ __forceinline__ uint64_t tile_desc(uint32_t tile_base, int kk) {
  if (MN) return smem_desc(tile_base + kk * 1024, /*lbo*/ 32 * KB * 4, /*sbo*/ 512, 1);
  if (KB == 32) return smem_desc(tile_base + kk * 32, /*lbo (unused)*/ 16, /*sbo*/ 1024, 2);
  return smem_desc(tile_base + kk * 32, /*lbo (unused)*/ 16, /*sbo*/ 512, 4);
}

// Which output tile, batch entry and k-block range the t-th tile of the product is.
struct TileInfo {
  int64_t m0, n0;
  int bz, split, kb0, nk;
  bool skip;
  int sk_tile, seg, segs;  // stream-K: tail tile, piece index and count (segs 1: whole tile)
};

__device__ __forceinline__ TileInfo tile_info(const TcArgs& a, int t, int bn, int bm, int bk) {
  TileInfo ti;
  int mt, nt;
  if (a.kmode == GEMM_K_FROM_ROW || a.kmode == GEMM_K_UP_TO_ROW) {
    // Triangular reductions (no splits): the row tile is the slowest index, heaviest first
    // (the first row tile reduces over all of k from the row on, the last up to the row), so
    // the round-robin's first rounds take the longest tiles and the last the shortest.
    const int per_m = a.n_tiles * a.batch;
    const int q = t / per_m, r = t - q * per_m;
    mt = a.kmode == GEMM_K_FROM_ROW ? q : a.m_tiles - 1 - q;
    nt = r % a.n_tiles;
    ti.bz = r / a.n_tiles;
    ti.split = 0;
  } else if (a.n_fast) {
    nt = t % a.n_tiles;
    int rest = t / a.n_tiles;
    mt = rest % a.m_tiles;
    rest /= a.m_tiles;
    ti.bz = rest % a.batch;
    ti.split = rest / a.batch;
  } else {
    mt = t % a.m_tiles;
    int rest = t / a.m_tiles;
    nt = rest % a.n_tiles;
    rest /= a.n_tiles;
    ti.bz = rest % a.batch;
    ti.split = rest / a.batch;
  }
  ti.m0 = (int64_t)mt * bm;
  ti.n0 = (int64_t)nt * bn;
  // Causal attention products: a tile strictly above the diagonal is skipped outright, and
  // reductions over a triangular operand stop at / start from the tile's first output row.
  ti.skip = a.kmode == GEMM_K_SKIP_UPPER && ti.n0 > ti.m0 + BM - 1;
  const int nk_all = (int)((a.k + bk - 1) / bk);
  int kb0 = 0, kb1 = nk_all;
  if (a.splits > 1) {
    kb0 = ti.split * a.kb_per_split;
    kb1 = kb0 + a.kb_per_split < nk_all ? kb0 + a.kb_per_split : nk_all;
  } else if (a.kmode == GEMM_K_UP_TO_ROW) {
    const int64_t kend = ti.m0 + BM < a.k ? ti.m0 + BM : a.k;
    kb1 = (int)((kend + bk - 1) / bk);
  } else if (a.kmode == GEMM_K_FROM_ROW) {
    kb0 = (int)(ti.m0 / bk);
  }
  ti.kb0 = kb0;
  ti.nk = (ti.skip || kb1 <= kb0) ? 0 : kb1 - kb0;
  ti.sk_tile = -1;
  ti.seg = 0;
  ti.segs = 1;
  return ti;
}

// Stream-K: the unit whose tail range holds tail k-block w, and where unit u's range starts.
__device__ __forceinline__ int sk_unit_of(const TcArgs& a, int64_t w) {
  const int64_t big = a.sk_r * (a.sk_q + 1);
  return w < big ? (int)(w / (a.sk_q + 1)) : (int)(a.sk_r + (w - big) / a.sk_q);
}
__device__ __forceinline__ int64_t sk_range_start(const TcArgs& a, int u) {
  return (int64_t)u * a.sk_q + (u < a.sk_r ? u : a.sk_r);
}

// The w-th work item of a unit (false: none left): whole tiles unit, unit + units, ... below
// the stream-K tail (all tiles without one), then the pieces of the unit's range of tail
// k-blocks, each inside one tail tile. Every warp role walks the same items.
__device__ __forceinline__ bool work_item(const TcArgs& a, int unit, int units, int w, int bn,
                                          int bm, int bk, TileInfo& ti) {
  const int total = a.m_tiles * a.n_tiles * a.batch * a.splits;
  const int whole = a.sk_tiles ? a.sk_first : total;
  const int nw = unit < whole ? (whole - unit + units - 1) / units : 0;
  if (w < nw) {
    ti = tile_info(a, unit + w * units, bn, bm, bk);
    return true;
  }
  if (!a.sk_tiles) return false;
  const int64_t nk = a.sk_nk;
  const int64_t b = sk_range_start(a, unit);
  const int64_t end = b + a.sk_q + (unit < a.sk_r ? 1 : 0);
  const int64_t e = w - nw;
  const int64_t start = e == 0 ? b : (b / nk + e) * nk;
  if (start >= end) return false;
  const int j = (int)(start / nk);
  const int64_t stop = ((int64_t)j + 1) * nk < end ? ((int64_t)j + 1) * nk : end;
  ti = tile_info(a, a.sk_first + j, bn, bm, bk);
  ti.kb0 = (int)(start - (int64_t)j * nk);
  ti.nk = (int)(stop - start);
  ti.sk_tile = j;
  const int uf = sk_unit_of(a, (int64_t)j * nk);
  ti.seg = unit - uf;
  ti.segs = sk_unit_of(a, ((int64_t)j + 1) * nk - 1) - uf + 1;
  return true;
}

// Stream-K partial slot of unit u's piece of tail tile j: its range's first piece (the range
// starts inside tile j) or its last.
__device__ __forceinline__ int64_t sk_slot(const TcArgs& a, int u, int j) {
  return 2 * (int64_t)u + (sk_range_start(a, u) >= (int64_t)j * a.sk_nk ? 0 : 1);
}

// A partial slot holds BM x BN floats in the order the epilogue warps produce them, so that
// every access is coalesced: [warp 4][chunk BN/32][k 8][lane 32] float4, where lane = row
// within the warp's 32 rows and (chunk, k) = columns 32 chunk + 4k .. + 3.
template <int BN>
__device__ __forceinline__ float4* sk_chunk(const TcArgs& a, int64_t slot, int ew, int cc) {
  return reinterpret_cast<float4*>(a.sk_ws) + ((slot * 4 + ew) * (BN / 32) + cc) * 8 * 32;
}

// Sum, in piece order, of the partials of tail tile j (pieces from unit u_first on) at this
// lane's row and 32 columns: what the accumulator of an uncut tile would hold there.
template <int BN>
__device__ __forceinline__ void sk_sum(const TcArgs& a, int u_first, int segs, int j, int ew,
                                       int lane, int cc, uint32_t (&r)[32]) {
  float v[32];
#pragma unroll 1
  for (int s = 0; s < segs; ++s) {
    const float4* p = sk_chunk<BN>(a, sk_slot(a, u_first + s, j), ew, cc) + lane;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 q = __ldcg(p + 32 * k);
      if (s == 0) {
        v[4 * k] = q.x; v[4 * k + 1] = q.y; v[4 * k + 2] = q.z; v[4 * k + 3] = q.w;
      } else {
        v[4 * k] += q.x; v[4 * k + 1] += q.y; v[4 * k + 2] += q.z; v[4 * k + 3] += q.w;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 32; ++k) r[k] = __float_as_uint(v[k]);
}

// PAIR = true: launched in clusters of two CTAs; each pair computes 256 x BN tiles with
// cta_group::2 MMAs issued by the even CTA (see mma_tf32_pair). Every role runs in both
// CTAs on its own 128 rows and half of B, except the MMA issuer (even CTA only). The split
// warps and the epilogue of the odd CTA arrive on the even CTA's barriers; the MMA commits
// arrive on both CTAs' barriers.
template <int BN, bool A_MN, bool B_MN, bool PAIR, bool ATM>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX,
               TcArgs args) {
  using L = Layout<BN, PAIR, ATM>;
  static_assert(!ATM || (!PAIR && !A_MN), "A in tensor memory: single CTA, K-major A");
  constexpr int TILE_M = PAIR ? 2 * BM : BM;
  constexpr int KB = L::BK;
  constexpr int RST = L::RST, LST = L::LST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* raw_ring = smem;                       // RST slots of L::RAW bytes
  uint8_t* lo_ring = smem + RST * L::RAW;         // LST slots of L::LO bytes
  uint8_t* ebuf_all = smem + L::RINGS;            // kEpiBytes of epilogue staging
  uint64_t* full = reinterpret_cast<uint64_t*>(ebuf_all + kEpiBytes);  // [RST] raw landed
  uint64_t* empty = full + RST;                   // [RST] raw slot consumed by the MMAs
  uint64_t* split = empty + RST;                  // [LST] lo slot written
  uint64_t* acc_full = split + LST;      // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain = acc_empty + 2;
  uint64_t* ebar_all = drain + 1;        // [4 warps][2]: epilogue TMA loads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar_all + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work unit: a CTA, or a CTA pair (tile t goes to unit t % units).
  const uint32_t rank = PAIR ? cluster_rank() : 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int64_t row_off = (int64_t)rank * BM;  // this CTA's rows within a pair tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < RST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int l = 0; l < LST; ++l) {
      // One arrival per split warp, plus (even CTA of a pair) the odd CTA's relay.
      mbar_init(&split[l], (kGroupThreads / 32) + (PAIR && rank == 0 ? 1 : 0));
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], PAIR ? 8 : 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    for (int b = 0; b < 8; ++b) mbar_init(&ebar_all[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if (PAIR) tmem_alloc2(tmem_slot, L::TMEM_COLS);
    else tmem_alloc(tmem_slot, L::TMEM_COLS);
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Single-CTA launches use programmatic dependent launch: the prologue above (barriers,
  // tensor memory) may overlap the kernel ahead on the stream; nothing in global memory is
  // touched before this wait.
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool stop = false;
      for (int w = 0; !stop; ++w) {
        TileInfo ti;
        if (!work_item(args, unit, units, w, BN, TILE_M, KB, ti)) break;
        for (int j = 0; j < ti.nk; ++j, ++it) {
          const int s = it % RST, round = it / RST;
          if (round > 0 && !wait_bar(&empty[s], (round - 1) & 1, abort_flag)) { stop = true; break; }
          uint8_t* a_raw = raw_ring + s * L::RAW;
          uint8_t* b_raw = a_raw + L::A_BYTES;
          mbar_arrive_expect_tx(&full[s], L::A_BYTES + L::B_BYTES);
          const int k0 = (ti.kb0 + j) * KB;
          const int hh = ti.bz % args.heads, bo = ti.bz / args.heads;
          const int ha = args.a_bcast ? 0 : hh, ba = args.a_bcast ? 0 : bo;
          const int hb = args.b_bcast ? 0 : hh, bb = args.b_bcast ? 0 : bo;
          const int am0 = (int)(ti.m0 + row_off);
          const int bn0 = (int)ti.n0 + (int)rank * L::B_ROWS;
          if (A_MN && args.a_chunked) {
            tma_load_5d(a_raw, &tmA, &full[s], 0, k0, am0 / 32, ha, ba);
          } else if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 32; ++c)
              tma_load_4d(a_raw + c * 32 * KB * 4, &tmA, &full[s], am0 + 32 * c, k0, ha, ba);
          } else if (args.a_fold > 0) {
            tma_load_4d(a_raw, &tmA, &full[s], k0 % args.a_fold, am0, 0, k0 / args.a_fold);
          } else {
            tma_load_4d(a_raw, &tmA, &full[s], k0, am0, ha, ba);
          }
          if (B_MN && args.b_chunked) {
            tma_load_5d(b_raw, &tmB, &full[s], 0, k0, bn0 / 32, hb, bb);
          } else if (B_MN) {
#pragma unroll
            for (int c = 0; c < L::B_ROWS / 32; ++c)
              tma_load_4d(b_raw + c * 32 * KB * 4, &tmB, &full[s], bn0 + 32 * c, k0, hb, bb);
          } else {
            tma_load_4d(b_raw, &tmB, &full[s], k0, bn0, hb, bb);
          }
        }
      }
      if (*abort_flag) {
        // Let the copies already issued land before the CTA's shared memory goes away.
        for (int j = it - RST; j < it; ++j) {
          if (j < 0) continue;
          wait_bar(&full[j % RST], (j / RST) & 1, abort_flag, false);
        }
      } else {
        // Tail: the MMA's last raw-slot releases (tcgen05.commit arrivals on this CTA's empty
        // barriers) land before the CTA may exit.
        for (int j = it - RST; j < it; ++j) {
          if (j < 0) continue;
          wait_bar(&empty[j % RST], (j / RST) & 1, abort_flag);
        }
      }
    }
  } else if (PAIR && warp == 2) {
    if (lane == 0 && rank == 1) {
      // Relay: once this CTA's split warps finished stage s (local barrier), one
      // cluster-scope release arrival tells the even CTA's MMA issuer.
      int it = 0;
      bool ok = true;
      for (int w = 0; ok; ++w) {
        TileInfo ti;
        if (!work_item(args, unit, units, w, BN, TILE_M, KB, ti)) break;
        for (int j = 0; j < ti.nk; ++j, ++it) {
          const int l = it % LST;
          if (!wait_bar(&split[l], (it / LST) & 1, abort_flag)) { ok = false; break; }
          mbar_arrive_cluster(map_to_rank(&split[l], 0));
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = instr_desc(TILE_M, BN, A_MN, B_MN);
      int it = 0, tc = 0;
      bool ok = true;
      for (int w = 0; ok; ++w) {
        TileInfo ti;
        if (!work_item(args, unit, units, w, BN, TILE_M, KB, ti)) break;
        if (ti.skip) continue;
        const int buf = tc % L::NACC;
        if (tc >= L::NACC) {
          const uint32_t par = ((tc / L::NACC) - 1) & 1;
          if (!wait_bar(&acc_empty[buf], par, abort_flag)) { ok = false; break; }
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int j = 0; j < ti.nk; ++j, ++it) {
          const int s = it % RST, l = it % LST;
          const uint32_t a_raw = smem_u32(raw_ring + s * L::RAW), b_raw = a_raw + L::A_BYTES;
          const uint32_t a_lo = smem_u32(lo_ring + l * L::LO);
          const uint32_t b_lo = a_lo + (ATM ? 0u : L::A_BYTES);
          if (!PAIR) {
            // hi x hi needs only what the TMA brought: issue it as soon as the raw slot has
            // landed, so the tensor pipe works while the split warps write lo; then the two
            // lo products (A's lo and hi from TMEM when ATM).
            // The TMA's writes are visible to the MMAs once the barrier completes (both in the
            // async proxy); the split warps fenced their stores for the async proxy before
            // arriving. Only A's hi/lo in TMEM (ATM) need the tcgen05 thread-sync fence.
            if (!wait_bar(&full[s], (it / RST) & 1, abort_flag)) { ok = false; break; }
#pragma unroll
            for (int kk = 0; kk < KB / 8; ++kk)
              mma_tf32(acc, tile_desc<A_MN, KB>(a_raw, kk), tile_desc<B_MN, KB>(b_raw, kk),
                       idesc, (j | kk) != 0);
            if (!args.raw) {
              if (!wait_bar(&split[l], (it / LST) & 1, abort_flag)) { ok = false; break; }
              if (ATM) tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < KB / 8; ++kk) {
                const uint64_t bh = tile_desc<B_MN, KB>(b_raw, kk);
                const uint64_t bl = tile_desc<B_MN, KB>(b_lo, kk);
                if (ATM) {
                  // A's hi (the raw bits) and lo of this lo slot in TMEM columns after the
                  // accumulators: [hi k 0..KB-1 | lo k 0..KB-1].
                  const uint32_t th = tmem + L::ACC_COLS + (uint32_t)(l * 2 * KB + kk * 8);
                  mma_tf32_ta(acc, th + KB, bh, idesc, 1);
                  mma_tf32_ta(acc, th, bl, idesc, 1);
                } else {
                  mma_tf32(acc, tile_desc<A_MN, KB>(a_lo, kk), bh, idesc, 1);
                  mma_tf32(acc, tile_desc<A_MN, KB>(a_raw, kk), bl, idesc, 1);
                }
              }
            }
            mma_commit(&empty[s]);  // frees the raw slot, and with it lo slot l (see the split)
            continue;
          }
          if (!wait_bar_cluster(&split[l], (it / LST) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < KB / 8; ++kk) {
            const uint64_t ah = tile_desc<A_MN, KB>(a_raw, kk), al = tile_desc<A_MN, KB>(a_lo, kk);
            const uint64_t bh = tile_desc<B_MN, KB>(b_raw, kk), bl = tile_desc<B_MN, KB>(b_lo, kk);
            if (PAIR) {
              if (args.raw) {
                mma_tf32_pair(acc, ah, bh, idesc, (j | kk) != 0);
              } else {
                mma_tf32_pair(acc, al, bh, idesc, (j | kk) != 0);
                mma_tf32_pair(acc, ah, bl, idesc, 1);
                mma_tf32_pair(acc, ah, bh, idesc, 1);
              }
            }
          }
          mma_commit_pair_both(&empty[s]);
        }
        if (!ok) break;
        // with nk == 0 this fires at once; the epilogue uses 0
        if (PAIR) mma_commit_pair_both(&acc_full[buf]);
        else mma_commit(&acc_full[buf]);
        ++tc;
      }
      if (!ok) {
        if (PAIR) mma_commit_pair_local(drain);
        else mma_commit(drain);
        wait_bar(drain, 0, abort_flag, false);  // MMAs already issued finish before dealloc
      }
    }
  } else if (warp >= kSplitWarp0 && warp < kEpiWarp0) {
    constexpr int kGroupWarps = kGroupThreads / 32;
    const int grp = (warp - kSplitWarp0) / kGroupWarps;
    const int t0 = threadIdx.x - (kSplitWarp0 + kGroupWarps * grp) * 32;  // 0 .. kGroupThreads-1
    int it = 0;
    // Plain TF32 on one CTA: the MMAs read only what the TMA brought, nothing to split.
    bool stop = !PAIR && args.raw;
    for (int w = 0; !stop; ++w) {
      TileInfo ti;
      if (!work_item(args, unit, units, w, BN, TILE_M, KB, ti)) break;
      for (int j = 0; j < ti.nk; ++j, ++it) {
        if (it % kSplitGroups != grp) continue;
        const int s = it % RST, l = it % LST;
        // Warp-uniform decision: the warp stays converged for the arrival below. The raw slot
        // has landed, and the lo slot (and its TMEM columns) is free again: its last user,
        // k-block it - LST, released its raw slot with the same commit (one commit per k-block
        // serves both rings; LST <= RST).
        const int prev = it - LST;
        const bool landed =
            wait_bar(&full[s], (it / RST) & 1, abort_flag) &&
            (prev < 0 || wait_bar(&empty[prev % RST], (prev / RST) & 1, abort_flag));
        if (!__all_sync(0xffffffffu, landed)) { stop = true; break; }
        uint8_t* st = raw_ring + s * L::RAW;
        uint8_t* lo = lo_ring + l * L::LO;
        auto lo_of = [](float x) {
          return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
        };
        auto lo4 = [&](const float4* x, float4* lo, int i) {
          const float4 v = x[i];
          lo[i] = make_float4(lo_of(v.x), lo_of(v.y), lo_of(v.z), lo_of(v.w));
        };
        if (!args.raw) {
          const float4* b_raw = reinterpret_cast<const float4*>(st + L::A_BYTES);
          float4* b_lo = reinterpret_cast<float4*>(lo + (ATM ? 0u : L::A_BYTES));
          if (!ATM) {
            const float4* a_raw = reinterpret_cast<const float4*>(st);
            float4* a_lo = reinterpret_cast<float4*>(lo);
#pragma unroll
            for (int i = t0; i < (int)(L::A_BYTES / 16); i += kGroupThreads) lo4(a_raw, a_lo, i);
          }
#pragma unroll
          for (int i = t0; i < (int)(L::B_BYTES / 16); i += kGroupThreads) lo4(b_raw, b_lo, i);
        }
        if (ATM) {
          // A rows to TMEM: the warp's lane quarter (warp % 4) holds rows 32 q .. 32 q + 31;
          // the group's warps of one quarter share its KB k values in units of 8. The TMA
          // wrote A K-major in rows of KB floats with the KB*4-byte swizzle: 16-byte chunk c
          // of row r sits at chunk c ^ ((r / 2) % 4) (64-byte rows) or c ^ (r % 8) (128-byte).
          constexpr int kUnits = KB / 8;
          constexpr int kWarpsPerQuarter = kGroupThreads / 128;
          constexpr int kUnitsPerWarp = kUnits / kWarpsPerQuarter;
          const int qr = warp & 3;
          const int u0 = (((warp - kSplitWarp0) >> 2) % kWarpsPerQuarter) * kUnitsPerWarp;
          const int r = 32 * qr + lane, sw = KB == 32 ? (r & 7) : ((r >> 1) & 3);
          const uint8_t* arow = st + r * (KB * 4);
#pragma unroll
          for (int uu = 0; uu < kUnitsPerWarp; ++uu) {
            const int u = u0 + uu;
            const float4 v0 = *reinterpret_cast<const float4*>(arow + (((2 * u) ^ sw) << 4));
            const float4 v1 =
                *reinterpret_cast<const float4*>(arow + (((2 * u + 1) ^ sw) << 4));
            const uint32_t taddr = tmem + ((uint32_t)(32 * qr) << 16) + L::ACC_COLS +
                                   (uint32_t)(l * 2 * KB + u * 8);
            const uint32_t hi[8] = {__float_as_uint(v0.x), __float_as_uint(v0.y),
                                    __float_as_uint(v0.z), __float_as_uint(v0.w),
                                    __float_as_uint(v1.x), __float_as_uint(v1.y),
                                    __float_as_uint(v1.z), __float_as_uint(v1.w)};
            tmem_st8(taddr, hi);
            if (!args.raw) {
              const uint32_t lo[8] = {
                  __float_as_uint(lo_of(v0.x)), __float_as_uint(lo_of(v0.y)),
                  __float_as_uint(lo_of(v0.z)), __float_as_uint(lo_of(v0.w)),
                  __float_as_uint(lo_of(v1.x)), __float_as_uint(lo_of(v1.y)),
                  __float_as_uint(lo_of(v1.z)), __float_as_uint(lo_of(v1.w))};
              tmem_st8(taddr + KB, lo);
            }
          }
          tmem_wait_st();
          tc_fence_before();
        }
        // One arrival per warp after all its lanes fenced (256 arrivals on one barrier would
        // serialise in the shared-memory atomics); in a pair the odd CTA's relay thread
        // forwards its stage to the even CTA.
        fence_proxy_async_smem();
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&split[l]);
      }
    }
  } else if (warp >= kEpiWarp0) {
    const int ew = warp - kEpiWarp0;  // == warp % 4: TMEM lanes 32*ew .. +31
    int tc = 0;
    const bool vec = args.c_hw == 0 && (args.ldc % 4 == 0) && (args.stride_c % 4 == 0) &&
                     (args.stride_ch % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(args.c) & 15) == 0) &&
                     (!args.bias || (reinterpret_cast<uintptr_t>(args.bias) & 15) == 0);
    // Shared-memory staging of this warp: two 32 x 32 boxes with their load barriers.
    uint8_t* ebuf = ebuf_all + ew * 2 * kEpiBox;
    uint64_t* ebar = ebar_all + 2 * ew;
    uint32_t eph = 0;  // phase bits of ebar[0], ebar[1]
    int q = 0;         // boxes stored so far (alternates the two buffers)
    for (int w = 0;; ++w) {
      TileInfo ti;
      if (!work_item(args, unit, units, w, BN, TILE_M, KB, ti)) break;
      if (ti.skip) continue;
      const int buf = tc % L::NACC;
      if (!PAIR && args.tma_c && args.splits == 1) {
        // Whole 32 x 32 boxes: lane = row in registers, written to shared memory with a
        // 128-byte swizzle (conflict-free), stored by one TMA store per box (rows and columns
        // past the product are clipped by the map). dS also reads its P boxes by TMA, two
        // boxes ahead, the first two issued before the accumulator is ready.
        const int hh = ti.bz % args.heads, bo = ti.bz / args.heads;
        const int row0 = (int)ti.m0 + 32 * ew;
        const bool rows_in = row0 < args.m;
        const int64_t left = (args.n - ti.n0 + 31) / 32;
        const int nch = (int)(left < BN / 32 ? left : BN / 32);
        const bool dsm = args.epi == GEMM_EPI_SOFTMAX_DS;
        const bool pmm = args.epi == GEMM_EPI_SOFTMAX_P;
        const bool causal = args.kmode == GEMM_K_SKIP_UPPER;
        if (dsm && rows_in) {
          if (lane == 0) {
            bulk_wait_read<0>();
            for (int b = 0; b < 2 && b < nch; ++b) {
              mbar_arrive_expect_tx(&ebar[b], kEpiBox);
              tma_load_4d(ebuf + b * kEpiBox, &tmX, &ebar[b], (int)ti.n0 + 32 * b, row0, hh, bo);
            }
          }
          __syncwarp();
        }
        const bool have =
            __all_sync(0xffffffffu, wait_bar(&acc_full[buf], (tc / L::NACC) & 1, abort_flag));
        if (!have) {
          if (dsm && rows_in)
            for (int b = 0; b < 2 && b < nch; ++b) wait_bar(&ebar[b], (eph >> b) & 1, abort_flag, false);
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(32 * ew) << 16);
        const int64_t row = (int64_t)row0 + lane;
        float rv = 0.f;
        if ((dsm || pmm) && row < args.m)
          rv = (dsm ? args.rv1 : args.rv0)[(int64_t)ti.bz * args.m + row];
        bool ok = true;
        // Stream-K piece of a tile cut between units: its partial (every column, unscaled)
        // goes to this unit's slot and the accumulator is released; the piece that completes
        // the count of this warp's 32 rows sums all pieces' partials below in place of the
        // accumulator. Nothing waits for another unit.
        const bool piece = ti.segs > 1;
        int u_first = 0;
        if (piece) {
          const int64_t slot = sk_slot(args, unit, ti.sk_tile);
#pragma unroll 1
          for (int cc = 0; cc < BN / 32; ++cc) {
            uint32_t r[32];
            tmem_ld32(acc + (uint32_t)(cc * 32), r);
            float4* dst = sk_chunk<BN>(args, slot, ew, cc) + lane;
#pragma unroll
            for (int k = 0; k < 8; ++k)
              dst[32 * k] = make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]),
                                   __uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
          __threadfence();
          __syncwarp();
          int arrived = 0;
          if (lane == 0) arrived = atomicAdd(&args.sk_cnt[ti.sk_tile * 4 + ew], 1);
          arrived = __shfl_sync(0xffffffffu, arrived, 0);
          if (arrived != ti.segs - 1) {
            ++tc;
            continue;
          }
          __threadfence();
          if (lane == 0) args.sk_cnt[ti.sk_tile * 4 + ew] = 0;  // zero for the next launch
          u_first = unit - ti.seg;
        }
#pragma unroll 1
        for (int cc = 0; cc < nch && rows_in; ++cc) {
          uint32_t r[32];
          if (piece) sk_sum<BN>(args, u_first, ti.segs, ti.sk_tile, ew, lane, cc, r);
          else tmem_ld32(acc + (uint32_t)(cc * 32), r);
          const int c0 = (int)ti.n0 + cc * 32;
          float4* box;
          if (dsm) {
            const int b = cc & 1;
            box = reinterpret_cast<float4*>(ebuf + b * kEpiBox);
            if (!__all_sync(0xffffffffu, wait_bar(&ebar[b], (eph >> b) & 1, abort_flag, false))) {
              ok = false;
              break;
            }
            eph ^= 1u << b;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float4 pv = box[lane * 8 + (k ^ (lane & 7))];
              const float a0 = ti.nk ? __uint_as_float(r[4 * k]) : 0.f;
              const float a1 = ti.nk ? __uint_as_float(r[4 * k + 1]) : 0.f;
              const float a2 = ti.nk ? __uint_as_float(r[4 * k + 2]) : 0.f;
              const float a3 = ti.nk ? __uint_as_float(r[4 * k + 3]) : 0.f;
              r[4 * k] = __float_as_uint(pv.x * (a0 - rv) * args.alpha);
              r[4 * k + 1] = __float_as_uint(pv.y * (a1 - rv) * args.alpha);
              r[4 * k + 2] = __float_as_uint(pv.z * (a2 - rv) * args.alpha);
              r[4 * k + 3] = __float_as_uint(pv.w * (a3 - rv) * args.alpha);
            }
            __syncwarp();  // every lane has read the box before it is overwritten
          } else {
            box = reinterpret_cast<float4*>(ebuf + (q & 1) * kEpiBox);
            ++q;
            if (lane == 0) bulk_wait_read<1>();  // the store from this buffer two boxes ago
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float a = ti.nk ? __uint_as_float(r[j]) : 0.f;
              float v;
              if (pmm) {
                // The fast exponential intrinsic: the argument is <= 0 up to rounding and
                // its relative error (a few ulp plus ~|x| 2^-22) stays far below 1e-4.
                // Exponential first, then a select: a conditional around it would make the
                // compiler branch per element.
                const float e = __expf(__fmul_rn(args.alpha, a) - rv);
                v = (causal && c0 + j > row) ? 0.f : e;
              } else {
                v = args.alpha * a;
                if (args.bias && c0 + j < args.n) v += args.bias[c0 + j];
              }
              r[j] = __float_as_uint(v);
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k)
            box[lane * 8 + (k ^ (lane & 7))] =
                make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]),
                            __uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_4d(&tmC, box, c0, row0, hh, bo);
            bulk_commit();
          }
          if (dsm && cc + 2 < nch) {
            if (lane == 0) {
              bulk_wait_read<0>();
              mbar_arrive_expect_tx(&ebar[cc & 1], kEpiBox);
              tma_load_4d(box, &tmX, &ebar[cc & 1], c0 + 64, row0, hh, bo);
            }
            __syncwarp();
          }
        }
        if (!piece) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        ++tc;
        if (!ok) break;
        continue;
      }
      // tcgen05.ld is warp-collective: decide per warp.
      const bool have = __all_sync(0xffffffffu, wait_bar(&acc_full[buf], (tc / L::NACC) & 1, abort_flag));
      if (!have) break;
      tc_fence_after();
      const int64_t row = ti.m0 + row_off + 32 * ew + lane;
      // Partial sums of a split reduction go to the workspace unscaled (the reduce kernel
      // applies alpha, beta and the bias). NCHW output: lanes are consecutive pixels, so the
      // 32 stores of one column are one coalesced line.
      const bool part = args.splits > 1;
      float* crow;
      int64_t cstep = 1;
      if (part) {
        crow = args.ws + ((int64_t)ti.split * args.m + row) * args.n;
      } else if (args.c_hw > 0) {
        crow = args.c + (int64_t)ti.bz * args.stride_ch + (row / args.c_hw) * args.stride_c +
               row % args.c_hw;
        cstep = args.ldc;
      } else {
        crow = args.c + (int64_t)(ti.bz / args.heads) * args.stride_c +
               (int64_t)(ti.bz % args.heads) * args.stride_ch + row * args.ldc;
      }
      const float alpha = part ? 1.f : args.alpha, beta = part ? 0.f : args.beta;
      const float* bias = part ? nullptr : args.bias;
      const bool vrow = part ? (args.n % 4 == 0) : vec;
      const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(32 * ew) << 16);
      // Attention softmax epilogues: P = exp(alpha acc - lse) (zero above the diagonal of a
      // causal product), or dS = P (acc - delta) alpha with P read from aux.
      const bool ds = args.epi == GEMM_EPI_SOFTMAX_DS && !part;
      const bool pm = args.epi == GEMM_EPI_SOFTMAX_P && !part;
      const bool causal = args.kmode == GEMM_K_SKIP_UPPER;
      const float* arow = ds ? args.aux + (crow - args.c) : nullptr;
      float rv = 0.f;
      if ((ds || pm) && row < args.m) rv = (ds ? args.rv1 : args.rv0)[(int64_t)ti.bz * args.m + row];
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(acc + (uint32_t)(cc * 32), r);
        const int64_t c0 = ti.n0 + cc * 32;
        if ((ds || pm) && row < args.m && c0 < args.n) {
          const bool full = vrow && c0 + 32 <= args.n;
#pragma unroll
          for (int h = 0; h < 32; h += 16) {
            float sv[16];
            if (ds && full) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const float4 t = *reinterpret_cast<const float4*>(arow + c0 + h + j);
                sv[j] = t.x; sv[j + 1] = t.y; sv[j + 2] = t.z; sv[j + 3] = t.w;
              }
            } else if (ds) {
#pragma unroll
              for (int j = 0; j < 16; ++j) sv[j] = c0 + h + j < args.n ? arow[c0 + h + j] : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float a = ti.nk ? __uint_as_float(r[h + j]) : 0.f;
              const float e = ds ? 0.f : __expf(__fmul_rn(alpha, a) - rv);
              r[h + j] = __float_as_uint(ds ? sv[j] * (a - rv) * alpha
                                            : ((causal && c0 + h + j > row) ? 0.f : e));
            }
            if (full) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(crow + c0 + h + j) =
                    make_float4(__uint_as_float(r[h + j]), __uint_as_float(r[h + j + 1]),
                                __uint_as_float(r[h + j + 2]), __uint_as_float(r[h + j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (c0 + h + j < args.n) crow[c0 + h + j] = __uint_as_float(r[h + j]);
            }
          }
        } else if (row < args.m && c0 < args.n) {
          if (vrow && c0 + 32 <= args.n) {
#pragma unroll
            for (int h = 0; h < 32; h += 16) {
              float4 old[4];
              if (beta != 0.f) {
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                  old[j / 4] = *reinterpret_cast<const float4*>(crow + c0 + h + j);
              }
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                float4 v;
                v.x = ti.nk ? alpha * __uint_as_float(r[h + j + 0]) : 0.f;
                v.y = ti.nk ? alpha * __uint_as_float(r[h + j + 1]) : 0.f;
                v.z = ti.nk ? alpha * __uint_as_float(r[h + j + 2]) : 0.f;
                v.w = ti.nk ? alpha * __uint_as_float(r[h + j + 3]) : 0.f;
                float4* dst = reinterpret_cast<float4*>(crow + c0 + h + j);
                if (beta != 0.f) {
                  const float4 o = old[j / 4];
                  v.x += beta * o.x; v.y += beta * o.y;
                  v.z += beta * o.z; v.w += beta * o.w;
                }
                if (bias) {
                  const float4 bb = *reinterpret_cast<const float4*>(bias + c0 + h + j);
                  v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
                }
                *dst = v;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int64_t col = c0 + j;
              if (col < args.n) {
                float* d = crow + col * cstep;
                float v = ti.nk ? alpha * __uint_as_float(r[j]) : 0.f;
                if (beta != 0.f) v += beta * *d;
                if (bias) v += bias[col];
                *d = v;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_remote(map_to_rank(&acc_empty[buf], 0));
        else mbar_arrive(&acc_empty[buf]);
      }
      ++tc;
    }
    if (lane == 0) bulk_wait_all();  // TMA stores complete before the kernel ends
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  // PAIR: neither CTA leaves (or frees TMEM) while the pair's MMAs may still read its shared
  // memory or write its TMEM.
  if (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc2(tmem, L::TMEM_COLS);
    else tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// Sum of the split partials in split order, then alpha / beta / bias into C's layout.
__global__ void __launch_bounds__(256)
splitk_reduce_kernel(const float* __restrict__ ws, int splits, GemmArgs<float> p) {
  const int64_t mn = p.m * p.n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += ws[sp * mn + i];
    const int64_t row = i / p.n, col = i % p.n;
    const int64_t off = gemm_c_offset(p, 0, row, col);
    float v = p.alpha * s;
    if (p.beta != 0.f) v += p.beta * p.c[off];
    if (p.bias) v += p.bias[col];
    p.c[off] = v;
  }
}

// The same for a plain row-major C whose rows are whole float4s: 16-byte accesses, the
// splits' loads of one vector issued together.
__global__ void __launch_bounds__(256)
splitk_reduce_vec4(const float4* __restrict__ ws, int splits, GemmArgs<float> p) {
  pdl_trigger();  // launched with launch_pdl: no global access before the wait
  pdl_wait();
  const int64_t mn4 = p.m * p.n / 4, n4 = p.n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    int sp = 0;
    for (; sp + 4 <= splits; sp += 4) {
      const float4 a = ws[sp * mn4 + i], b = ws[(sp + 1) * mn4 + i];
      const float4 c = ws[(sp + 2) * mn4 + i], d = ws[(sp + 3) * mn4 + i];
      s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
      s.x += b.x; s.y += b.y; s.z += b.z; s.w += b.w;
      s.x += c.x; s.y += c.y; s.z += c.z; s.w += c.w;
      s.x += d.x; s.y += d.y; s.z += d.z; s.w += d.w;
    }
    for (; sp < splits; ++sp) {
      const float4 a = ws[sp * mn4 + i];
      s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
    }
    const int64_t row = i / n4, c4 = i % n4;
    float4* dst = reinterpret_cast<float4*>(p.c + row * p.ldc) + c4;
    float4 v = make_float4(p.alpha * s.x, p.alpha * s.y, p.alpha * s.z, p.alpha * s.w);
    if (p.beta != 0.f) {
      const float4 o = *dst;
      v.x += p.beta * o.x; v.y += p.beta * o.y; v.z += p.beta * o.z; v.w += p.beta * o.w;
    }
    if (p.bias) {
      const float4 bb = reinterpret_cast<const float4*>(p.bias)[c4];
      v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
    }
    *dst = v;
  }
}

// Chunked 5-D maps for MN-major operands on (default) or off (TG_GEMM_CHUNKED=0, for the
// probes that compare both).
static bool chunked_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM_CHUNKED");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Column-fastest tile order where it applies (default) or never (TG_GEMM_NFAST=0, probes).
static bool nfast_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM_NFAST");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Stream-K tail on (default) or off (TG_GEMM_STREAMK=0, for the probes that compare both).
static bool streamk_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM_STREAMK");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// The stream-K partial slots and arrival counters of one (device, stream): allocated at the
// stream's first stream-K product (2 slots of 128 x 256 floats per SM, 39 MB on B200, and
// 8 counters per SM, zeroed on the stream), kept for the process. Products on one stream run
// one after another, so they share it; a stream being captured gets none (no allocation
// inside a capture) and its products run without the stream-K tail.
struct SkWorkspace {
  float* ws = nullptr;
  int* cnt = nullptr;
};

static int sk_workspace(cudaStream_t stream, SkWorkspace* out) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, SkWorkspace> cache;
  int dev = 0;
  TG_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, stream});
  if (it != cache.end()) {
    *out = it->second;
    return TG_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  TG_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
  if (cs != cudaStreamCaptureStatusNone)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: no stream-K workspace inside a capture");
  const size_t units = (size_t)sm_count();
  SkWorkspace w;
  if (cudaMalloc(&w.ws, 2 * units * BM * 256 * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&w.cnt, 2 * units * 4 * sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    if (w.ws) cudaFree(w.ws);
    return set_error(TG_ERR_OOM, "gemm_tc: stream-K workspace");
  }
  TG_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, 2 * units * 4 * sizeof(int), stream));
  cache[{dev, stream}] = w;
  *out = w;
  return TG_OK;
}

template <int BN, bool A_MN, bool B_MN, bool PAIR, bool ATM>
static int launch(const GemmArgs<float>& p, int splits, cudaStream_t stream) {
  // ATM: A in tensor memory (single CTA, K-major A); the MMAs then read only B from shared
  // memory, and the split pass writes no A lo there.
  static_assert(!ATM || (!PAIR && !A_MN), "A in tensor memory: single CTA, K-major A");
  using L = Layout<BN, PAIR, ATM>;
  static_assert(L::RST >= 3 && L::LST >= 2, "GEMM rings too shallow");
  // A lo slot is known free from the raw ring's barrier of the k-block that last used it
  // (one commit serves both rings): that barrier must not have been re-armed since.
  static_assert(L::LST <= L::RST, "the lo ring may not be deeper than the raw ring");
  constexpr int TILE_M = PAIR ? 2 * BM : BM;
  auto kernel = gemm_tc_kernel<BN, A_MN, B_MN, PAIR, ATM>;
  CUtensorMap ta, tb;
  int rc;
  // A: K-major = m rows of k; MN-major = k rows of m. Likewise B with n. An operand shared
  // by every batch entry (stride 0) gets a map of depth 1; a folded A has depth k / a_fold.
  constexpr int KB = L::BK;
  constexpr CUtensorMapSwizzle kSwK =
      KB == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  constexpr CUtensorMapSwizzle kSwMN = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const bool a_bcast = p.batch > 1 && p.stride_a == 0 && p.stride_ah == 0;
  const bool b_bcast = p.batch > 1 && p.stride_b == 0 && p.stride_bh == 0;
  const int64_t nb = p.batch / p.heads;
  const int64_t ah = a_bcast ? 1 : p.heads, an = a_bcast ? 1 : nb;
  const int64_t bh = b_bcast ? 1 : p.heads, bn = b_bcast ? 1 : nb;
  // MN-major operands whose MN extent is a multiple of 32 (no box reaches past a row) take
  // the chunked map: one copy per k-block.
  bool a_chunked = false, b_chunked = false;
  if (A_MN && p.m % 32 == 0 && chunked_enabled() &&
      make_map(&ta, p.a, p.m, p.k, p.lda, ah, p.stride_ah, an, p.stride_a, 32, KB, kSwMN,
               BM / 32) == TG_OK)
    a_chunked = true;
  if (A_MN && !a_chunked) {
    cudaGetLastError();
    rc = make_map(&ta, p.a, p.m, p.k, p.lda, ah, p.stride_ah, an, p.stride_a, 32, KB, kSwMN);
  } else if (A_MN) {
    rc = TG_OK;
  } else if (p.a_fold > 0)
    rc = make_map(&ta, p.a, p.a_fold, p.m, p.lda, 1, 0, p.k / p.a_fold, p.stride_a, KB, BM,
                  kSwK);
  else rc = make_map(&ta, p.a, p.k, p.m, p.lda, ah, p.stride_ah, an, p.stride_a, KB, BM, kSwK);
  if (rc != TG_OK) return rc;
  if (B_MN && p.n % 32 == 0 && chunked_enabled() &&
      make_map(&tb, p.b, p.n, p.k, p.ldb, bh, p.stride_bh, bn, p.stride_b, 32, KB, kSwMN,
               L::B_ROWS / 32) == TG_OK)
    b_chunked = true;
  if (B_MN && b_chunked)
    rc = TG_OK;
  else if (B_MN)
    rc = make_map(&tb, p.b, p.n, p.k, p.ldb, bh, p.stride_bh, bn, p.stride_b, 32, KB, kSwMN);
  else
    rc = make_map(&tb, p.b, p.k, p.n, p.ldb, bh, p.stride_bh, bn, p.stride_b, KB, L::B_ROWS,
                  kSwK);
  if (rc != TG_OK) return rc;
  const size_t smem = L::RINGS + kEpiBytes + 1024 + 512;
  static bool configured = false;
  static int max_pairs = 0;
  if (!configured) {
    TG_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    if (PAIR) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(2 * (sm_count() / 2));
      q.blockDim = dim3(kThreads);
      q.dynamicSmemBytes = smem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      q.attrs = at;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kernel, &q) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sm_count() / 2;
      }
      max_pairs = n;
    }
    configured = true;
  }
  TcArgs a{};
  a.m = p.m; a.n = p.n; a.k = p.k;
  a.c = p.c; a.ldc = p.ldc; a.stride_c = p.stride_c; a.bias = p.bias;
  a.alpha = p.alpha; a.beta = p.beta;
  a.kmode = p.kmode; a.raw = p.precision;
  a.m_tiles = (int)((p.m + TILE_M - 1) / TILE_M);
  a.n_tiles = (int)((p.n + BN - 1) / BN);
  a.batch = (int)p.batch;
  a.a_fold = (int)p.a_fold;
  a.a_bcast = a_bcast; a.b_bcast = b_bcast;
  a.c_hw = p.c_hw;
  a.heads = (int)p.heads;
  a.stride_ch = p.stride_ch;
  a.epi = p.epi;
  a.rv0 = p.rv0;
  a.rv1 = p.rv1;
  a.aux = p.aux;
  const int nk_all = (int)((p.k + KB - 1) / KB);
  a.splits = 1;
  a.kb_per_split = nk_all;
  if (splits > 1) {
    a.kb_per_split = (nk_all + splits - 1) / splits;
    a.splits = (nk_all + a.kb_per_split - 1) / a.kb_per_split;  // every split non-empty
    a.ws = p.workspace;
  }
  // Epilogue through shared memory and TMA stores: whole-tile outputs (no split partials,
  // no NCHW scatter, no accumulation into C) whose rows suit a tensor map.
  CUtensorMap tcm = ta, txm = ta;
  a.tma_c = 0;
  a.a_chunked = a_chunked;
  a.b_chunked = b_chunked;
  // Row-fastest order makes the SMs' concurrent tiles share a column tile, so with few column
  // tiles and many row tiles A (the larger operand) is read once per column tile: e.g. the
  // GPT-2 head's weight gradient read its 1.65 GB operand three times from DRAM (5.2 GB).
  // Unbatched products only: batched ones (the convolution's per-image input gradients)
  // measured 8 % slower over the CNN step in column-fastest order.
  a.n_fast = p.kmode == GEMM_K_FULL && a.batch == 1 && a.n_tiles > 1 && a.n_tiles <= 4 &&
             a.m_tiles >= 4 * a.n_tiles && nfast_enabled();
  {
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const bool strides_ok = p.ldc % 4 == 0 && (p.heads == 1 || p.stride_ch % 4 == 0) &&
                            (nb == 1 || p.stride_c % 4 == 0);
    const bool want = !PAIR && a.splits == 1 && p.c_hw == 0 && p.beta == 0.f && p.m >= 32 &&
                      p.n >= 32 && strides_ok && al16(p.c) &&
                      (p.epi != GEMM_EPI_SOFTMAX_DS || (p.aux && al16(p.aux)));
    if (want &&
        make_map(&tcm, p.c, p.n, p.m, p.ldc, p.heads, p.stride_ch, nb, p.stride_c, 32, 32,
                 CU_TENSOR_MAP_SWIZZLE_128B) == TG_OK &&
        (p.epi != GEMM_EPI_SOFTMAX_DS ||
         make_map(&txm, p.aux, p.n, p.m, p.ldc, p.heads, p.stride_ch, nb, p.stride_c, 32, 32,
                  CU_TENSOR_MAP_SWIZZLE_128B) == TG_OK))
      a.tma_c = 1;
  }
  const int64_t tiles = (int64_t)a.m_tiles * a.n_tiles * a.batch * a.splits;
  // Stream-K tail: when the tiles fill the SMs' last round only partly, the last one or two
  // rounds' k-blocks are shared out evenly. Modelled makespan in k-blocks: the whole rounds,
  // then the shared range and about one k-block of fix-up (partials written and summed).
  // Only for long reductions (64 k-blocks or more per tile): measured on B200, the 8192-row
  // products with k = 3072 gain 2-8 %, those with k = 768 lose 1-2 % (SMs of a part-empty
  // last round run faster than the model assumes, which shrinks what there is to win).
  if (!PAIR && a.splits == 1 && a.tma_c && p.epi == GEMM_EPI_STORE &&
      p.kmode == GEMM_K_FULL && nk_all >= 64 && streamk_enabled()) {
    const int64_t units = tiles < sm_count() ? tiles : sm_count();
    const int64_t rounds = (tiles + units - 1) / units;
    if (tiles > units && tiles % units) {
      const int64_t whole = (tiles / units - 1) * units;
      const int64_t wk = (tiles - whole) * nk_all;
      const double cost =
          (double)(whole / units * nk_all) + (double)((wk + units - 1) / units) + 1.0;
      SkWorkspace w;
      if (cost < 0.96 * (double)(rounds * nk_all)) {
        if (sk_workspace(stream, &w) == TG_OK) {
          a.sk_first = (int)whole;
          a.sk_tiles = (int)(tiles - whole);
          a.sk_nk = nk_all;
          a.sk_q = wk / units;
          a.sk_r = wk % units;
          a.sk_ws = w.ws;
          a.sk_cnt = w.cnt;
        } else {
          cudaGetLastError();
        }
      }
    }
  }
  if (PAIR) {
    const int pairs = (int)(tiles < max_pairs ? tiles : max_pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    TG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, ta, tb, tcm, txm, a));
  } else {
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    launch_pdl(kernel, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tcm, txm, a);
  }
  if (a.splits > 1) {
    const int64_t mn = p.m * p.n;
    const bool v4 = p.c_hw == 0 && p.n % 4 == 0 && p.ldc % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(p.c) & 15) == 0 &&
                    (!p.bias || (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0);
    const int64_t work = v4 ? mn / 4 : mn;
    const int blocks = (int)((work + 255) / 256 < 8 * sm_count() ? (work + 255) / 256
                                                                    : 8 * sm_count());
    if (v4)
      launch_pdl(splitk_reduce_vec4, dim3(blocks), dim3(256), 0, stream,
                 reinterpret_cast<const float4*>(p.workspace),
                                                     a.splits, p);
    else
      splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(p.workspace, a.splits, p);
    return check_launch("gemm_tc(split-k)", 2);
  }
  return check_launch(PAIR ? "gemm_tc(pair)" : "gemm_tc");
}

// A 256-wide tile with A in tensor memory keeps one accumulator (no epilogue overlap) to
// make room for A; TG_GEMM_ATM256=0|1 chooses it for the probes that decide the default.
static bool atm_wide() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM_ATM256");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

template <int BN, bool PAIR>
static int launch_any(const GemmArgs<float>& p, bool a_mn, bool b_mn, int splits,
                      cudaStream_t stream) {
  // A in tensor memory wherever the accumulators leave room (tiles up to 192 wide; 256 wide
  // only with one accumulator) and A is K-major.
  constexpr bool kAtm = !PAIR && BN <= 192;
  if (!PAIR && BN > 192 && !a_mn && atm_wide()) {
    if (!b_mn) return launch<BN, false, false, PAIR, !PAIR>(p, splits, stream);
    return launch<BN, false, true, PAIR, !PAIR>(p, splits, stream);
  }
  if (!a_mn && !b_mn) return launch<BN, false, false, PAIR, kAtm>(p, splits, stream);
  if (!a_mn && b_mn) return launch<BN, false, true, PAIR, kAtm>(p, splits, stream);
  if (a_mn && !b_mn) return launch<BN, true, false, PAIR, false>(p, splits, stream);
  return launch<BN, true, true, PAIR, false>(p, splits, stream);
}

// CTA pairs are opt-in (TG_GEMM_PAIR=1). Measured on B200 they run at about 0.9x of the
// single-CTA kernel: the in-kernel lo split makes every stage of the pair wait for a
// cross-SM hand-off (split warps -> relay -> cluster-scope acquire by the MMA issuer), which
// costs more than the halved B-operand traffic saves.
static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("TG_GEMM_PAIR");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

}  // namespace tc

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int gemm_tc_f32(const GemmArgs<float>& p, cudaStream_t stream) {
  if (p.batch < 1 || p.batch > 65535 || p.m <= 0 || p.n <= 0 || p.k <= 0)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: batch/empty shape");
  if (!aligned16(p.a) || !aligned16(p.b) || (p.lda % 4) || (p.ldb % 4))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: operands not 16-byte aligned");
  if (p.batch > 1 && ((p.stride_a % 4) || (p.stride_b % 4) || (p.stride_ah % 4) ||
                      (p.stride_bh % 4)))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: batch strides not 16-byte aligned");
  if (p.heads < 1 || p.batch % p.heads)
    return set_error(TG_ERR_ARG, "gemm_tc: batch %lld is not a multiple of heads %lld",
                     (long long)p.batch, (long long)p.heads);
  if (p.m > INT32_MAX / 2 || p.n > INT32_MAX / 2 || p.k > INT32_MAX / 2)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: dimension beyond int32");
  if (p.a_fold > 0 && (p.trans_a || p.batch != 1 || p.a_fold % 16 || p.k % p.a_fold ||
                       (p.stride_a % 4) || p.k / p.a_fold > INT32_MAX))
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: folded A needs K-major, fold %% 16 == 0");
  if (p.c_hw > 0 && p.heads != 1)
    return set_error(TG_ERR_UNSUPPORTED, "gemm_tc: NCHW output takes no heads");
  const bool a_mn = p.trans_a != 0;   // A stored k x m
  const bool b_mn = p.trans_b == 0;   // B stored k x n
  // Tile width BN and split count s chosen together by modelled makespan, in units of a
  // k-block of a 64-wide tile:
  //   ceil(tiles(BN) * s / SMs) * (ceil(nk / s) + 2 + part(BN, s)) * kb(BN)
  // kb = 7 : 8 : 10 for BN = 64 : 128 : 256 is the measured time of one k-block (B200: a
  // k-block of a narrow tile costs nearly as much as of a wide one, so wide tiles and split
  // reductions win when the output has few tiles); every tile pays about two k-blocks of
  // pipeline fill and epilogue; a split tile about 12 * BN / 256 more for writing its fp32
  // partial and reading it back in the reduction. Splits need a caller workspace (batch 1,
  // full reductions) and keep at least 8 k-blocks each.
  const int64_t mt = (p.m + tc::BM - 1) / tc::BM, sms = tc::sm_count();
  const bool can_split = p.workspace && p.batch == 1 && p.kmode == GEMM_K_FULL;
  const int64_t fit =
      can_split ? (int64_t)(p.workspace_bytes / (sizeof(float) * (size_t)(p.m * p.n))) : 1;
  // k-block depth per tile width (tc::Layout::BK) and the time of one k-block.
  auto bk_of = [](int bn) { return bn <= 128 ? 32 : 16; };
  auto kb_cost = [](int bn) { return bn == 256 ? 10.0 : (bn == 128 ? 12.0 : 10.0); };
  int best = 0, splits = 1;
  double best_cost = 0.0;
  for (int bn : {256, 128, 64}) {
    // A folded k-block stays inside one image; the 16-deep tiles always qualify.
    if (p.a_fold > 0 && p.a_fold % bk_of(bn)) continue;
    if (bn > 64 && p.n <= bn / 2 && !(bn == 256 && p.a_fold > 0 && p.a_fold % 32)) continue;
    const int64_t nk = (p.k + bk_of(bn) - 1) / bk_of(bn);
    const int64_t tiles = mt * ((p.n + bn - 1) / bn) * p.batch;
    int64_t smax = can_split ? nk / 8 : 1;
    if (smax > fit) smax = fit;
    if (smax > sms) smax = sms;
    if (smax < 1) smax = 1;
    for (int64_t sp = 1; sp <= smax; ++sp) {
      const double part = sp > 1 ? 12.0 * bn / 256.0 : 0.0;
      const double cost = (double)((tiles * sp + sms - 1) / sms) *
                          ((double)((nk + sp - 1) / sp) + 2.0 + part) * kb_cost(bn);
      if (best == 0 || cost < best_cost - 1e-9) {
        best_cost = cost;
        best = bn;
        splits = (int)sp;
      }
    }
  }
  // TG_GEMM_BN=64|128|256 pins the tile width (unsplit) for kernel probes.
  static int forced_bn = -1;
  if (forced_bn < 0) {
    const char* e = getenv("TG_GEMM_BN");
    const int v = e ? atoi(e) : 0;
    forced_bn = (v == 64 || v == 128 || v == 192 || v == 256) ? v : 0;
  }
  if (forced_bn && !(p.a_fold > 0 && p.a_fold % bk_of(forced_bn))) {
    best = forced_bn;
    splits = 1;
  }
  // CTA pairs (256-row tiles, cta_group::2) for plain single products when their makespan
  // wins. A pair tile is two single tiles' work on two SMs; with the B-operand traffic per SM
  // halved it is modelled at 3/4 of a single tile's time.
  if (splits == 1 && p.batch == 1 && p.kmode == GEMM_K_FULL && p.epi == GEMM_EPI_STORE &&
      p.a_fold == 0 && p.m > tc::BM && best >= 128 && tc::pair_enabled()) {
    const int64_t pairs = sms / 2;
    const int64_t mt2 = (p.m + 2 * tc::BM - 1) / (2 * tc::BM);
    const int64_t tiles2 = mt2 * ((p.n + best - 1) / best);
    const int64_t nk16 = (p.k + 15) / 16;  // pair tiles are 16 deep
    const double pair_cost =
        (double)((tiles2 + pairs - 1) / pairs) * ((double)nk16 + 2.0) * 10.0 * 0.75;
    if (pair_cost < best_cost) {
      if (best == 128) return tc::launch_any<128, true>(p, a_mn, b_mn, 1, stream);
      return tc::launch_any<256, true>(p, a_mn, b_mn, 1, stream);
    }
  }
  if (best == 64) return tc::launch_any<64, false>(p, a_mn, b_mn, splits, stream);
  if (best == 128) return tc::launch_any<128, false>(p, a_mn, b_mn, splits, stream);
  if (best == 192) return tc::launch_any<192, false>(p, a_mn, b_mn, splits, stream);
  return tc::launch_any<256, false>(p, a_mn, b_mn, splits, stream);
}

}  // namespace tg

extern "C" int tg_gemm_tc_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tg::tc::g_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(tg::tc::g_status, &z, sizeof(int));
  }
  return v;
}
