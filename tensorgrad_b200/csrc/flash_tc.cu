// Fused attention forward on the tensor cores for head dims 32 and 64 (ops/attention.py:71-88):
// O = softmax(scale Q K^T) V and lse per row, without storing the scores.
//
// One CTA (512 threads, persistent) per (batch-head, 128-query block) work item, key blocks of
// 64, everything in fp32 with the 3xTF32 split (hi = the raw bits, which the tensor core
// truncates; lo = x - hi):
//   warp 0 (lane 0): TMA producer: the item's Q (128 x D) once, then K and V blocks (64 x D)
//                    through a STAGES-deep ring.
//   warps 4..7     : Q's hi and lo into tensor memory (the A operand of S = Q K^T); lo of each
//                    K and V block in shared memory.
//   warp 1 (lane 0): MMA issuer: S_j = Q K_j^T into one of two TMEM score buffers, then
//                    O += P_{j-1} V_{j-1} (P from TMEM), so S_j overlaps the softmax of j-1.
//   warps 8..15    : online softmax, lane = query row, two warps per lane quarter (one per
//                    32-key half of a block, agreeing on the row max through two TMEM columns):
//                    S_j from TMEM, scale and causal / length mask, running max and sum, O
//                    rescaled in TMEM when the max grows, P_j's hi and lo into TMEM; at the end
//                    O / sum to global memory and lse = max + log(sum).
// TMEM columns: O [0, D), S [D, D + 128) (two buffers), P hi/lo [D + 128, D + 256), Q hi/lo
// [D + 256, 3 D + 256), the max exchange [3 D + 256, 3 D + 260). Every wait is bounded; on expiry the kernel records TG_ERR_TIMEOUT in
// this unit's status word, stops, drains and frees its TMEM.
#include "common.cuh"
#include "expfma.cuh"
#include "tc_ptx.cuh"

namespace tg {
namespace tc {
namespace {

constexpr int FQ = 128;  // query rows per item (TMEM lanes)
constexpr int FK = 64;   // keys per block
constexpr int kFThreads = 512;
constexpr int kSplit0 = 4, kSoft0 = 12;
// The P / dS kernel: split warps 4..7, element-wise warps 8..15.
constexpr int kPSplit0 = 4, kPElem0 = 8;

// Every kExpFmaEvery-th exponential of the softmax warps (by column, fixed at compile time)
// can run on the FMA pipe (exp_fma) instead of the XU pipe's approximate exponential; 0 =
// none. Measured on B200 (causal MHA 16 x 8 x 512 x 64, forward + backward): every 3rd
// 2648 and every 2nd 2608 calls/s against 2706 with none, so the XU pipe, although the
// busiest unit in the counters, is not what bounds these kernels, and the default is none.
#ifndef TG_EXP_FMA_EVERY
#define TG_EXP_FMA_EVERY 0
#endif
constexpr int kExpFmaEvery = TG_EXP_FMA_EVERY;

__device__ __forceinline__ float softmax_exp(float x, int c) {
  if (kExpFmaEvery > 0 && c % (kExpFmaEvery > 0 ? kExpFmaEvery : 1) == kExpFmaEvery - 1)
    return exp_fma(x);
  return __expf(x);
}

// Set only by tg_attention_set_wait_test: the forward's TMA producer then issues no load at
// all (not even the first item's Q), so the first wait on a load times out and the kernel's
// abort-and-drain path runs with nothing in flight.
__device__ int g_withhold_loads = 0;

struct FlashArgs {
  int64_t Tq, Tk, H, BH;
  int causal;
  float scale;
  float* o;
  int64_t o_sb, o_sh, o_st;
  float* lse;
  int q_blocks, items;
};

template <int D>
struct FLayout {
  static constexpr uint32_t Q_BYTES = FQ * D * 4;
  static constexpr uint32_t KV = FK * D * 4;  // one block of K or V (raw or lo)
  static constexpr uint32_t STAGE = 4 * KV;   // K raw, K lo, V raw, V lo
  static constexpr int STAGES = D == 64 ? 3 : 6;
  static constexpr uint32_t O_COL = 0, S_COL = D, P_COL = D + 2 * FK, Q_COL = D + 4 * FK;
  static constexpr uint32_t SMEM = Q_BYTES + STAGES * STAGE + 1024 + 512;
  // Columns through which the two softmax warps of a lane quarter exchange one value per row:
  // [parity][half].
  static constexpr uint32_t X_COL = 3 * D + 4 * FK;
};

__device__ __forceinline__ void item_of(const FlashArgs& a, int item, int& bh, int& qb) {
  // Longest items (last query blocks of a causal product) first.
  qb = a.q_blocks - 1 - item / (int)a.BH;
  bh = item % (int)a.BH;
}

__device__ __forceinline__ int key_blocks(const FlashArgs& a, int qb) {
  const int64_t end = a.causal ? ((int64_t)(qb + 1) * FQ < a.Tk ? (int64_t)(qb + 1) * FQ : a.Tk)
                               : a.Tk;
  return (int)((end + FK - 1) / FK);
}

template <int D>
__global__ void __launch_bounds__(kFThreads, 1)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, FlashArgs a) {
  using L = FLayout<D>;
  constexpr int ST = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* q_smem = smem;
  uint8_t* kv_smem = smem + L::Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(kv_smem + ST * L::STAGE);
  uint64_t* q_full = bars;
  uint64_t* q_ready = bars + 1;
  uint64_t* q_empty = bars + 2;
  uint64_t* p_full = bars + 3;
  uint64_t* p_empty = bars + 4;
  uint64_t* o_full = bars + 5;
  uint64_t* o_empty = bars + 6;
  uint64_t* drain = bars + 7;
  uint64_t* s_full = bars + 8;    // [2]
  uint64_t* s_empty = bars + 10;  // [2]
  uint64_t* kv_full = bars + 12;  // [ST]
  uint64_t* kv_split = kv_full + ST;
  uint64_t* kv_empty = kv_split + ST;
  uint64_t* xbar = kv_empty + ST;  // [4]: the two softmax warps of a lane quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto k_raw = [&](int s) { return kv_smem + s * L::STAGE; };
  auto k_lo = [&](int s) { return kv_smem + s * L::STAGE + L::KV; };
  auto v_raw = [&](int s) { return kv_smem + s * L::STAGE + 2 * L::KV; };
  auto v_lo = [&](int s) { return kv_smem + s * L::STAGE + 3 * L::KV; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 4);
    mbar_init(q_empty, 1);
    mbar_init(p_full, 8);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 8);
    mbar_init(drain, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 8);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_split[s], 4);
      mbar_init(&kv_empty[s], 1);
    }
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();  // launched with launch_pdl: the prologue above touches no global memory
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0, tq = 0;
      bool ok = *(volatile int*)&g_withhold_loads == 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
        int bh, qb;
        item_of(a, item, bh, qb);
        const int h = (int)(bh % a.H), b = (int)(bh / a.H);
        // Q's shared memory is free once the split warps moved the previous item's Q to TMEM.
        if (tq > 0 && !wait_bar(q_ready, (tq - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tma_load_4d(q_smem + c * FQ * 128, &tmQ, q_full, 32 * c, qb * FQ, h, b);
        const int nkb = key_blocks(a, qb);
        for (int j = 0; j < nkb; ++j, ++it) {
          const int s = it % ST, round = it / ST;
          if (round > 0 && !wait_bar(&kv_empty[s], (round - 1) & 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[s], 2 * L::KV);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_4d(k_raw(s) + c * FK * 128, &tmK, &kv_full[s], 32 * c, j * FK, h, b);
            tma_load_4d(v_raw(s) + c * FK * 128, &tmV, &kv_full[s], 32 * c, j * FK, h, b);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = instr_desc(FQ, FK, false, false);
      constexpr uint32_t idO = instr_desc(FQ, D, false, true);
      int it = 0, tq = 0, sj = 0, pj = 0;
      bool ok = true;
      // O += P V of the key block held in stage s; first: the item's first block.
      auto issue_pv = [&](int s, bool first) -> bool {
        if (!wait_bar(p_full, pj & 1, abort_flag)) return false;
        if (first && tq > 0 && !wait_bar(o_empty, (tq - 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t vr = smem_u32(v_raw(s)), vl = smem_u32(v_lo(s));
#pragma unroll
        for (int kk = 0; kk < FK / 8; ++kk) {
          const uint64_t vh = smem_desc(vr + kk * 1024, FK * 128, 512, 1);
          const uint64_t vlo = smem_desc(vl + kk * 1024, FK * 128, 512, 1);
          const uint32_t ph = tmem + L::P_COL + kk * 8, plo = ph + FK;
          mma_tf32_ta(tmem + L::O_COL, plo, vh, idO, (first && kk == 0) ? 0u : 1u);
          mma_tf32_ta(tmem + L::O_COL, ph, vlo, idO, 1);
          mma_tf32_ta(tmem + L::O_COL, ph, vh, idO, 1);
        }
        mma_commit(p_empty);
        mma_commit(&kv_empty[s]);
        ++pj;
        return true;
      };
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
        int bh, qb;
        item_of(a, item, bh, qb);
        const int nkb = key_blocks(a, qb);
        if (!wait_bar(q_ready, tq & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        int prev_s = -1;
        for (int j = 0; j < nkb; ++j, ++it) {
          const int s = it % ST, round = it / ST;
          if (!wait_bar(&kv_split[s], round & 1, abort_flag)) { ok = false; break; }
          const int b = sj & 1;
          if (sj >= 2 && !wait_bar(&s_empty[b], ((sj >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t kr = smem_u32(k_raw(s)), kl = smem_u32(k_lo(s));
          const uint32_t sacc = tmem + L::S_COL + b * FK;
#pragma unroll
          for (int kk = 0; kk < D / 8; ++kk) {
            const uint32_t off = (kk >> 2) * FK * 128 + (kk & 3) * 32;
            const uint64_t kh = smem_desc(kr + off, 16, 1024, 2);
            const uint64_t klo = smem_desc(kl + off, 16, 1024, 2);
            const uint32_t qh = tmem + L::Q_COL + kk * 8, qlo = qh + D;
            mma_tf32_ta(sacc, qlo, kh, idS, kk != 0);
            mma_tf32_ta(sacc, qh, klo, idS, 1);
            mma_tf32_ta(sacc, qh, kh, idS, 1);
          }
          mma_commit(&s_full[b]);
          ++sj;
          if (j == nkb - 1) mma_commit(q_empty);  // Q's TMEM free once these MMAs finish
          if (j > 0 && !issue_pv(prev_s, j == 1)) { ok = false; break; }
          prev_s = s;
        }
        if (!ok) break;
        if (!issue_pv(prev_s, nkb == 1)) { ok = false; break; }
        mma_commit(o_full);
      }
      if (!ok) {
        mma_commit(drain);
        wait_bar(drain, 0, abort_flag, false);
      }
    }
  } else if (warp >= kPSplit0 && warp < kPElem0) {
    const int t0 = threadIdx.x - kPSplit0 * 32;
    const int qr = warp & 3;  // lane quarter
    auto lo_of = [](float x) { return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); };
    int it = 0, tq = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
      int bh, qb;
      item_of(a, item, bh, qb);
      const int nkb = key_blocks(a, qb);
      const bool landed = wait_bar(q_full, tq & 1, abort_flag) &&
                          (tq == 0 || wait_bar(q_empty, (tq - 1) & 1, abort_flag));
      if (!__all_sync(0xffffffffu, landed)) break;
#pragma unroll
      for (int qc = 0; qc < D / 32; ++qc) {
        // Row r = 32 qr + lane of the 128-byte-swizzled box of d chunk qc: 16-byte chunk c
        // sits at c ^ (r % 8).
        const int r = 32 * qr + lane, sw = r & 7;
        const uint8_t* row = q_smem + qc * FQ * 128 + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 v0 = *reinterpret_cast<const float4*>(row + (((2 * u) ^ sw) << 4));
          const float4 v1 = *reinterpret_cast<const float4*>(row + (((2 * u + 1) ^ sw) << 4));
          const uint32_t taddr = tmem + ((uint32_t)(32 * qr) << 16) + L::Q_COL + 32 * qc + 8 * u;
          const uint32_t hi[8] = {__float_as_uint(v0.x), __float_as_uint(v0.y),
                                  __float_as_uint(v0.z), __float_as_uint(v0.w),
                                  __float_as_uint(v1.x), __float_as_uint(v1.y),
                                  __float_as_uint(v1.z), __float_as_uint(v1.w)};
          const uint32_t lo[8] = {__float_as_uint(lo_of(v0.x)), __float_as_uint(lo_of(v0.y)),
                                  __float_as_uint(lo_of(v0.z)), __float_as_uint(lo_of(v0.w)),
                                  __float_as_uint(lo_of(v1.x)), __float_as_uint(lo_of(v1.y)),
                                  __float_as_uint(lo_of(v1.z)), __float_as_uint(lo_of(v1.w))};
          tmem_st8(taddr, hi);
          tmem_st8(taddr + D, lo);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
      for (int j = 0; j < nkb; ++j, ++it) {
        const int s = it % ST, round = it / ST;
        if (!__all_sync(0xffffffffu, wait_bar(&kv_full[s], round & 1, abort_flag))) {
          ok = false;
          break;
        }
        const float4* kr = reinterpret_cast<const float4*>(k_raw(s));
        float4* kl = reinterpret_cast<float4*>(k_lo(s));
        const float4* vr = reinterpret_cast<const float4*>(v_raw(s));
        float4* vl = reinterpret_cast<float4*>(v_lo(s));
#pragma unroll
        for (int i = t0; i < (int)(L::KV / 16); i += 128) {
          const float4 x = kr[i], y = vr[i];
          kl[i] = make_float4(lo_of(x.x), lo_of(x.y), lo_of(x.z), lo_of(x.w));
          vl[i] = make_float4(lo_of(y.x), lo_of(y.y), lo_of(y.z), lo_of(y.w));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&kv_split[s]);
      }
    }
  } else if (warp >= kPElem0) {
    // Eight warps: lane quarter ew = warp % 4 (query rows), half hh of each 64-key block
    // (and of O's columns). The two warps of a quarter agree on the running max through
    // `xch` and a two-arrival barrier per exchange (bounded, like every wait here).
    const int ew = warp & 3, hh = (warp - kPElem0) >> 2;
    const uint32_t lanes = (uint32_t)(32 * ew) << 16;
    constexpr int OC = D / 2;  // O columns of this warp
    int tq = 0, sj = 0, pjs = 0, xs = 0;
    bool ok = true;
    // Exchange one value per row with the partner warp through two TMEM columns (same
    // lanes, alternating by parity so a slot is rewritten only after the partner read it);
    // returns the partner's value.
    auto exchange = [&](float v) -> float {
      const uint32_t xcol = tmem + lanes + L::X_COL + (uint32_t)((xs & 1) * 2);
      tmem_st1(xcol + hh, __float_as_uint(v));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[ew]);
      const bool got = __all_sync(0xffffffffu, wait_bar(&xbar[ew], xs & 1, abort_flag));
      ++xs;
      if (!got) {
        ok = false;
        return v;
      }
      tc_fence_after();
      return __uint_as_float(tmem_ld1(xcol + (1 - hh)));
    };
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
      int bh, qb;
      item_of(a, item, bh, qb);
      const int nkb = key_blocks(a, qb);
      const int64_t row = (int64_t)qb * FQ + 32 * ew + lane;
      float m = -INFINITY, l = 0.f;  // l: this warp's half of the row sum
      for (int j = 0; j < nkb; ++j) {
        const int b = sj & 1;
        if (!__all_sync(0xffffffffu, wait_bar(&s_full[b], (sj >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r0[32];
        tmem_ld32(tmem + lanes + L::S_COL + b * FK + 32 * hh, r0);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[b]);
        ++sj;
        const int64_t key0 = (int64_t)j * FK + 32 * hh;
        float mloc = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int64_t key = key0 + c;
          const bool valid = key < a.Tk && (!a.causal || key <= row);
          const float x = __fmul_rn(__uint_as_float(r0[c]), a.scale);
          const float v = valid ? x : -INFINITY;
          r0[c] = __float_as_uint(v);
          mloc = fmaxf(mloc, v);
        }
        mloc = fmaxf(mloc, exchange(mloc));
        if (!ok) break;
        // The running max used for the exponentials moves only when a block's max exceeds it
        // by more than 8 (a factor e^8 ~ 3e3, harmless in fp32): O and the sum are then
        // rescaled far less often. lse = max + log(sum) holds for any such max.
        const float m_new = mloc > m + 8.f ? mloc : m;
        const float corr = __expf(m - m_new);  // 0 for the first block (m = -inf), else <= 1
        float lsum = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p = softmax_exp(__uint_as_float(r0[c]) - m_new, c);
          lsum += p;
          r0[c] = __float_as_uint(p);
        }
        l = l * corr + lsum;
        m = m_new;
        // P and O are free once the previous block's O += P V has finished.
        if (pjs >= 1 && !__all_sync(0xffffffffu, wait_bar(p_empty, (pjs - 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // P first (its registers are then free), then O rescaled when the max grew.
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t hi[8], lo[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float p = __uint_as_float(r0[8 * u + e]);
            hi[e] = __float_as_uint(p);
            lo[e] = __float_as_uint(p - __uint_as_float(__float_as_uint(p) & 0xFFFFE000u));
          }
          tmem_st8(tmem + lanes + L::P_COL + 32 * hh + 8 * u, hi);
          tmem_st8(tmem + lanes + L::P_COL + FK + 32 * hh + 8 * u, lo);
        }
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
          uint32_t ov[32];
          tmem_ld32(tmem + lanes + L::O_COL + (D == 64 ? 32 * hh : 0), ov);
          if (D == 64 || hh == 0) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint32_t w[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) w[e] = __float_as_uint(__uint_as_float(ov[8 * u + e]) * corr);
              tmem_st8(tmem + lanes + L::O_COL + (D == 64 ? 32 * hh : 0) + 8 * u, w);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        ++pjs;
      }
      if (!ok) break;
      const float l_all = l + exchange(l);
      if (!ok) break;
      if (!__all_sync(0xffffffffu, wait_bar(o_full, tq & 1, abort_flag))) break;
      tc_fence_after();
      const float inv = 1.f / l_all;
      const int h = (int)(bh % a.H), b = (int)(bh / a.H);
      float* orow = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + row * a.o_st;
      {
        const int c0 = D == 64 ? 32 * hh : 0;
        uint32_t ov[32];
        tmem_ld32(tmem + lanes + L::O_COL + c0, ov);
        if (row < a.Tq && (D == 64 || hh == 0)) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(orow + c0 + e) =
                make_float4(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv,
                            __uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv);
        }
      }
      if (row < a.Tq && hh == 0) a.lse[(int64_t)bh * a.Tq + row] = m + logf(l_all);
      (void)OC;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch_flash(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                 float* o, float* lse, cudaStream_t st) {
  using L = FLayout<D>;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, q, D, s->tq, s->q_st, s->heads, s->q_sh, s->batch, s->q_sb, 32, FQ,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&mk, k, D, s->tk, s->k_st, s->heads, s->k_sh, s->batch, s->k_sb, 32, FK,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&mv, v, D, s->tk, s->v_st, s->heads, s->v_sh, s->batch, s->v_sb, 32, FK,
                     CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)))
    return rc;
  static bool configured = false;
  if (!configured) {
    TG_CUDA_TRY(cudaFuncSetAttribute(flash_fwd_kernel<D>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM));
    configured = true;
  }
  FlashArgs a{};
  a.Tq = s->tq; a.Tk = s->tk; a.H = s->heads; a.BH = s->batch * s->heads;
  a.causal = s->causal;
  a.scale = (float)(1.0 / sqrt((double)D));
  a.o = o; a.o_sb = s->o_sb; a.o_sh = s->o_sh; a.o_st = s->o_st;
  a.lse = lse;
  a.q_blocks = (int)((s->tq + FQ - 1) / FQ);
  a.items = (int)(a.BH * a.q_blocks);
  const int grid = a.items < sm_count() ? a.items : sm_count();
  launch_pdl(flash_fwd_kernel<D>, dim3(grid), dim3(kFThreads), L::SMEM, st, mq, mk, mv, a);
  return check_launch("attention forward (fused)");
}

// ------------------------------------------------------------------ backward: P and dS
// The two score products of the attention backward in one kernel: per (batch-head, 128-query
// block) item and 64-key block, S = Q K^T and dP = dO V^T into TMEM, then (lane = query row)
// P = exp(scale S - lse), dS = P (dP - delta) scale, masked like the forward, written to the
// row-major P and dS blocks (row stride ldS) that the dV, dK and dQ products read.
//   warp 0: TMA of Q and dO once per item, K and V blocks through a ring;
//   warps 4..7: Q's and dO's hi/lo into TMEM, lo of each K and V block;
//   warp 1: both products of a block into one of two TMEM buffer pairs;
//   warps 8..15: the element-wise VJP and the stores, two warps per lane quarter (one per
//   32-key half of a block).
// TMEM: S [0, 128) and dP [128, 256) (two 64-column buffers each), Q hi/lo [256, 384), dO
// hi/lo [384, 512).
struct PdsArgs {
  int64_t Tq, Tk, H, BH, ldS;
  int causal;
  float scale;
  const float* lse;
  const float* delta;
  float* P;
  float* dS;
  int q_blocks, items;
};

template <int D>
struct PLayout {
  static constexpr uint32_t Q_BYTES = FQ * D * 4;  // one of Q, dO
  static constexpr uint32_t KV = FK * D * 4;
  static constexpr uint32_t STAGE = 4 * KV;
  static constexpr int STAGES = D == 64 ? 2 : 5;
  static constexpr uint32_t S_COL = 0, DP_COL = 2 * FK, Q_COL = 4 * FK, DO_COL = 4 * FK + 2 * D;
  static constexpr uint32_t BOX = 32 * 32 * 4;  // one 32 x 32 output box
  static constexpr uint32_t STAGING = 8 * BOX;  // one box per element-wise warp
  static constexpr uint32_t SMEM = 2 * Q_BYTES + STAGES * STAGE + STAGING + 1024 + 512;
};

__device__ __forceinline__ void pds_item(const PdsArgs& a, int item, int& bh, int& qb) {
  qb = a.q_blocks - 1 - item / (int)a.BH;
  bh = item % (int)a.BH;
}

__device__ __forceinline__ int pds_blocks(const PdsArgs& a, int qb) {
  const int64_t end = a.causal ? ((int64_t)(qb + 1) * FQ < a.Tk ? (int64_t)(qb + 1) * FQ : a.Tk)
                               : a.Tk;
  return (int)((end + FK - 1) / FK);
}

template <int D>
__global__ void __launch_bounds__(kFThreads, 1)
attn_pds_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmO,
                const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmS,
                PdsArgs a) {
  using L = PLayout<D>;
  constexpr int ST = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* q_smem = smem;
  uint8_t* do_smem = smem + L::Q_BYTES;
  uint8_t* kv_smem = smem + 2 * L::Q_BYTES;
  uint8_t* staging = kv_smem + ST * L::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + L::STAGING);
  uint64_t* q_full = bars;
  uint64_t* q_ready = bars + 1;
  uint64_t* q_empty = bars + 2;
  uint64_t* drain = bars + 3;
  uint64_t* sd_full = bars + 4;   // [2]
  uint64_t* sd_empty = bars + 6;  // [2]
  uint64_t* kv_full = bars + 8;   // [ST]
  uint64_t* kv_split = kv_full + ST;
  uint64_t* kv_empty = kv_split + ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_empty + ST);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto k_raw = [&](int s) { return kv_smem + s * L::STAGE; };
  auto k_lo = [&](int s) { return kv_smem + s * L::STAGE + L::KV; };
  auto v_raw = [&](int s) { return kv_smem + s * L::STAGE + 2 * L::KV; };
  auto v_lo = [&](int s) { return kv_smem + s * L::STAGE + 3 * L::KV; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 4);
    mbar_init(q_empty, 1);
    mbar_init(drain, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sd_full[b], 1);
      mbar_init(&sd_empty[b], 8);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_split[s], 4);
      mbar_init(&kv_empty[s], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();  // launched with launch_pdl: the prologue above touches no global memory
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0, tq = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
        int bh, qb;
        pds_item(a, item, bh, qb);
        const int h = (int)(bh % a.H), b = (int)(bh / a.H);
        if (tq > 0 && !wait_bar(q_ready, (tq - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, 2 * L::Q_BYTES);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          tma_load_4d(q_smem + c * FQ * 128, &tmQ, q_full, 32 * c, qb * FQ, h, b);
          tma_load_4d(do_smem + c * FQ * 128, &tmO, q_full, 32 * c, qb * FQ, h, b);
        }
        const int nkb = pds_blocks(a, qb);
        for (int j = 0; j < nkb; ++j, ++it) {
          const int s = it % ST, round = it / ST;
          if (round > 0 && !wait_bar(&kv_empty[s], (round - 1) & 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[s], 2 * L::KV);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_4d(k_raw(s) + c * FK * 128, &tmK, &kv_full[s], 32 * c, j * FK, h, b);
            tma_load_4d(v_raw(s) + c * FK * 128, &tmV, &kv_full[s], 32 * c, j * FK, h, b);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = instr_desc(FQ, FK, false, false);
      int it = 0, tq = 0, sj = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
        int bh, qb;
        pds_item(a, item, bh, qb);
        const int nkb = pds_blocks(a, qb);
        if (!wait_bar(q_ready, tq & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int j = 0; j < nkb; ++j, ++it) {
          const int s = it % ST, round = it / ST;
          if (!wait_bar(&kv_split[s], round & 1, abort_flag)) { ok = false; break; }
          const int b = sj & 1;
          if (sj >= 2 && !wait_bar(&sd_empty[b], ((sj >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t kr = smem_u32(k_raw(s)), kl = smem_u32(k_lo(s));
          const uint32_t vr = smem_u32(v_raw(s)), vl = smem_u32(v_lo(s));
          const uint32_t sacc = tmem + L::S_COL + b * FK, dacc = tmem + L::DP_COL + b * FK;
#pragma unroll
          for (int kk = 0; kk < D / 8; ++kk) {
            const uint32_t off = (kk >> 2) * FK * 128 + (kk & 3) * 32;
            const uint64_t kh = smem_desc(kr + off, 16, 1024, 2);
            const uint64_t klo = smem_desc(kl + off, 16, 1024, 2);
            const uint64_t vh = smem_desc(vr + off, 16, 1024, 2);
            const uint64_t vlo = smem_desc(vl + off, 16, 1024, 2);
            const uint32_t qh = tmem + L::Q_COL + kk * 8, qlo = qh + D;
            const uint32_t oh = tmem + L::DO_COL + kk * 8, olo = oh + D;
            mma_tf32_ta(sacc, qlo, kh, idS, kk != 0);
            mma_tf32_ta(sacc, qh, klo, idS, 1);
            mma_tf32_ta(sacc, qh, kh, idS, 1);
            mma_tf32_ta(dacc, olo, vh, idS, kk != 0);
            mma_tf32_ta(dacc, oh, vlo, idS, 1);
            mma_tf32_ta(dacc, oh, vh, idS, 1);
          }
          mma_commit(&sd_full[b]);
          mma_commit(&kv_empty[s]);
          ++sj;
          if (j == nkb - 1) mma_commit(q_empty);
        }
      }
      if (!ok) {
        mma_commit(drain);
        wait_bar(drain, 0, abort_flag, false);
      }
    }
  } else if (warp >= kPSplit0 && warp < kPElem0) {
    const int t0 = threadIdx.x - kPSplit0 * 32;
    const int qr = warp & 3;
    auto lo_of = [](float x) { return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); };
    int it = 0, tq = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++tq) {
      int bh, qb;
      pds_item(a, item, bh, qb);
      const int nkb = pds_blocks(a, qb);
      const bool landed = wait_bar(q_full, tq & 1, abort_flag) &&
                          (tq == 0 || wait_bar(q_empty, (tq - 1) & 1, abort_flag));
      if (!__all_sync(0xffffffffu, landed)) break;
#pragma unroll
      for (int qc = 0; qc < D / 32; ++qc) {
        const int r = 32 * qr + lane, sw = r & 7;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const uint8_t* row = (which ? do_smem : q_smem) + qc * FQ * 128 + r * 128;
          const uint32_t col0 = which ? L::DO_COL : L::Q_COL;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float4 v0 = *reinterpret_cast<const float4*>(row + (((2 * u) ^ sw) << 4));
            const float4 v1 = *reinterpret_cast<const float4*>(row + (((2 * u + 1) ^ sw) << 4));
            const uint32_t taddr = tmem + ((uint32_t)(32 * qr) << 16) + col0 + 32 * qc + 8 * u;
            const uint32_t hi[8] = {__float_as_uint(v0.x), __float_as_uint(v0.y),
                                    __float_as_uint(v0.z), __float_as_uint(v0.w),
                                    __float_as_uint(v1.x), __float_as_uint(v1.y),
                                    __float_as_uint(v1.z), __float_as_uint(v1.w)};
            const uint32_t lo[8] = {__float_as_uint(lo_of(v0.x)), __float_as_uint(lo_of(v0.y)),
                                    __float_as_uint(lo_of(v0.z)), __float_as_uint(lo_of(v0.w)),
                                    __float_as_uint(lo_of(v1.x)), __float_as_uint(lo_of(v1.y)),
                                    __float_as_uint(lo_of(v1.z)), __float_as_uint(lo_of(v1.w))};
            tmem_st8(taddr, hi);
            tmem_st8(taddr + D, lo);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
      for (int j = 0; j < nkb; ++j, ++it) {
        const int s = it % ST, round = it / ST;
        if (!__all_sync(0xffffffffu, wait_bar(&kv_full[s], round & 1, abort_flag))) {
          ok = false;
          break;
        }
        const float4* kr = reinterpret_cast<const float4*>(k_raw(s));
        float4* kl = reinterpret_cast<float4*>(k_lo(s));
        const float4* vr = reinterpret_cast<const float4*>(v_raw(s));
        float4* vl = reinterpret_cast<float4*>(v_lo(s));
#pragma unroll
        for (int i = t0; i < (int)(L::KV / 16); i += 128) {
          const float4 x = kr[i], y = vr[i];
          kl[i] = make_float4(lo_of(x.x), lo_of(x.y), lo_of(x.z), lo_of(x.w));
          vl[i] = make_float4(lo_of(y.x), lo_of(y.y), lo_of(y.z), lo_of(y.w));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&kv_split[s]);
      }
    }
  } else if (warp >= kPElem0) {
    // Eight warps: lane quarter warp % 4 (rows), half hh of the 64 keys of a block.
    const int ew = warp & 3, hh = (warp - kPElem0) >> 2;
    const uint32_t lanes = (uint32_t)(32 * ew) << 16;
    float4* box = reinterpret_cast<float4*>(staging + (warp - kPElem0) * L::BOX);
    int tq = 0, sj = 0;
    for (int item = blockIdx.x; item < a.items; item += gridDim.x, ++tq) {
      int bh, qb;
      pds_item(a, item, bh, qb);
      const int nkb = pds_blocks(a, qb);
      const int row0 = qb * FQ + 32 * ew;
      const int64_t row = (int64_t)row0 + lane;
      const bool live = row < a.Tq;
      const float lse_r = live ? a.lse[bh * a.Tq + row] : 0.f;
      const float delta_r = live ? a.delta[bh * a.Tq + row] : 0.f;
      bool ok = true;
      for (int j = 0; j < nkb; ++j) {
        const int b = sj & 1;
        if (!__all_sync(0xffffffffu, wait_bar(&sd_full[b], (sj >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int64_t key0 = (int64_t)j * FK + 32 * hh;
        uint32_t sv[32], dv[32];
        tmem_ld32(tmem + lanes + L::S_COL + b * FK + 32 * hh, sv);
        tmem_ld32(tmem + lanes + L::DP_COL + b * FK + 32 * hh, dv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sd_empty[b]);
        ++sj;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int64_t key = key0 + c;
          const bool valid = key < a.Tk && (!a.causal || key <= row);
          const float e = softmax_exp(__fmul_rn(__uint_as_float(sv[c]), a.scale) - lse_r, c);
          const float p = valid ? e : 0.f;
          sv[c] = __float_as_uint(p);
          dv[c] = __float_as_uint(p * (__uint_as_float(dv[c]) - delta_r) * a.scale);
        }
        // 32 x 32 boxes of P, then dS, through this warp's shared-memory box (128-byte
        // swizzle: lane = row, 16-byte chunk k at k ^ (lane % 8)) and one TMA store each;
        // rows and keys past the product are clipped by the maps.
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const uint32_t* v = which ? dv : sv;
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
#pragma unroll
          for (int kq = 0; kq < 8; ++kq)
            box[lane * 8 + (kq ^ (lane & 7))] =
                make_float4(__uint_as_float(v[4 * kq]), __uint_as_float(v[4 * kq + 1]),
                            __uint_as_float(v[4 * kq + 2]), __uint_as_float(v[4 * kq + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < a.Tq) {
            tma_store_4d(which ? &tmS : &tmP, box, (int)key0, row0, 0, bh);
            bulk_commit();
          }
        }
      }
      if (!ok) break;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch_pds(const tg_attn_shape* s, const float* q, const float* k, const float* v,
               const float* dout, const float* lse, const float* delta, float* P, float* dS,
               int64_t ldS, cudaStream_t st) {
  using L = PLayout<D>;
  CUtensorMap mq, mo, mk, mv;
  int rc;
  if ((rc = make_map(&mq, q, D, s->tq, s->q_st, s->heads, s->q_sh, s->batch, s->q_sb, 32, FQ,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&mo, dout, D, s->tq, s->o_st, s->heads, s->o_sh, s->batch, s->o_sb, 32, FQ,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&mk, k, D, s->tk, s->k_st, s->heads, s->k_sh, s->batch, s->k_sb, 32, FK,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&mv, v, D, s->tk, s->v_st, s->heads, s->v_sh, s->batch, s->v_sb, 32, FK,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  // P and dS: (B*H) blocks of Tq rows x Tk keys, row stride ldS.
  CUtensorMap mp, md;
  const int64_t bh = s->batch * s->heads;
  if ((rc = make_map(&mp, P, s->tk, s->tq, ldS, 1, 0, bh, s->tq * ldS, 32, 32,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map(&md, dS, s->tk, s->tq, ldS, 1, 0, bh, s->tq * ldS, 32, 32,
                     CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  static bool configured = false;
  if (!configured) {
    TG_CUDA_TRY(cudaFuncSetAttribute(attn_pds_kernel<D>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM));
    configured = true;
  }
  PdsArgs a{};
  a.Tq = s->tq; a.Tk = s->tk; a.H = s->heads; a.BH = s->batch * s->heads; a.ldS = ldS;
  a.causal = s->causal;
  a.scale = (float)(1.0 / sqrt((double)D));
  a.lse = lse; a.delta = delta; a.P = P; a.dS = dS;
  a.q_blocks = (int)((s->tq + FQ - 1) / FQ);
  a.items = (int)(a.BH * a.q_blocks);
  const int grid = a.items < sm_count() ? a.items : sm_count();
  launch_pdl(attn_pds_kernel<D>, dim3(grid), dim3(kFThreads), L::SMEM, st, mq, mo, mk, mv, mp,
             md, a);
  return check_launch("attention backward (P, dS)");
}

}  // namespace
}  // namespace tc

// The fused forward takes fp32 heads of 32 or 64 features with the tensor-core path's
// layout rules (16-byte strides and bases), at least one key, and a bounded item count.
// The causal mask of both fused kernels is `key <= query` (aligned at the top left), which
// is the reference's `key <= query + tk - tq` only when tq == tk; other causal shapes go to
// the batched-GEMM path, which applies the shift.
bool flash_fwd_supported(const tg_attn_shape* s) {
  return (s->head_dim == 32 || s->head_dim == 64) && s->tk >= 1 && s->tq >= 1 &&
         (!s->causal || s->tq == s->tk) &&
         s->batch * s->heads * ((s->tq + 127) / 128) < (int64_t)1 << 30;
}

int flash_fwd_tc(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                 float* o, float* lse, cudaStream_t st) {
  if (s->head_dim == 32) return tc::launch_flash<32>(s, q, k, v, o, lse, st);
  return tc::launch_flash<64>(s, q, k, v, o, lse, st);
}

// P and dS of the attention backward (row stride ldS), same shapes as the fused forward.
int attn_pds_tc(const tg_attn_shape* s, const float* q, const float* k, const float* v,
                const float* dout, const float* lse, const float* delta, float* P, float* dS,
                int64_t ldS, cudaStream_t st) {
  if (s->head_dim == 32) return tc::launch_pds<32>(s, q, k, v, dout, lse, delta, P, dS, ldS, st);
  return tc::launch_pds<64>(s, q, k, v, dout, lse, delta, P, dS, ldS, st);
}

}  // namespace tg

// The fused attention kernels' timeout record (this unit's status word); reset when asked.
extern "C" int tg_attention_tc_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tg::tc::g_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(tg::tc::g_status, &z, sizeof(int));
  }
  return v;
}

// Test support for the bounded waits of the fused attention kernels (no reference
// counterpart): a wait budget in clock cycles (<= 0 restores the default of about two
// seconds) and, with withhold_loads != 0, a forward whose producer issues no load, so that
// the first wait on a load runs out, the kernel records TG_ERR_TIMEOUT and drains.
// Synchronous; affects later launches of this unit's kernels only.
namespace tg {
namespace tc {
namespace {
__global__ void exp_fma_test_kernel(const float* __restrict__ x, float* __restrict__ y,
                                    int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = exp_fma(x[i]);
}
}  // namespace
}  // namespace tc
}  // namespace tg

// Test-only: y = exp_fma(x) elementwise (the FMA-pipe exponential of the fused kernels).
extern "C" int tg_test_exp_fma(int64_t n, const float* x, float* y, void* stream) {
  TG_CHECK_ARG(n >= 0 && (n == 0 || (x && y)), "tg_test_exp_fma: bad arguments");
  if (n == 0) return TG_OK;
  const int64_t blocks = (n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184;
  tg::tc::exp_fma_test_kernel<<<(int)blocks, 256, 0, tg::as_stream(stream)>>>(x, y, n);
  return tg::check_launch("exp_fma test");
}

extern "C" int tg_attention_set_wait_test(int64_t budget_cycles, int withhold_loads) {
  const long long b = budget_cycles > 0 ? (long long)budget_cycles : tg::tc::kTimeoutCycles;
  const int w = withhold_loads ? 1 : 0;
  TG_CUDA_TRY(cudaMemcpyToSymbol(tg::tc::g_wait_budget, &b, sizeof(b)));
  TG_CUDA_TRY(cudaMemcpyToSymbol(tg::tc::g_withhold_loads, &w, sizeof(w)));
  return TG_OK;
}
