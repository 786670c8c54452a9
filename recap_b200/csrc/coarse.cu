// Corrected coarse tail on sm_100a tensor cores.
//
// For a 128-row query block i of bank b (rows < rows), every omitted key block j
// (partition[b][i][j] == 0, j < nB) enters a softmax with the logit
//     s q.kbar_j + ln n_j + [ s^2/2 (qsq . w_j)  if s^2 (qsq . w_j) <= theta^2 ]
// and the output is  o + g * drift,  with g the gated share of the mass
// (_coarse_tail_kernel, recap/kernels/coarse_tail.py:36-186, and its wrapper
// 194-312).  qsq = (Q U)^2 and drift = s Q C_vk^T (rotated_query_square and
// value_drift, recap/sparse/closure.py:84-93) are computed here from the Q tile
// with tcgen05 MMAs and never reach HBM.  Rounding follows the reference: kbar,
// vbar, w, U and C_vk in bf16, qsq and drift rounded to bf16 as the bf16 bmm outputs
// they replace, P rounded to bf16 before P vbar, the output rounded to bf16 and the
// drift added in bf16 arithmetic.
//
// Rank folding: with 0 < rank and rank + 4 <= 64, the per-block variances w_j are
// folded (recap/sparse/closure.py:96-104): every column c >= rank holds the same tail
// value.  Then  qsq . w_j = sum_{c<rank} qsq_c w_jc + w_j,rank * T  with
// T = sum_{c>=rank} qsq_c, and the quadratic term is one MMA over K = 16 (rank <= 12):
// the A row is (qsq_0 .. qsq_{rank-1}, T0_hi, T0_lo, T1_hi, T1_lo, 0 ...) with T0 and T1
// the two column halves' partial tails, each split into two bf16 parts (hi + lo equals
// the part to 2^-17), the B row the first 16 folded columns of w_j (columns rank ..
// rank + 3 all hold the tail).  Otherwise the product runs over all D columns.
//
// The omitted set is a mask over all nB block means, processed in tiles of 128
// (kbar, w and vbar^T of a bank stay in L2).  One CTA per (query block, bank),
// 12 warps:
//   warp 0      TMA producer of Q, U^T (prologue), the (kbar, w) tiles and C_vk;
//   warp 1      TMEM allocator and MMA issuer;
//   warp 2      TMA producer of the vbar^T tiles;
//   warps 4-11  two threads per query row (warps w and w + 4 share TMEM lanes), each
//               with half of every tile's 64-block halves and half of the head
//               dimension: qsq, the gated online softmax (log2 domain, lazy rescaling
//               of O, the row maximum exchanged between the halves every tile), P
//               into TMEM, the epilogue.  Two softmax warps per SM sub-partition hide
//               each other's latencies.
// TMEM: S1 = Q kbar^T double-buffered in columns [0,128) and [128,256), S2 = qsq w^T
// in [256,384), O in [384,384+D).  Q U goes to the O columns before the first P.V,
// and the drift Q C_vk^T to the S2 columns after the last S2 has been read.  P
// (bf16) overwrites the first 64 columns of its S1 buffer and is the A operand of
// O += P vbar from TMEM; S1(j+2) reuses that buffer only after P.V(j), issued
// before it by the same thread.  The softmax reads S2(j) first and releases it, so
// S2(j+1) and the products of the previous tile run while it computes.
// The epilogue also writes the per-block sum of (lse - old_lse) for the drift centre
// (recap/operator.py:148-150).
// Two paths per tile: a tile whose logits provably stay within kBoundSlack of every row's
// running max (|q| |kbar| bound, per warp) runs one pass (logit, gate, exponential, sums
// and P per element); any other tile forms all its logits, exchanges the row maximum
// between the two halves, rescales O if needed, then exponentiates.
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

constexpr int kThreads = 384;
constexpr int kSoftmaxWarp0 = 4;
constexpr int kTileN = 128;         // block means per tile
constexpr int kMaxBlocks = 2048;    // nB_pad limit (column terms in shared memory)
constexpr float kRescaleThreshold = 8.0f;
constexpr float kLog2e = 1.4426950408889634f;
// Largest logit excess over the running max (log2 units) the bounded path accepts
// (exponentials below 2^64 stay finite in fp32 and bf16 with room for the sums).
constexpr float kBoundSlack = 64.0f;
// Column pairs (of the 16 in every 32-column chunk) whose exponentials come from the
// FP32-pipe polynomial instead of MUFU: an eighth (tail 4.07 -> 4.00 ms on the bench
// workload; a quarter 4.02, 3/8 4.07).
constexpr uint32_t kCoarsePolyPairs = 0x0101u;

// FOLD: the quadratic term over K = 16 * k2 <= 64 (one 64-column atom of w);
// otherwise over all D columns.
template <int D, bool FOLD>
struct CoarseSmem {
  static constexpr int kTileQ = 128 * D * 2;
  static constexpr int kQsqBytes = FOLD ? 128 * 128 : kTileQ;  // A operand of S2
  static constexpr int kOpK = kTileN * D * 2;                  // kbar tile: 128 rows x D
  static constexpr int kOpW = FOLD ? kTileN * 128 : kTileN * D * 2;
  static constexpr int kKW = kOpK + kOpW;                      // one (kbar, w) stage
  static constexpr int kOpV = D * kTileN * 2;                  // one vbar^T stage: D rows x 128
  static constexpr int kKWStages = (D == 128 && !FOLD) ? 1 : 2;
  static constexpr int kVStages = 2;
  static constexpr int kQ = 0;
  static constexpr int kQsq = kQ + kTileQ;
  static constexpr int kKWRing = kQsq + kQsqBytes;
  static constexpr int kVRing = kKWRing + kKWStages * kKW;
  static constexpr int kCol = kVRing + kVStages * kOpV;       // fp32 column terms [kMaxBlocks]
  static constexpr int kTileKn = kCol + kMaxBlocks * 4;  // largest |kbar| per tile [kMaxBlocks / 128]
  static constexpr int kXchg = kTileKn + (kMaxBlocks / 128) * 4;  // row maxima [2 slots][2 halves][128]
  static constexpr int kSums = kXchg + 2 * 2 * 128 * 4;  // (l, g) per half [2][2][128], then T partials [128]
  static constexpr int kBars = kSums + (2 * 2 * 128 + 128) * 4;
  // pro_full, pro_mma, qsq_ready, kw_full[2], kw_empty[2], v_full[2], v_empty[2],
  // s1full[2], s2full, s2free, pfull[2], ofull, c_full, xfull, done, xsum, xchg[2 slots][4 quarters],
  // ofin
  static constexpr int kNumBars = 3 + 8 + 2 + 2 + 6 + 1 + 8 + 1;
  static constexpr int kMisc = kBars + kNumBars * 8;
  static constexpr int kTotal = kMisc + 16 + 4 * 4;
  static_assert(kOpV >= D * D * 2, "U^T is staged in a vbar^T slot");
  static_assert(kKW >= D * D * 2, "C_vk is staged in a (kbar, w) slot");
};

// Phase discipline: a waiter tests an mbarrier phase by its parity, which tells the current
// phase from the one before it only; a wait is sound only where the waiter can never be
// two phases behind the barrier.  So a barrier that completes once per tile is waited on
// only by a role that cannot fall two tiles behind it, and the epilogue's wait for the
// last P.V has its own single-phase barrier (ofin): ofull completes once per P.V, and
// the last two P.V can still run when the epilogue starts.  pfull is double-buffered by
// the S1 buffer holding P: the softmax arrives on pfull[j & 1] for tile j + 2 only after
// S1(j + 2), which the MMA warp issues after it has waited for pfull[j & 1] of tile j.
struct CoarseBars {
  uint64_t *pro_full, *pro_mma, *qsq_ready, *kw_full, *kw_empty, *v_full, *v_empty, *s1full, *s2full, *s2free,
      *pfull, *ofull, *c_full, *xfull, *done, *xchg, *xsum, *ofin;
};

__device__ __forceinline__ CoarseBars carve(uint8_t* base) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  CoarseBars r;
  r.pro_full = b;
  r.pro_mma = b + 1;
  r.qsq_ready = b + 2;
  r.kw_full = b + 3;
  r.kw_empty = b + 5;
  r.v_full = b + 7;
  r.v_empty = b + 9;
  r.s1full = b + 11;
  r.s2full = b + 13;
  r.s2free = b + 14;
  r.pfull = b + 15;  // [S1 buffer]
  r.ofull = b + 17;
  r.c_full = b + 18;
  r.xfull = b + 19;
  r.done = b + 20;
  r.xsum = b + 21;
  r.xchg = b + 22;  // [slot * 4 + lane quarter]
  r.ofin = b + 30;
  return r;
}

template <int D, bool FOLD>
__global__ void __launch_bounds__(kThreads, 1)
    coarse_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_ut,
                  const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_kbar,
                  const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_vbt,
                  const CoarseArgs a) {
  using L = CoarseSmem<D, FOLD>;
  constexpr int KWS = L::kKWStages;
  constexpr int VS = L::kVStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sQsq = smem + L::kQsq;
  uint8_t* sKW = smem + L::kKWRing;
  uint8_t* sV = smem + L::kVRing;
  float* colterm = reinterpret_cast<float*>(smem + L::kCol);
  float* rowmax = reinterpret_cast<float*>(smem + L::kXchg);
  float* tile_kn = reinterpret_cast<float*>(smem + L::kTileKn);
  float* rowsums = reinterpret_cast<float*>(smem + L::kSums);
  CoarseBars bars = carve(smem + L::kBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  float* row_part = reinterpret_cast<float*>(smem + L::kMisc + 16);

  const int qb = blockIdx.x;
  const int bank = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nB = a.nB;
  const int n_tiles = a.nB_pad / kTileN;
  // K-steps of the quadratic term
  const int k2 = FOLD ? (a.rank + 4 + 15) / 16 : D / 16;

  if (threadIdx.x == 0) {
    mbar_init(bars.pro_full, 1);
    mbar_init(bars.pro_mma, 1);
    mbar_init(bars.qsq_ready, 8);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bars.kw_full + s, 1);
      mbar_init(bars.kw_empty + s, 1);
      mbar_init(bars.v_full + s, 1);
      mbar_init(bars.v_empty + s, 1);
      mbar_init(bars.s1full + s, 1);
    }
    mbar_init(bars.s2full, 1);
    mbar_init(bars.s2free, 8);
    mbar_init(bars.pfull, 8);
    mbar_init(bars.pfull + 1, 8);
    mbar_init(bars.ofin, 1);
    for (int i = 0; i < 8; ++i) mbar_init(bars.xchg + i, 2);  // the two warps of a lane quarter
    mbar_init(bars.xsum, 8);
    mbar_init(bars.ofull, 1);
    mbar_init(bars.c_full, 1);
    mbar_init(bars.xfull, 1);
    mbar_init(bars.done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    // the Q tile and U^T depend on nothing computed here: start their loads first
    const uint64_t stream = l2_evict_first();  // the Q tile: read once here
    const int qrow = bank * a.S_pad + qb * 128;
    mbar_expect_tx(bars.pro_full, L::kTileQ + D * D * 2);
#pragma unroll
    for (int at = 0; at < D / 64; ++at) {
      tma_load_2d_hint(sQ + at * 128 * 128, &tm_q, bars.pro_full, at * 64, qrow, stream);
      // U^T waits in the second vbar^T slot, which the second tile needs last
      tma_load_2d(sV + (1 % VS) * L::kOpV + at * D * 128, &tm_ut, bars.pro_full, at * 64, bank * D);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  if (threadIdx.x < kMaxBlocks / 128) tile_kn[threadIdx.x] = 0.f;
  if (FOLD) {
    // the folded quadratic term's A tile: the columns past the tails stay zero
    for (int i = threadIdx.x; i < L::kQsqBytes / 16; i += kThreads)
      reinterpret_cast<uint4*>(sQsq)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_async_smem();
  }
  __syncthreads();
  {
    // per-column term (log2 units): ln n_j for omitted blocks, -inf for kept or padding;
    // the largest |bf16(kbar_j)| of every tile of 128 block means
    const uint8_t* prow = a.partition + (static_cast<size_t>(bank) * nB + qb) * nB;
    const float* kmn = a.k_mean_norm ? a.k_mean_norm + static_cast<size_t>(bank) * nB : nullptr;
    // every load of this thread first (one latency), then the column terms
    constexpr int kPer = (kMaxBlocks + kThreads - 1) / kThreads;
    uint8_t pr[kPer];
    float cl[kPer], kv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = i * kThreads + threadIdx.x;
      const bool in = j < nB;
      pr[i] = in ? prow[j] : 1;
      cl[i] = in ? a.counts_log[j] : 0.f;
      kv[i] = (in && kmn != nullptr) ? kmn[j] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int base = i * kThreads;
      if (base >= a.nB_pad) break;
      const int j = base + threadIdx.x;
      float kn = kv[i];
      if (j < a.nB_pad) colterm[j] = (j < nB && pr[i] == 0) ? cl[i] * kLog2e : -INFINITY;
      if (kmn != nullptr) {
        // one warp's 32 blocks lie in one tile (128 and kThreads are multiples of 32)
        for (int o = 16; o > 0; o >>= 1) kn = fmaxf(kn, __shfl_xor_sync(0xffffffffu, kn, o));
        if ((threadIdx.x & 31) == 0 && j < a.nB_pad)
          atomicMax(reinterpret_cast<int*>(tile_kn + j / kTileN), __float_as_int(kn));  // kn >= 0
      }
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s1 = tmem;          // two S1 buffers (P aliases their first 64 columns)
  const uint32_t t_s2 = tmem + 256;    // S2; the drift at the end
  const uint32_t t_o = tmem + 384;     // O; Q U in the prologue

  if (warp == 0) {
    // ================================================================ Q, U^T, (kbar, w), C_vk
    if (lane == 0) {
      const uint64_t keep = l2_evict_last();    // per-bank operands: read by every query block
      bool ok = true;
      int j = 0;
      for (; ok && j < n_tiles; ++j) {
        const int st = j % KWS;
        if (j >= KWS &&
            !mbar_wait(bars.kw_empty + st, ((j / KWS) - 1) & 1, abort_flag, a.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* base = sKW + st * L::kKW;
        const int brow = bank * a.nB_pad + j * kTileN;
        mbar_expect_tx(bars.kw_full + st, L::kKW);
#pragma unroll
        for (int at = 0; at < D / 64; ++at)
          tma_load_2d_hint(base + at * kTileN * 128, &tm_kbar, bars.kw_full + st, at * 64, brow, keep);
#pragma unroll
        for (int at = 0; at < (FOLD ? 1 : D / 64); ++at)
          tma_load_2d_hint(base + L::kOpK + at * kTileN * 128, &tm_w, bars.kw_full + st, at * 64, brow, keep);
      }
      // C_vk into the (kbar, w) slot that the tile after the last would use
      int loads = j;
      if (ok) {
        const int st = n_tiles % KWS;
        if (n_tiles >= KWS &&
            !mbar_wait(bars.kw_empty + st, ((n_tiles / KWS) - 1) & 1, abort_flag, a.status, kStatusTimeoutProducer))
          ok = false;
        if (ok) {
          mbar_expect_tx(bars.c_full, D * D * 2);
#pragma unroll
          for (int at = 0; at < D / 64; ++at)
            tma_load_2d(sKW + st * L::kKW + at * D * 128, &tm_c, bars.c_full, at * 64, bank * D);
          mbar_drain(bars.c_full, 0);
        }
      }
      const int first = loads > KWS ? loads - KWS : 0;
      for (int k = first; k < loads; ++k) mbar_drain(bars.kw_full + (k % KWS), (k / KWS) & 1);
      mbar_drain(bars.pro_full, 0);
    }
  } else if (warp == 2) {
    // ================================================================ vbar^T tiles
    if (lane == 0) {
      const uint64_t keep = l2_evict_last();
      bool ok = true;
      int j = 0;
      for (; ok && j < n_tiles; ++j) {
        const int st = j % VS;
        if (j >= VS) {
          ok = mbar_wait(bars.v_empty + st, ((j / VS) - 1) & 1, abort_flag, a.status, kStatusTimeoutProducer);
        } else if (st == 1 % VS) {
          // the slot still holds U^T until the prologue MMA has read it
          ok = mbar_wait(bars.pro_mma, 0, abort_flag, a.status, kStatusTimeoutProducer);
        }
        if (!ok) break;
        uint8_t* base = sV + st * L::kOpV;
        mbar_expect_tx(bars.v_full + st, L::kOpV);
#pragma unroll
        for (int at = 0; at < kTileN / 64; ++at)
          tma_load_2d_hint(base + at * D * 128, &tm_vbt, bars.v_full + st, j * kTileN + at * 64, bank * D, keep);
      }
      const int first = j > VS ? j - VS : 0;
      for (int k = first; k < j; ++k) mbar_drain(bars.v_full + (k % VS), (k / VS) & 1);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    // The whole warp runs the issue sequence (converged, uniform values); one elected
    // lane issues every MMA and commit.
    {
      const uint32_t leader = elect_leader();
      const uint32_t q0 = smem_u32(sQ), qs0 = smem_u32(sQsq), kw0 = smem_u32(sKW), v0 = smem_u32(sV);
      auto wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, a.status, code));
      };
      bool ok = wait(bars.pro_full, 0, kStatusTimeoutTma);
      if (ok) {
        // Q U into the O columns
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, D);
        const uint32_t ut = v0 + (1 % VS) * L::kOpV;
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t offb = (s >> 2) * (D * 128) + (s & 3) * 32;
          mma_bf16_ss_w(leader, t_o, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(ut + offb), idesc, s > 0);
        }
        mma_commit_w(leader, bars.pro_mma);
      }
      auto issue_s1 = [&](int j) -> bool {
        const int st = j % KWS;
        if (!wait(bars.kw_full + st, (j / KWS) & 1, kStatusTimeoutTma)) return false;
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, kTileN);
        const uint32_t kb = kw0 + st * L::kKW;
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t offb = (s >> 2) * (kTileN * 128) + (s & 3) * 32;
          mma_bf16_ss_w(leader, t_s1 + (j & 1) * kTileN, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(kb + offb), idesc, s > 0);
        }
        mma_commit_w(leader, bars.s1full + (j & 1));
        return true;
      };
      // S2(j) reads the (kbar, w) slot of tile j last: release it afterwards
      auto issue_s2 = [&](int j) -> bool {
        const int st = j % KWS;
        if (!wait(bars.kw_full + st, (j / KWS) & 1, kStatusTimeoutTma)) return false;
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, kTileN);
        const uint32_t wb = kw0 + st * L::kKW + L::kOpK;
        for (int s = 0; s < k2; ++s) {
          const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t offb = (s >> 2) * (kTileN * 128) + (s & 3) * 32;
          mma_bf16_ss_w(leader, t_s2, sdesc_k_sw128(qs0 + offq), sdesc_k_sw128(wb + offb), idesc, s > 0);
        }
        mma_commit_w(leader, bars.s2full);
        mma_commit_w(leader, bars.kw_empty + st);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        if (!wait(bars.pfull + (j & 1), (j >> 1) & 1, kStatusTimeoutMma)) return false;
        const int st = j % VS;
        if (!wait(bars.v_full + st, (j / VS) & 1, kStatusTimeoutTma)) return false;
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, D);
        const uint32_t vb = v0 + st * L::kOpV;
        const uint32_t p = t_s1 + (j & 1) * kTileN;
#pragma unroll
        for (int s = 0; s < kTileN / 16; ++s) {
          // P of blocks 16 s .. 16 s + 15: half s / 4 keeps its P in the first 32 of its own
          // 64 S1 columns
          const uint32_t offv = (s >> 2) * (D * 128) + (s & 3) * 32;
          const uint32_t pa = p + (s >> 2) * 64 + (s & 3) * 8;
          mma_bf16_ts_w(leader, t_o, pa, sdesc_k_sw128(vb + offv), idesc, (j > 0 || s > 0) ? 1u : 0u);
        }
        mma_commit_w(leader, bars.ofull);
        if (j == n_tiles - 1) mma_commit_w(leader, bars.ofin);  // O complete
        mma_commit_w(leader, bars.v_empty + st);
        return true;
      };
      // S1 of the first tiles do not need qsq (the O columns hold Q U until then).  With
      // one (kbar, w) slot the second tile's operands arrive only after S2(0) has read
      // the first ones.
      if (ok) ok = issue_s1(0);
      if (ok && n_tiles > 1 && KWS > 1) ok = issue_s1(1);
      if (ok) ok = wait(bars.qsq_ready, 0, kStatusTimeoutMma);
      if (ok) ok = issue_s2(0);
      if (ok && n_tiles > 1 && KWS == 1) ok = issue_s1(1);
      // drift: Q C_vk^T into the S2 columns once the last S2 has been read
      auto issue_drift = [&]() -> bool {
        if (!wait(bars.s2free, (n_tiles - 1) & 1, kStatusTimeoutMma)) return false;
        if (!wait(bars.c_full, 0, kStatusTimeoutTma)) return false;
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, D);
        const uint32_t cb = kw0 + (n_tiles % KWS) * L::kKW;
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t offb = (s >> 2) * (D * 128) + (s & 3) * 32;
          mma_bf16_ss_w(leader, t_s2, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(cb + offb), idesc, s > 0);
        }
        mma_commit_w(leader, bars.xfull);
        return true;
      };
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          ok = wait(bars.s2free, j & 1, kStatusTimeoutMma);
          if (ok) ok = issue_s2(j + 1);
        } else {
          // the drift goes out while the softmax still works on the last tile, ahead of
          // the last P.V (it needs only the freed S2 columns, Q and C_vk)
          ok = issue_drift();
        }
        if (ok) ok = issue_pv(j);
        if (ok && j + 2 < n_tiles) ok = issue_s1(j + 2);
      }
      mma_commit_w(leader, bars.done);
      mbar_drain(bars.done, 0);
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ================================================================ softmax + epilogue
    const int h = (warp - kSoftmaxWarp0) >> 2;  // half: blocks [64h, 64h + 64) of each tile
    const int q4 = warp & 3;                    // TMEM lane quarter this warp may access
    const int t = q4 * 32 + lane;               // query row
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    constexpr int kHalf = kTileN / 2;           // block means per thread and tile
    constexpr int kDh = D / 2;                  // head-dimension columns per thread
    const float scale = a.scale;
    const float s_l2 = scale * kLog2e;                           // S1 -> log2 units
    const float h_l2 = 0.5f * scale * scale * kLog2e;            // gated S2 -> log2 units
    const float gate_max = a.theta * a.theta / (scale * scale);  // s^2 quad <= theta^2
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      bool r = mbar_wait(bar, parity, abort_flag, a.status, kStatusTimeoutSoftmax);
      return __all_sync(0xffffffffu, r);
    };
    bool ok = wait_all(bars.pro_mma, 0);
    if (ok) {
      tc_fence_after();
      // qsq = bf16(bf16(q U)^2): the A operand of the quadratic term (row t, K-major,
      // 128-byte swizzle); each half squares D/2 columns of q U
      const uint32_t qsq_row = smem_u32(sQsq) + t * 128;
      if (FOLD) {
        // (qsq_0 .. qsq_{rank-1}, T0_hi, T0_lo, T1_hi, T1_lo, 0 ...) over 16 k2 columns:
        // each half stores the qsq_k of its own columns (rank < 64: all in half 0) and
        // its partial tail at columns rank + 2h, rank + 2h + 1; the rest was zeroed
        const int rank = a.rank;
        float tail = 0.f;
#pragma unroll 1
        for (int c = 0; c < kDh / 32; ++c) {
          float v[32];
          tmem_ld32(t_o + h * kDh + c * 32 + lane_base, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 2) bf16_round2(v[e], v[e + 1]);
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float s0 = v[e] * v[e], s1 = v[e + 1] * v[e + 1];
            bf16_round2(s0, s1);
            v[e] = s0;
            v[e + 1] = s1;
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int k = h * kDh + c * 32 + e;
            const float q2 = v[e];
            if (k < rank) {
              const __nv_bfloat16 hb = __float2bfloat16_rn(q2);
              asm volatile("st.shared.b16 [%0], %1;" ::"r"(qsq_row + (((k >> 3) ^ (t & 7)) << 4) + (k & 7) * 2),
                           "h"(*reinterpret_cast<const unsigned short*>(&hb))
                           : "memory");
            } else {
              tail += q2;
            }
          }
        }
        const __nv_bfloat16 hi = __float2bfloat16_rn(tail);
        const __nv_bfloat16 lo = __float2bfloat16_rn(tail - __bfloat162float(hi));
        const int k_hi = rank + 2 * h, k_lo = rank + 2 * h + 1;
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(qsq_row + (((k_hi >> 3) ^ (t & 7)) << 4) + (k_hi & 7) * 2),
                     "h"(*reinterpret_cast<const unsigned short*>(&hi))
                     : "memory");
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(qsq_row + (((k_lo >> 3) ^ (t & 7)) << 4) + (k_lo & 7) * 2),
                     "h"(*reinterpret_cast<const unsigned short*>(&lo))
                     : "memory");
      } else {
#pragma unroll 1
        for (int c = 0; c < kDh / 32; ++c) {
          float v[32];
          tmem_ld32(t_o + h * kDh + c * 32 + lane_base, v);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0 = v[2 * e], x1 = v[2 * e + 1];
            bf16_round2(x0, x1);
            pk[e] = pack_bf16(x0 * x0, x1 * x1);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int k = h * kDh + c * 32 + q * 8;
            st_shared_v4(qsq_row + (k >> 6) * 16384 + ((((k & 63) >> 3) ^ (t & 7)) << 4), pk[4 * q], pk[4 * q + 1],
                         pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.qsq_ready);
    }
    float m_run = -INFINITY;  // running max (log2 domain), identical in both halves
    float l_run = 0.f, g_run = 0.f;  // this half's share of the row sum and of the gated mass
    // Logit bound: s q.kbar_j <= s |q| |kbar_j|, ln n_j <= ln 128, and the gated quadratic
    // term is at most theta^2 / 2; with the largest |kbar| of a tile this bounds every logit
    // of the tile.  A warp whose rows all stay within kBoundSlack of the running max skips
    // the tile's maximum, the exchange with the other half and the rescale; both warps of a
    // lane quarter see the same |q|, bound and running max, so they decide alike.
    float qn_l2 = INFINITY;
    if (ok && a.k_mean_norm != nullptr) {
      const uint32_t qrow = smem_u32(sQ) + t * 128;  // Q landed: the prologue MMA has read it
      float ss = 0.f;
#pragma unroll
      for (int at = 0; at < D / 64; ++at) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w0, w1, w2, w3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                       : "r"(qrow + at * 16384 + ((c ^ (t & 7)) << 4)));
          const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[e]));
            ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
          }
        }
      }
      qn_l2 = sqrtf(ss) * s_l2 * 1.001f + 1.0e-3f;
    }
    const float bound_add = 7.01f + 0.5f * a.theta * a.theta * kLog2e * 1.001f + 0.1f;
    // the epilogue's drift-centre input, loaded now so that its latency is spent here
    const size_t orow_pre = static_cast<size_t>(bank) * a.rows + (qb * 128 + t);
    const float old_lse_pre = (h == 0 && a.center_partial != nullptr) ? a.old_lse[orow_pre] : 0.f;
    int n_xchg = 0;  // exchanges this warp pair has made (slot and parity of its barrier)
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int b = j & 1;
      ok = wait_all(bars.s1full + b, (j >> 1) & 1);
      if (ok) ok = wait_all(bars.s2full, j & 1);
      if (!ok) break;
      tc_fence_after();
      // A bounded tile keeps the running max of every row of the warp (by |q| and the tile's
      // largest |kbar| its logits stay within kBoundSlack of it), so each logit is
      // exponentiated as soon as it is formed: one pass over the sixteen-column steps, with
      // the gate a predicate that serves the gated logit and the gated mass.  The arithmetic,
      // its order and the four partial sums are those of the two-pass path below with
      // alpha = 1 and an unchanged max, so the two give the same bits.
      const bool bounded =
          m_run != -INFINITY && __all_sync(0xffffffffu, qn_l2 * tile_kn[j] + bound_add <= m_run + kBoundSlack);
      if (bounded && j * kTileN + h * kHalf >= nB) {
        // Every column of this half is padding past the last block mean (column term -inf):
        // its exponentials are 0 (2^-125 on the polynomial pairs, below the last bit of any
        // row sum) and the padded v_bar rows are 0, so the half writes P = 0, takes part in
        // the tile's two barriers and leaves the issue slots to the other half.
        uint32_t zero[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) zero[i] = 0u;
#pragma unroll
        for (int c = 0; c < kHalf / 32; ++c) tmem_st16(t_s1 + b * kTileN + h * kHalf + c * 16 + lane_base, zero);
        __syncwarp();
        if (lane == 0) mbar_arrive(bars.s2free);  // this half reads no S2 column of the tile
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bars.pfull + b);
        continue;
      }
      if (bounded) {
        static_assert(kHalf / 16 >= 2, "S2 is released after the second-to-last step's loads");
        const float neg_m = -m_run;
        float ls[4] = {0.f, 0.f, 0.f, 0.f}, gs[4] = {0.f, 0.f, 0.f, 0.f};
        float sa1[16], sa2[16], sb1[16], sb2[16];
        uint32_t pk[16];
        tmem_ld16(t_s1 + b * kTileN + h * kHalf + lane_base, sa1);
        tmem_ld16(t_s2 + h * kHalf + lane_base, sa2);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < kHalf / 16; ++k) {
          float (&v1)[16] = (k & 1) ? sb1 : sa1;
          float (&v2)[16] = (k & 1) ? sb2 : sa2;
          if (k + 1 < kHalf / 16) {
            float (&n1)[16] = (k & 1) ? sa1 : sb1;
            float (&n2)[16] = (k & 1) ? sa2 : sb2;
            tmem_ld16(t_s1 + b * kTileN + h * kHalf + (k + 1) * 16 + lane_base, n1);
            tmem_ld16(t_s2 + h * kHalf + (k + 1) * 16 + lane_base, n2);
          }
          const float4* ct4 = reinterpret_cast<const float4*>(colterm + j * kTileN + h * kHalf + k * 16);
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const float4 ct = ct4[e4];
            const float cts[4] = {ct.x, ct.y, ct.z, ct.w};
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
              const int el = 4 * e4 + 2 * q2;      // first element of the pair in this step
              const int i = (k & 1) * 8 + el / 2;  // the pair's index in its 32-column chunk
              float y[2];
              bool gated[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const float quad = v2[el + u];
                const float base = fmaf(v1[el + u], s_l2, cts[2 * q2 + u]);
                gated[u] = quad <= gate_max;
                y[u] = gated[u] ? fmaf(quad, h_l2, base) : base;
              }
              add2(y[0], y[1], neg_m, neg_m);
              float p0, p1;
              if ((kCoarsePolyPairs >> i) & 1u) {
                exp2_poly2(p0, p1, y[0], y[1]);
              } else {
                p0 = fast_exp2(y[0]);
                p1 = fast_exp2(y[1]);
              }
              add2(ls[(i & 1) * 2], ls[(i & 1) * 2 + 1], p0, p1);
              if (gated[0]) gs[(i & 1) * 2] += p0;
              if (gated[1]) gs[(i & 1) * 2 + 1] += p1;
              pk[i] = pack_bf16(p0, p1);
            }
          }
          // P of blocks 64h + 32c .. + 31 (c = k / 2) into columns whose S1 values were read
          if (k & 1) tmem_st16(t_s1 + b * kTileN + h * kHalf + (k >> 1) * 16 + lane_base, pk);
          if (k + 1 < kHalf / 16) tmem_wait_ld();  // the next step's columns have landed
          if (k == kHalf / 16 - 2) {
            // every S2 column of this tile is in registers: the next quadratic term may go
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bars.s2free);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bars.pfull + b);
        l_run = l_run + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
        g_run = g_run + ((gs[0] + gs[1]) + (gs[2] + gs[3]));
        continue;
      }
      float x[kHalf];
      uint32_t gate[2];
      uint32_t one;  // 1, opaque to the compiler: the mask bits below stay multiply-adds
      asm volatile("mov.b32 %0, 1;" : "=r"(one));
      // Sixteen columns of S1 and S2 per step; the next step's TMEM loads go out before
      // this step's logits, so their latency overlaps the arithmetic.
      float sa1[16], sa2[16], sb1[16], sb2[16];
      tmem_ld16(t_s1 + b * kTileN + h * kHalf + lane_base, sa1);
      tmem_ld16(t_s2 + h * kHalf + lane_base, sa2);
      tmem_wait_ld();
      uint32_t gm = 0;
#pragma unroll
      for (int k = 0; k < kHalf / 16; ++k) {
        float (&v1)[16] = (k & 1) ? sb1 : sa1;
        float (&v2)[16] = (k & 1) ? sb2 : sa2;
        if (k + 1 < kHalf / 16) {
          float (&n1)[16] = (k & 1) ? sa1 : sb1;
          float (&n2)[16] = (k & 1) ? sa2 : sb2;
          tmem_ld16(t_s1 + b * kTileN + h * kHalf + (k + 1) * 16 + lane_base, n1);
          tmem_ld16(t_s2 + h * kHalf + (k + 1) * 16 + lane_base, n2);
        }
        const float4* ct4 = reinterpret_cast<const float4*>(colterm + j * kTileN + h * kHalf + k * 16);
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {
          const float4 ct = ct4[e4];
          const float cts[4] = {ct.x, ct.y, ct.z, ct.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int el = 4 * e4 + i;         // element of this step
            const int e = (k & 1) * 16 + el;   // bit of the 32-column chunk's mask
            const float quad = v2[el];
            // The gate as a branch around the gated product and the mask bit, the bit
            // set by a multiply-add with an opaque 1 (kept on the FMA pipe): this loop
            // is bound by the integer pipe, where selects of the factor and of the bit
            // cost more (bench tail 3.445 ms with selects, 3.223 with the branch and an
            // OR, 3.152 with the multiply-add).
            const float base = fmaf(v1[el], s_l2, cts[i]);
            float xg = base;
            if (quad <= gate_max) {
              xg = fmaf(quad, h_l2, base);
              asm("mad.lo.u32 %0, %1, %2, %0;" : "+r"(gm) : "r"(one), "r"(1u << e));
            }
            x[k * 16 + el] = xg;
          }
        }
        if (k & 1) {
          // opaque copy: the exponential phase then tests these packed bits instead of the
          // compiler keeping 32 comparison results per word alive (which spills)
          asm volatile("mov.b32 %0, %1;" : "=r"(gate[k >> 1]) : "r"(gm));
          gm = 0;
        }
        tmem_wait_ld();  // the next step's columns have landed
      }
      // S2 has been read: the next tile's quadratic term may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.s2free);
      float alpha = 1.f;
      bool rescale = false;
      {
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = max3(x[k], x[8 + k], x[16 + k]);
#pragma unroll
        for (int i = 24; i < kHalf - 8; i += 16) {
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = max3(mx[k], x[i + k], x[i + 8 + k]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], x[kHalf - 8 + k]);
        float m_half = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
        // exchange the half maxima with the other warp of this lane quarter (double-buffered
        // by the parity of the exchange count)
        const int slot = n_xchg & 1;
        rowmax[(slot * 2 + h) * 128 + t] = m_half;
        __syncwarp();
        if (lane == 0) mbar_arrive(bars.xchg + slot * 4 + q4);
        ok = wait_all(bars.xchg + slot * 4 + q4, (n_xchg >> 1) & 1);
        if (!ok) break;
        ++n_xchg;
        const float m_tile = fmaxf(m_half, rowmax[(slot * 2 + (h ^ 1)) * 128 + t]);
        if (m_tile != -INFINITY) {
          if (m_run == -INFINITY) {
            m_run = m_tile;  // nothing accumulated yet: O, l and g are zero
          } else if (m_tile > m_run + kRescaleThreshold) {
            alpha = fast_exp2(m_run - m_tile);
            m_run = m_tile;
            rescale = true;
          }
        }
      }
      // O must hold P.V(j-1) before it is rescaled; P.V(j) starts after pfull below.  The
      // parity wait is sound: S1(j), waited for above, was committed after P.V(j-2), so
      // ofull is at phase j-1 or j here.
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        ok = wait_all(bars.ofull, (j - 1) & 1);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kDh / 8; ++c) {
          float o[8];
          tmem_ld8(t_o + h * kDh + c * 8 + lane_base, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; i += 2) mul2(o[i], o[i + 1], alpha, alpha);
          tmem_st8(t_o + h * kDh + c * 8 + lane_base, o);
        }
      }
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;  // exp2(-inf + 0) = 0
      float ls[4] = {0.f, 0.f, 0.f, 0.f}, gs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e0 = 2 * i, e1 = 2 * i + 1;
          float y0 = x[c * 32 + e0], y1 = x[c * 32 + e1];
          add2(y0, y1, neg_m, neg_m);
          float p0, p1;
          if ((kCoarsePolyPairs >> i) & 1u) {
            exp2_poly2(p0, p1, y0, y1);
          } else {
            p0 = fast_exp2(y0);
            p1 = fast_exp2(y1);
          }
          add2(ls[(i & 1) * 2], ls[(i & 1) * 2 + 1], p0, p1);
          // gated mass: predicated adds into four partial sums (short dependency chains)
          if ((gate[c] >> e0) & 1u) gs[(i & 1) * 2] += p0;
          if ((gate[c] >> e1) & 1u) gs[(i & 1) * 2 + 1] += p1;
          pk[i] = pack_bf16(p0, p1);
        }
        // P of blocks 64h + 32c .. + 31 (two per column), in this half's own S1 columns
        tmem_st16(t_s1 + b * kTileN + h * kHalf + c * 16 + lane_base, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.pfull + b);
      l_run = l_run * alpha + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
      g_run = g_run * alpha + ((gs[0] + gs[1]) + (gs[2] + gs[3]));
    }
    // combine the halves' row sums
    float l_tot = l_run, g_tot = g_run;
    if (ok) {
      rowsums[(h * 2 + 0) * 128 + t] = l_run;
      rowsums[(h * 2 + 1) * 128 + t] = g_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.xsum);
      ok = wait_all(bars.xsum, 0);
      if (ok) {
        l_tot += rowsums[((h ^ 1) * 2 + 0) * 128 + t];
        g_tot += rowsums[((h ^ 1) * 2 + 1) * 128 + t];
      }
    }
    if (ok) {
      ok = wait_all(bars.ofin, 0);  // every P.V has completed (ofull may be two phases ahead)
      if (ok) ok = wait_all(bars.xfull, 0);
    }
    if (ok) {
      tc_fence_after();
      const bool has_tail = l_tot > 0.f;
      const float safe_l = fmaxf(l_tot, 1.0e-30f);
      const float inv_l = 1.f / safe_l;
      const float lse = has_tail ? (m_run + __log2f(l_tot)) * 0.69314718055994531f : -INFINITY;
      const float g_bf = bf16_round(has_tail ? g_tot * inv_l : 0.f);
      const int r = qb * 128 + t;
      const size_t orow = static_cast<size_t>(bank) * a.rows + r;
      // the merged rows are staged in the first vbar^T slot (free once the last P.V has
      // completed): row t at 2 D bytes, its 16-byte chunks XOR-swizzled by t mod 8; each
      // warp then stores its 32 half-rows as whole D-byte runs, 256 / D rows per instruction
      const uint32_t stage = smem_u32(sV);
      // 16 columns of O and of the drift per step; the next step's TMEM loads go out
      // before this step's arithmetic.
      float oa[16], xa[16], ob[16], xb[16];
      tmem_ld16(t_o + h * kDh + lane_base, oa);
      tmem_ld16(t_s2 + h * kDh + lane_base, xa);
      tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < kDh / 16; ++k) {
        float (&ov)[16] = (k & 1) ? ob : oa;
        float (&xv)[16] = (k & 1) ? xb : xa;
        if (k + 1 < kDh / 16) {
          tmem_ld16(t_o + h * kDh + (k + 1) * 16 + lane_base, (k & 1) ? oa : ob);
          tmem_ld16(t_s2 + h * kDh + (k + 1) * 16 + lane_base, (k & 1) ? xa : xb);
        }
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float o0 = ov[2 * e] * inv_l, o1 = ov[2 * e + 1] * inv_l;
          bf16_round2(o0, o1);
          if (!has_tail) o0 = o1 = 0.f;
          float x0 = xv[2 * e], x1 = xv[2 * e + 1];
          bf16_round2(x0, x1);
          float d0 = scale * x0, d1 = scale * x1;
          bf16_round2(d0, d1);
          float g0 = g_bf * d0, g1 = g_bf * d1;
          bf16_round2(g0, g1);
          w[e] = pack_bf16(o0 + g0, o1 + g1);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int j = (h * kDh + k * 16) / 8 + q;  // 16-byte chunk of the row
          st_shared_v4(stage + t * (2 * D) + ((j ^ (t & 7)) << 4), w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
        tmem_wait_ld();  // the next step's columns have landed
      }
      __syncwarp();
      {
        constexpr int kHalfChunks = kDh / 8;      // 16-byte chunks of a half-row
        constexpr int kRowsPer = 32 / kHalfChunks;
        const int jj = h * kHalfChunks + lane % kHalfChunks;
#pragma unroll 1
        for (int i0 = 0; i0 < 32; i0 += kRowsPer) {
          const int ti = q4 * 32 + i0 + lane / kHalfChunks;
          uint32_t w0, w1, w2, w3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                       : "r"(stage + ti * (2 * D) + ((jj ^ (ti & 7)) << 4)));
          st_stream_v4(a.out + (static_cast<size_t>(bank) * a.rows + qb * 128 + ti) * D + jj * 8,
                       make_uint4(w0, w1, w2, w3));
        }
      }
      if (h == 0) {
        a.lse[orow] = lse;
        if (a.center_partial != nullptr) {
          float dv = lse - old_lse_pre;
          for (int o = 16; o > 0; o >>= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
          if (lane == 0) row_part[q4] = dv;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && a.center_partial != nullptr && !*abort_flag)
    a.center_partial[static_cast<size_t>(bank) * (a.rows / 128) + qb] =
        ((row_part[0] + row_part[1]) + (row_part[2] + row_part[3]));
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool FOLD>
int launch_coarse_t(const CoarseLaunch& L, cudaStream_t s) {
  const CoarseArgs& a = L.args;
  dim3 grid(a.rows / 128, a.banks);
  int smem = CoarseSmem<D, FOLD>::kTotal + 1024;
  if (smem < 120 * 1024) smem = 120 * 1024;  // one CTA per SM: it holds all 512 TMEM columns
  cudaFuncSetAttribute(coarse_kernel<D, FOLD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  coarse_kernel<D, FOLD><<<grid, kThreads, smem, s>>>(L.tm_q, L.tm_basis_t, L.tm_cvk, L.tm_kmean, L.tm_var,
                                                      L.tm_vmean_t, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace

int launch_coarse(const CoarseLaunch& L, cudaStream_t s) {
  const CoarseArgs& a = L.args;
  if (a.rows % 128 || a.nB_pad % kTileN || a.nB_pad > kMaxBlocks || a.rank < 0) return kErrShape;
  if (a.rows == 0) return kOk;
  const bool fold = a.rank > 0 && a.rank + 4 <= 64 && a.rank + 4 <= L.D;
  if (L.D == 128) return fold ? launch_coarse_t<128, true>(L, s) : launch_coarse_t<128, false>(L, s);
  if (L.D == 64) return fold ? launch_coarse_t<64, true>(L, s) : launch_coarse_t<64, false>(L, s);
  return kErrShape;
}

}  // namespace recap
