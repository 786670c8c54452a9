// Block-sparse attention forward on sm_100a: for every 128-row query block of
// every bank, exact softmax attention over the key blocks it keeps, with the
// natural-log log-sum-exp of each row.  Replaces the external block_sparse_attn
// call of recap/kernels/block_sparse.py:78-139 and the dense flash call of
// recap/operator.py:254-256 (the same kernel run with every key block kept).
//
// One CTA per (bank, pair of query blocks A and B); 10 warps:
//   warp 0      TMA producer: both Q tiles, then the K and V^T tiles in the order the
//               MMA warp consumes them, through a ring of NST shared-memory slots;
//   warp 1      TMEM allocator and MMA issuer (the warp runs the issue loop, one
//               elected lane issues each tcgen05 instruction);
//   warps 2-5   softmax and epilogue of tile A, warps 6-9 of tile B: one query row per
//               thread (TMEM lane = row), online softmax in the log2 domain with lazy
//               rescaling of O.
// Key-block order: each tile's kept list is reordered so that the blocks both tiles
// keep come first, in the same order.  For those rounds one K tile and one V^T tile in
// shared memory serve both tiles; afterwards each tile streams its own blocks.  The
// softmax order of blocks does not change the result beyond fp32 rounding.
//
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [256+D,256+2D).
// P_x (bf16, two per column) overwrites the first 64 columns of S_x and is the A
// operand of O_x += P_x V straight from TMEM.  MMA issue order:
//   S_A(0) S_B(0), then for r = 0, 1, ...:  PV_A(r) S_A(r+1) PV_B(r) S_B(r+1)
// so the tensor core computes one tile's products while the other tile's softmax
// runs.  S_x(r+1) is issued after PV_x(r) by the same thread, so it overwrites P_x(r)
// only after that product has read it (tcgen05.mma operations of one thread execute
// in issue order), and the commit that signals S_x(r+1) also covers PV_x(r): when the
// softmax sees S_x(r+1), O_x is complete up to block r and may be rescaled.
//
// The epilogue either writes O (bf16) and LSE, or applies the corrected merge of
// recap/kernels/detail_cache.py:188-301 (drift-weighted refinement + coarse tail,
// merged in log-mass space) and writes the result straight to the native token
// order (the Layout.restore gather of recap/sparse/layout.py:90-92).
//
// Refresh mode (recap/operator.py:253-258 and 366-373: the dense flash call and the
// block-sparse head over the same Q, K, V): every key block, with each tile's kept
// blocks first, in the order the sparse step walks them.  When a tile's softmax reaches
// its first omitted block, O holds exactly the kept blocks' products, so that tile's
// head output and LSE are written then (for the query blocks below dense_start the same
// arithmetic and order as the head-only pass, so the same bits); the walk goes on over
// the omitted blocks to the dense result.
// Lists: A = [both keep | A only | B only | neither], B = [both | B only | A only |
// neither], so the first and last parts share their K / V^T tiles.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace recap {

namespace {

constexpr int kThreads = 320;
constexpr int kSoftmaxWarp0 = 2;
constexpr int kMaxKeyBlocks = 2048;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by 2^8
// Largest logit excess over the running max (log2 units) the bounded path accepts: every
// exponential stays below 2^64, finite in fp32 and bf16 with room for the row sums.
constexpr float kBoundSlack = 64.0f;
// Of the 16 column pairs of every 32-key chunk, the ones whose bit is set here take
// their exponentials from exp2_poly2 on the FP32 pipe instead of the MUFU unit.  With
// the tensor core fed at its full rate, a round's 32 MMAs (2048 clk) and the two tiles'
// 2 x 128 x 128 exponentials on MUFU (2048 clk at 16 per clock) take the same time;
// moving a quarter of them to the FP32 pipe makes the softmax the shorter of the two
// (main loop 103 -> 95 clk per MMA on the bench workload; an eighth: 97, 3/8: 100).
constexpr uint32_t kPolyPairs = 0x1111u;
// The same for the blocks a REFRESH pass walks after a query block's kept ones: there
// nearly every block takes the bounded path (no row maximum), which leaves the FP32 pipe
// less room; a sixteenth measured best (REFRESH pass 143.2-143.6 ms against 147.5 with a
// quarter, 144.5-146.2 with an eighth, 145.3-148.9 with none, 162+ with a half).
constexpr uint32_t kPolyPairsOmitted = 0x0001u;

template <int D>
struct FmhaSmem {
  static constexpr int kTileBytes = 128 * D * 2;  // Q, K (128 x D) and V^T (D x 128) tiles
  static constexpr int kNst = D == 128 ? 4 : 8;
  static constexpr int kQ = 0;                        // Q_A, Q_B
  static constexpr int kKV = kQ + 2 * kTileBytes;     // ring of K / V^T tiles
  static constexpr int kBars = kKV + kNst * kTileBytes;
  // qfull, full[NST], empty[NST], sfull[2], pfull[2], ofin[2], done, efull[2]
  static constexpr int kNumBars = 1 + 2 * kNst + 9;
  static constexpr int kMisc = kBars + kNumBars * 8;  // tmem base, abort flag, LA, LB, nS, kept A, kept B
  static constexpr int kList = kMisc + 32;            // uint16 list_a[2048], only_b[2048]
  static constexpr int kRows = kList + 2 * kMaxKeyBlocks * 2;  // staged partition rows, 2 x 2048 bytes
  static constexpr int kCounts = kRows + 2 * kMaxKeyBlocks;   // per-warp list counts [warps][3]
  static constexpr int kTotal = kCounts + 3 * (kThreads / 32) * 4;
};

// Phase discipline: an mbarrier phase is tested by its parity, which tells the current
// phase from the one before it only, so every wait below is by a role that cannot be two
// phases behind the barrier.  The epilogue tiles of a merged query block land in ring slots
// but complete on their own single-phase barrier efull[tile]: they are loaded after the
// whole walk, which for a pair of very unequal tiles (a block keeping every key block next
// to one keeping a tenth) is hundreds of slot phases after the epilogue's tile finished.
struct Bars {
  uint64_t *qfull, *full, *empty, *sfull, *pfull, *ofin, *done, *efull;
};

template <int NST>
__device__ __forceinline__ Bars carve_bars(uint8_t* base) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  Bars r;
  r.qfull = b;
  r.full = b + 1;
  r.empty = b + 1 + NST;
  r.sfull = b + 1 + 2 * NST;
  r.pfull = b + 3 + 2 * NST;
  r.ofin = b + 5 + 2 * NST;
  r.done = b + 7 + 2 * NST;
  r.efull = b + 8 + 2 * NST;
  return r;
}

// The two query blocks of this CTA.  Dense query blocks (attending every key block)
// come first over all banks, then the sparse ones; pairs are adjacent blocks of the
// reordered sequence.  qb < 0: the CTA has one tile.
struct Item {
  int bank, qa, qb;
};

// Output row of bank `bank` at native position `pos` (in the caller's buffer, or in the token
// shard of the rank that holds `pos`).
__device__ __forceinline__ __nv_bfloat16* out_row(const FmhaArgs& a, int bank, int pos) {
  if (a.n_ranks > 1) {
    const int q = pos / a.tokens_per_rank;
    return a.o_rank[q] + static_cast<int64_t>(bank) * a.o_bank_stride +
           static_cast<int64_t>(pos - q * a.tokens_per_rank) * a.o_row_stride;
  }
  return a.o + static_cast<int64_t>(bank) * a.o_bank_stride + static_cast<int64_t>(pos) * a.o_row_stride;
}

__device__ __forceinline__ Item decode_item(const FmhaArgs& a, int b) {
  Item it;
  const int NB = a.NB;
  if (a.all_blocks) {
    const int per = (NB + 1) / 2;
    it.bank = b / per;
    const int k = b - it.bank * per;
    it.qa = 2 * k;
    it.qb = 2 * k + 1 < NB ? 2 * k + 1 : -1;
    return it;
  }
  const int nd_items = (NB - a.dense_start + 1) / 2;
  const int ns_items = (a.dense_start + 1) / 2;
  if (b < a.banks * nd_items) {
    it.bank = b / nd_items;
    const int k = b - it.bank * nd_items;
    it.qa = a.dense_start + 2 * k;
    it.qb = it.qa + 1 < NB ? it.qa + 1 : -1;
  } else {
    b -= a.banks * nd_items;
    it.bank = b / ns_items;
    const int k = b - it.bank * ns_items;
    it.qa = 2 * k;
    it.qb = 2 * k + 1 < a.dense_start ? 2 * k + 1 : -1;
  }
  return it;
}

__host__ __device__ __forceinline__ int fmha_grid(int banks, int NB, int dense_start, int all_blocks) {
  if (all_blocks) return banks * ((NB + 1) / 2);
  return banks * ((NB - dense_start + 1) / 2 + (dense_start + 1) / 2);
}

enum : int { kOpS = 0, kOpPV = 1 };

// The MMA op sequence shared by the producer and the MMA issuer:
//   S_A(0) S_B(0), then per round r: PV_A(r) S_A(r+1) PV_B(r) S_B(r+1)
// with the ops of an exhausted tile dropped.  `op(tile, kind, round)` returns false to
// stop the walk.
template <typename Op>
__device__ __forceinline__ bool walk_ops(int LA, int LB, Op&& op) {
  if (LA > 0 && !op(0, kOpS, 0)) return false;
  if (LB > 0 && !op(1, kOpS, 0)) return false;
  const int R = LA > LB ? LA : LB;
  for (int r = 0; r < R; ++r) {
    if (r < LA) {
      if (!op(0, kOpPV, r)) return false;
      if (r + 1 < LA && !op(0, kOpS, r + 1)) return false;
    }
    if (r < LB) {
      if (!op(1, kOpPV, r)) return false;
      if (r + 1 < LB && !op(1, kOpS, r + 1)) return false;
    }
  }
  return true;
}

template <int D, bool kRefresh>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_vt, const __grid_constant__ CUtensorMap tm_go,
                    const __grid_constant__ CUtensorMap tm_det, const FmhaArgs args) {
  using L = FmhaSmem<D>;
  constexpr int NST = L::kNst;
  constexpr uint32_t kTileBytes = L::kTileBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sKV = smem + L::kKV;
  Bars bars = carve_bars<NST>(smem + L::kBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  int* lens = reinterpret_cast<int*>(smem + L::kMisc + 8);  // LA, LB, nS
  uint16_t* list_a = reinterpret_cast<uint16_t*>(smem + L::kList);
  uint16_t* only_b = list_a + kMaxKeyBlocks;
  uint8_t* row_a = smem + L::kRows;
  uint8_t* row_b = row_a + kMaxKeyBlocks;
  int* counts = reinterpret_cast<int*>(smem + L::kCounts);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Item it = decode_item(args, blockIdx.x);
  const int NB = args.NB;
  const bool has_b = it.qb >= 0;
  constexpr bool refresh = kRefresh;  // a template parameter: the sparse-step code is unchanged
  const bool every = args.all_blocks && !refresh;  // no partition: every block is kept
  const bool dense_a = every || it.qa >= args.dense_start;
  const bool dense_b = every || (has_b && it.qb >= args.dense_start);

  // ---- the two partition rows of the key-block lists: every byte load of this thread
  // goes out first, so that their latency overlaps the barrier setup and the TMEM
  // allocation; they are staged in shared memory below.
  const size_t part_bank = static_cast<size_t>(it.bank) * args.nB;
  constexpr int kPer = (kMaxKeyBlocks + kThreads - 1) / kThreads;
  uint8_t row_va[kPer], row_vb[kPer];
  {
    const uint8_t* pa = dense_a ? nullptr : args.partition + (part_bank + it.qa) * args.nB;
    const uint8_t* pb = (has_b && !dense_b) ? args.partition + (part_bank + it.qb) * args.nB : nullptr;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int j = threadIdx.x + i * kThreads;
      row_va[i] = (pa != nullptr && j < args.dense_start) ? pa[j] : 0;
      row_vb[i] = (pb != nullptr && j < args.dense_start) ? pb[j] : 0;
    }
  }

  // ---- setup: barriers and TMEM; the Q tiles depend on nothing else, so their loads go
  // out as soon as their barrier exists
  if (threadIdx.x == 0) {
    mbar_init(bars.qfull, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(bars.full + s, 1);
      mbar_init(bars.empty + s, 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bars.sfull + x, 1);
      mbar_init(bars.pfull + x, 4);  // one arrival per softmax warp of the tile
      mbar_init(bars.ofin + x, 1);
    }
    mbar_init(bars.done, 1);
    mbar_init(bars.efull, 1);
    mbar_init(bars.efull + 1, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_vt);
    const uint64_t stream = l2_evict_first();  // query tiles are read once
    mbar_expect_tx(bars.qfull, has_b ? 2 * kTileBytes : kTileBytes);
    const int qrow_a = it.bank * args.S_pad + it.qa * 128;
#pragma unroll
    for (int a = 0; a < D / 64; ++a) tma_load_2d_hint(sQ + a * 128 * 128, &tm_q, bars.qfull, a * 64, qrow_a, stream);
    if (has_b) {
      const int qrow_b = it.bank * args.S_pad + it.qb * 128;
#pragma unroll
      for (int a = 0; a < D / 64; ++a)
        tma_load_2d_hint(sQ + kTileBytes + a * 128 * 128, &tm_q, bars.qfull, a * 64, qrow_b, stream);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int j = threadIdx.x + i * kThreads;
    if (j < args.dense_start) {
      row_a[j] = row_va[i];
      row_b[j] = row_vb[i];
    }
  }
  __syncthreads();  // barriers, TMEM address and staged rows are visible to all
  tc_fence_after();
  {
    // Key-block lists by a block-wide compaction in one pass: thread q takes blocks
    // 8q .. 8q + 7 (two 32-bit words of each staged row), counts its blocks kept by both
    // tiles / by A only / by B only, and writes them at its exclusive prefix over the
    // threads before it, so every category keeps ascending block order (shared blocks
    // first in list_a, then A's own).  8 kThreads >= kMaxKeyBlocks.
    static_assert(8 * kThreads >= kMaxKeyBlocks, "one compaction pass");
    constexpr int kWarps = kThreads / 32;
    const int q = threadIdx.x;
    uint32_t bs = 0, ba = 0, bb = 0, bn = 0;  // bit e: block 8q + e in the category
    if (8 * q < NB) {
      const uint2 wa = reinterpret_cast<const uint2*>(row_a)[q];
      const uint2 wb = reinterpret_cast<const uint2*>(row_b)[q];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = 8 * q + e;
        const bool in = j < NB;
        const bool forced = j >= args.dense_start;
        const uint32_t va = ((e < 4 ? wa.x : wa.y) >> (8 * (e & 3))) & 0xffu;
        const uint32_t vb = ((e < 4 ? wb.x : wb.y) >> (8 * (e & 3))) & 0xffu;
        const bool ka = in && (dense_a || forced || va != 0);
        const bool kb = in && has_b && (dense_b || forced || vb != 0);
        bs |= (ka && kb) ? 1u << e : 0u;
        ba |= (ka && !kb) ? 1u << e : 0u;
        bb |= (kb && !ka) ? 1u << e : 0u;
        bn |= (refresh && in && !ka && !kb) ? 1u << e : 0u;  // walked after the kept ones
      }
    }
    // inclusive warp scans of the counts: (shared | A-only << 16) and (B-only | neither << 16)
    const uint32_t m1 = __popc(bs) | (__popc(ba) << 16), m2 = __popc(bb) | (__popc(bn) << 16);
    uint32_t i1 = m1, i2 = m2;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t u1 = __shfl_up_sync(0xffffffffu, i1, o);
      const uint32_t u2 = __shfl_up_sync(0xffffffffu, i2, o);
      if (lane >= o) {
        i1 += u1;
        i2 += u2;
      }
    }
    if (lane == 31) {
      counts[2 * warp] = static_cast<int>(i1);
      counts[2 * warp + 1] = static_cast<int>(i2);
    }
    __syncthreads();
    uint32_t b1 = i1 - m1, b2 = i2 - m2, t1 = 0, t2 = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t c1 = static_cast<uint32_t>(counts[2 * w]), c2 = static_cast<uint32_t>(counts[2 * w + 1]);
      if (w < warp) {
        b1 += c1;
        b2 += c2;
      }
      t1 += c1;
      t2 += c2;
    }
    const int n_shared = t1 & 0xffff, ta = t1 >> 16, tb = t2 & 0xffff, tn = t2 >> 16;
    int os = b1 & 0xffff, oa = n_shared + (b1 >> 16), ob = b2 & 0xffff;
    if (!refresh) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint16_t j = static_cast<uint16_t>(8 * q + e);
        if ((bs >> e) & 1u) list_a[os++] = j;
        if ((ba >> e) & 1u) list_a[oa++] = j;
        if ((bb >> e) & 1u) only_b[ob++] = j;
      }
    } else {
      // list_a = [shared | A only | B only | neither]; only_b (B's rounds from n_shared on)
      // = [B only | A only | neither]
      int oa_b = tb + (b1 >> 16);
      int ob_a = n_shared + ta + (b2 & 0xffff);
      int on_a = n_shared + ta + tb + (b2 >> 16);
      int on_b = tb + ta + (b2 >> 16);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint16_t j = static_cast<uint16_t>(8 * q + e);
        if ((bs >> e) & 1u) list_a[os++] = j;
        if ((ba >> e) & 1u) {
          list_a[oa++] = j;
          only_b[oa_b++] = j;
        }
        if ((bb >> e) & 1u) {
          only_b[ob++] = j;
          list_a[ob_a++] = j;
        }
        if ((bn >> e) & 1u) {
          list_a[on_a++] = j;
          only_b[on_b++] = j;
        }
      }
    }
    if (threadIdx.x == 0) {
      const int all = n_shared + ta + tb + tn;  // refresh: NB
      lens[0] = refresh ? all : n_shared + ta;
      lens[1] = has_b ? (refresh ? all : n_shared + tb) : 0;
      lens[2] = n_shared;
      lens[3] = n_shared + ta;  // kept by A
      lens[4] = n_shared + tb;  // kept by B
    }
  }
  __syncthreads();
  const uint32_t tmem = *tmem_slot;
  const int LA = lens[0];
  const int LB = lens[1];
  const int nS = lens[2];
  auto block_of = [&](int x, int round) -> int {
    return (x == 0 || round < nS) ? list_a[round] : only_b[round - nS];
  };
  // Whether tile B's op of this round uses the K / V^T tile that tile A's op loaded: the
  // shared prefix, and in refresh mode every later round whose two blocks coincide (the
  // blocks neither tile keeps, or all of them when one tile keeps every block).
  auto shared_round = [&](int round) -> bool {
    return round < nS || (refresh && LB > 0 && list_a[round] == only_b[round - nS]);
  };

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0 && LA + LB > 0) {
      const uint64_t keep = l2_evict_last();  // K and V tiles: re-read by many CTAs
      int load_no = 0;
      walk_ops(LA, LB, [&](int x, int kind, int round) -> bool {
        if (x == 1 && shared_round(round)) return true;  // the tile-A op of this round loaded it
        const int slot = load_no % NST;
        if (load_no >= NST &&
            !mbar_wait(bars.empty + slot, ((load_no / NST) - 1) & 1, abort_flag, args.status,
                       kStatusTimeoutProducer))
          return false;
        uint8_t* dst = sKV + slot * kTileBytes;
        const int blk = block_of(x, round);
        mbar_expect_tx(bars.full + slot, kTileBytes);
        if (kind == kOpS) {
          const int krow = it.bank * args.S_pad + blk * 128;
#pragma unroll
          for (int a = 0; a < D / 64; ++a)
            tma_load_2d_hint(dst + a * 128 * 128, &tm_k, bars.full + slot, a * 64, krow, keep);
        } else {
#pragma unroll
          for (int a = 0; a < 2; ++a)
            tma_load_2d_hint(dst + a * D * 128, &tm_vt, bars.full + slot, blk * 128 + a * 64, it.bank * D, keep);
        }
        ++load_no;
        return true;
      });
      // The epilogue's coarse output and refinement tiles (one 128-row tile of each per
      // merged query block) go into the ring slots as they come free, as loads number
      // n_own, n_own + 1, ... after the walk's n_own loads; they complete on efull[tile].
      const int n_walk = load_no;
      bool e_issued[2] = {false, false};
      if (args.tma_epilogue && !*abort_flag) {
        const uint64_t stream = l2_evict_first();  // read once
#pragma unroll 1
        for (int y = 0; y < 2; ++y) {
          const int qblock = y == 0 ? it.qa : it.qb;
          if (qblock < 0 || (qblock + 1) * 128 > args.rows) continue;
          const int row0 = it.bank * args.rows + qblock * 128;
          bool ok_y = true;
#pragma unroll 1
          for (int k = 0; k < 2 && ok_y; ++k) {
            const int slot = load_no % NST;
            if (load_no >= NST &&
                !mbar_wait(bars.empty + slot, ((load_no / NST) - 1) & 1, abort_flag, args.status,
                           kStatusTimeoutProducer)) {
              ok_y = false;
              break;
            }
            uint8_t* dst = sKV + slot * kTileBytes;
            if (k == 0) {
              mbar_expect_tx(bars.efull + y, 2 * kTileBytes);
              e_issued[y] = true;
            }
#pragma unroll
            for (int a = 0; a < D / 64; ++a)
              tma_load_2d_hint(dst + a * 128 * 128, k == 0 ? &tm_go : &tm_det, bars.efull + y, a * 64, row0, stream);
            ++load_no;
          }
          if (!ok_y) break;
        }
      }
      // The CTA that starts when this one ends is about blockIdx.x + the number of SMs: put
      // its Q tiles and partition rows into L2 now, so that its prologue does not wait on
      // HBM (a hint: a wrong guess costs 64 KB of reads).
      if (args.q != nullptr && !*abort_flag) {
        const int nxt = blockIdx.x + args.num_sms;  // one CTA per SM
        if (nxt < static_cast<int>(gridDim.x)) {
          const Item in = decode_item(args, nxt);
#pragma unroll
          for (int y = 0; y < 2; ++y) {
            const int qblock = y == 0 ? in.qa : in.qb;
            if (qblock < 0) continue;
            prefetch_l2_bulk(args.q + (static_cast<size_t>(in.bank) * args.S_pad + qblock * 128) * D, kTileBytes);
            const bool dense_q = (args.all_blocks && !refresh) || qblock >= args.dense_start;
            if (!dense_q) {
              // the whole 16-byte pieces inside the partition row
              const uintptr_t lo = reinterpret_cast<uintptr_t>(args.partition +
                                                               (static_cast<size_t>(in.bank) * args.nB + qblock) * args.nB);
              const uintptr_t a16 = (lo + 15) & ~static_cast<uintptr_t>(15);
              const uintptr_t e16 = (lo + args.dense_start) & ~static_cast<uintptr_t>(15);
              if (e16 > a16) prefetch_l2_bulk(reinterpret_cast<const void*>(a16), static_cast<uint32_t>(e16 - a16));
            }
          }
        }
      }
      // Leave no bulk copy in flight: wait for the last loads this thread issued.
      const int first = n_walk > NST ? n_walk - NST : 0;
      for (int k = first; k < n_walk; ++k) mbar_drain(bars.full + (k % NST), (k / NST) & 1);
      for (int y = 0; y < 2; ++y)
        if (e_issued[y]) mbar_drain(bars.efull + y, 0);
    }
    if (lane == 0) mbar_drain(bars.qfull, 0);
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    // The whole warp runs the issue loop (uniform values, converged control flow) and
    // one elected lane issues every MMA and commit.
    if (LA + LB > 0) {
      const uint32_t leader = elect_leader();
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D);
      const uint32_t q_lo = sdesc_sw128_lo(smem_u32(sQ));    // + x * kTileBytes / 16 for Q_x
      const uint32_t kv_lo = sdesc_sw128_lo(smem_u32(sKV));  // + slot * kTileBytes / 16
      int load_no = 0;
      int slot_k = 0, slot_v = 0;  // latest slot of each kind (K for S, V^T for PV)
      if (__all_sync(0xffffffffu, mbar_wait(bars.qfull, 0, abort_flag, args.status, kStatusTimeoutTma))) {
        walk_ops(LA, LB, [&](int x, int kind, int round) -> bool {
          const bool shared = shared_round(round);
          const bool reuse = x == 1 && shared;
          int slot;
          if (!reuse) {
            slot = load_no % NST;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(bars.full + slot, (load_no / NST) & 1, abort_flag, args.status, kStatusTimeoutTma)))
              return false;
            ++load_no;
            if (kind == kOpS)
              slot_k = slot;
            else
              slot_v = slot;
          } else {
            slot = kind == kOpS ? slot_k : slot_v;
          }
          const uint32_t t_sx = tmem + 128 * x;
          const uint32_t tile_lo = kv_lo + slot * (kTileBytes >> 4);
          if (kind == kOpS) {
            tc_fence_after();
            const uint32_t qx_lo = q_lo + x * (kTileBytes >> 4);
#pragma unroll
            for (int s = 0; s < D / 16; ++s) {
              const uint32_t off = ((s >> 2) * (128 * 128) + (s & 3) * 32) >> 4;
              mma_bf16_ss_lo_w(leader, t_sx, qx_lo + off, tile_lo + off, idesc_s, s > 0);
            }
            mma_commit_w(leader, bars.sfull + x);
          } else {
            if (!__all_sync(0xffffffffu, mbar_wait(bars.pfull + x, round & 1, abort_flag, args.status, kStatusTimeoutMma)))
              return false;
            tc_fence_after();
            const uint32_t t_ox = tmem + 256 + D * x;
#pragma unroll
            for (int s = 0; s < 8; ++s) {
              const uint32_t off_v = ((s >> 2) * (D * 128) + (s & 3) * 32) >> 4;
              mma_bf16_ts_lo_w(leader, t_ox, t_sx + 8 * s, tile_lo + off_v, idesc_o, (round > 0 || s > 0) ? 1u : 0u);
            }
            if (round == (x == 0 ? LA : LB) - 1) mma_commit_w(leader, bars.ofin + x);
          }
          if (x == 1 || !shared) mma_commit_w(leader, bars.empty + slot);  // last user of the slot
          return true;
        });
      }
      // All MMAs issued by the leader complete before TMEM is released.
      mma_commit_w(leader, bars.done);
      mbar_drain(bars.done, 0);
    }
  } else {
    // ================================================================ softmax + epilogue
    const int x = (warp - kSoftmaxWarp0) >> 2;  // tile
    const int q4 = warp & 3;                    // TMEM lane quarter this warp may access
    const int t = q4 * 32 + lane;               // query row within the block
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    const int Lx = x == 0 ? LA : LB;
    const int qblock = x == 0 ? it.qa : it.qb;
    const uint32_t t_sx = tmem + 128 * x + lane_base;
    const uint32_t t_ox = tmem + 256 + D * x + lane_base;
    const float scale_log2 = args.scale_log2;
    float m_run = -INFINITY;  // running max, log2 domain (scaled)
    float l_run = 0.f;        // running row sum at m_run
    // Refresh mode: the round at which O holds exactly this tile's kept blocks (written
    // before that round's exponentials; == Lx: after the walk, in the epilogue).
    const int head_round = refresh ? (x == 0 ? lens[3] : lens[4]) : -1;
    // Head output and LSE of this row from O and the running max / sum (the head-only
    // pass's epilogue arithmetic).  Warp-collective: the TMEM loads run on every lane.
    auto write_head = [&](float m_h, float l_h) {
      const int hr = qblock * 128 + t;  // reordered row
      const bool live = hr < args.S;
      const float inv_h = 1.f / l_h;
      __nv_bfloat16* hrow = args.head_o + (static_cast<size_t>(it.bank) * args.S + (live ? hr : 0)) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(t_ox + c * 32, v);
        tmem_wait_ld();
        if (!live) continue;
        uint4* dst = reinterpret_cast<uint4*>(hrow + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16(v[8 * q + 0] * inv_h, v[8 * q + 1] * inv_h);
          w.y = pack_bf16(v[8 * q + 2] * inv_h, v[8 * q + 3] * inv_h);
          w.z = pack_bf16(v[8 * q + 4] * inv_h, v[8 * q + 5] * inv_h);
          w.w = pack_bf16(v[8 * q + 6] * inv_h, v[8 * q + 7] * inv_h);
          st_stream_v4(dst + q, w);
        }
      }
      if (live) args.head_lse[static_cast<size_t>(it.bank) * args.S + hr] = (m_h + __log2f(l_h)) * 0.69314718055994531f;
    };
    // Logit bound: |q.k| <= |q| |k|, so every logit of key block j is at most
    // qn_l2 * k_norm_max[j] (log2 units).  From the second block on, a warp whose rows all
    // satisfy bound <= m_run + kBoundSlack exponentiates against m_run as it stands: no row
    // maximum and no rescale, and every p stays below 2^kBoundSlack.  Other warps take the
    // exact path.  The result is the same up to fp32 rounding; only the scale of the
    // accumulated values differs, which the final division by the row sum removes.
    float qn_l2 = INFINITY;
    const float* knm = args.k_norm_max ? args.k_norm_max + static_cast<size_t>(it.bank) * NB : nullptr;
    bool ok = Lx > 0;
    if (ok && knm != nullptr) {
      // |q| of this row from the Q tile
      ok = mbar_wait(bars.qfull, 0, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      const uint32_t qrow = smem_u32(sQ) + x * kTileBytes + t * 128;
      float ss = 0.f;
#pragma unroll
      for (int a = 0; a < D / 64; ++a) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w0, w1, w2, w3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                       : "r"(qrow + a * 16384 + ((c ^ (t & 7)) << 4)));
          const uint32_t ws[4] = {w0, w1, w2, w3};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[e]));
            ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
          }
        }
      }
      qn_l2 = sqrtf(ss) * scale_log2 * 1.001f + 1.0e-3f;
    }
    for (int r = 0; ok && r < Lx; ++r) {
      const float kn = (knm != nullptr && r > 0) ? knm[block_of(x, r)] : INFINITY;
      ok = mbar_wait(bars.sfull + x, r & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // O is complete up to block r - 1 (the commit of S(r) covers PV(r - 1)) and PV(r) waits
      // for this warp's pfull arrival: the kept blocks' output can be read now.
      if (refresh && r == head_round) write_head(m_run, l_run);
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(t_sx + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      // keys past the end of the sequence (last, partial key block)
      const int valid = args.S - block_of(x, r) * 128;
      if (valid < 128) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= valid) s[i] = -INFINITY;
      }
      float alpha = 1.f;
      bool rescale = false;
      const bool bounded = __all_sync(0xffffffffu, qn_l2 * kn <= m_run + kBoundSlack);  // false at r = 0
      if (!bounded) {
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = max3(s[k], s[8 + k], s[16 + k]);
#pragma unroll
        for (int i = 24; i < 128; i += 16) {
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = max3(mx[k], s[i + k], s[i + 8 + k]);
        }
        const float m_all = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
        const float m_tile = m_all * scale_log2;
        if (r == 0) {
          m_run = m_tile;
        } else if (m_tile > m_run + kRescaleThreshold) {
          alpha = fast_exp2(m_run - m_tile);
          m_run = m_tile;
          rescale = true;
        }
      }
      const float neg_m = -m_run;
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
      // exponentials, row sums and P of this block; kMask picks the pairs whose
      // exponentials come from the FP32-pipe polynomial
      auto exp_pass = [&](auto mask_tag) {
        constexpr uint32_t kMask = decltype(mask_tag)::value;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float y0, y1;
            fma2(y0, y1, s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1], scale_log2, scale_log2, neg_m, neg_m);
            float p0, p1;
            if ((kMask >> i) & 1u) {
              exp2_poly2(p0, p1, y0, y1);
            } else {
              p0 = fast_exp2(y0);
              p1 = fast_exp2(y1);
            }
            add2(sum[(i & 1) * 2], sum[(i & 1) * 2 + 1], p0, p1);
            pk[i] = pack_bf16(p0, p1);
          }
          tmem_st16(t_sx + c * 16, pk);
        }
      };
      // The REFRESH pass's omitted blocks (after the head is written) take their own split;
      // the kept blocks keep the block-sparse pass's, so the head keeps its bits.
      if (refresh && r >= head_round)
        exp_pass(std::integral_constant<uint32_t, kPolyPairsOmitted>{});
      else
        exp_pass(std::integral_constant<uint32_t, kPolyPairs>{});
      // O holds P.V of blocks 0..r-1 complete (the commit of S(r) covers PV(r-1));
      // PV(r) is not issued before this warp's pfull arrival below.
      if (r > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(t_ox + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 2) mul2(o[i], o[i + 1], alpha, alpha);
          tmem_st32(t_ox + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.pfull + x);
      l_run = l_run * alpha + ((sum[0] + sum[1]) + (sum[2] + sum[3]));
    }
    // Epilogue.  For a merged (video) query block the coarse output and refinement tiles
    // arrive by TMA in the freed ring slots; each thread merges its row from shared memory
    // into the coarse-output slot, then every warp stores its 32 rows as whole 256-byte
    // rows (two per instruction) at their native positions.  The row's indices and merge
    // scalars are loaded before the wait for the last P.V, so their latency overlaps it.
    const int r = qblock * 128 + t;  // reordered row
    int pos = r < args.S ? (args.out_pos ? args.out_pos[r] : r) : -1;
    const bool video = args.epilogue == 1 && r < args.rows;  // whole blocks: rows is a multiple of 128
    const size_t vrow = static_cast<size_t>(it.bank) * args.rows + (video ? r : 0);
    float gl = 0.f, dl = 0.f, ogl = 0.f, cshift = 0.f;
    if (ok && video) {
      gl = args.gl[vrow];
      dl = args.dl[vrow];
      ogl = args.ogl[vrow];
      cshift = args.center[it.bank];
    }
    const bool staged = video && args.tma_epilogue;
    uint32_t s_go = 0, s_det = 0;  // shared addresses of this tile's staged tiles
    int n_go = 0;                  // load number of this tile's coarse-output tile
    if (staged) {
      const int n_own = (LA > 0) + (LB > 0 && nS == 0) + LA + max(0, LA - 1) + max(0, LB - nS) +
                        max(0, LB - 1 - max(nS - 1, 0));
      const bool a_merged = (it.qa + 1) * 128 <= args.rows;
      n_go = n_own + (x == 1 && a_merged ? 2 : 0);
      s_go = smem_u32(sKV) + (n_go % NST) * kTileBytes;
      s_det = smem_u32(sKV) + ((n_go + 1) % NST) * kTileBytes;
    }
    if (ok) {
      ok = mbar_wait(bars.ofin + x, 0, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok && staged) {
      ok = mbar_wait(bars.efull + x, 0, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      if (refresh && head_round >= Lx) write_head(m_run, l_run);  // the tile keeps every block
      const bool in_seq = pos >= 0 && pos < args.S;  // a corrupt index writes nothing
      if (!in_seq) pos = 0;
      const float inv_l = 1.f / l_run;
      const float lse_h = (m_run + __log2f(l_run)) * 0.69314718055994531f;
      const size_t bank_rows = static_cast<size_t>(it.bank) * args.S;
      __nv_bfloat16* orow = out_row(args, it.bank, pos);
      if (staged) {
        // corrected merge (recap/kernels/detail_cache.py:267-292)
        const float admit = expf(-fabsf(gl - ogl - cshift));
        const float cl = gl + dl;
        const float tc = fmaxf(gl, cl);
        const float ms = (1.f - admit) * expf(gl - tc);
        const float mc = admit * expf(cl - tc);
        const float td = fmaxf(ms + mc, 1.0e-30f);
        const float inv_td = 1.f / td;
        const float tail_l = tc + logf(td);
        const float common = fmaxf(lse_h, tail_l);
        const float wh = expf(lse_h - common);
        const float wt = expf(tail_l - common);
        const float inv_den = 1.f / fmaxf(wh + wt, 1.0e-30f);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          tmem_ld32(t_ox + c * 32, v);
          tmem_wait_ld();
          // row t, columns 32 c .. 32 c + 31: four 16-byte chunks of the 128-byte-swizzled tile
          const uint32_t row_off = (c >> 1) * (128 * 128) + t * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t off = row_off + (((((c & 1) * 4 + q) ^ (t & 7))) << 4);
            uint32_t gw[4], dw[4];
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(gw[0]), "=r"(gw[1]), "=r"(gw[2]), "=r"(gw[3])
                         : "r"(s_go + off));
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(dw[0]), "=r"(dw[1]), "=r"(dw[2]), "=r"(dw[3])
                         : "r"(s_det + off));
            uint32_t res[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 gf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[e]));
              const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dw[e]));
              const int i0 = 8 * q + 2 * e;
              float oh0 = v[i0] * inv_l, oh1 = v[i0 + 1] * inv_l;
              bf16_round2(oh0, oh1);
              const float to0 = (gf.x * ms + (gf.x + df.x) * mc) * inv_td;
              const float to1 = (gf.y * ms + (gf.y + df.y) * mc) * inv_td;
              res[e] = pack_bf16((oh0 * wh + to0 * wt) * inv_den, (oh1 * wh + to1 * wt) * inv_den);
            }
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(s_go + off), "r"(res[0]), "r"(res[1]),
                         "r"(res[2]), "r"(res[3])
                         : "memory");
          }
        }
        __syncwarp();
        // the warp's 32 rows, 256 / (D / 8) rows per instruction, each row whole
        constexpr int kChunks = D / 8;            // 16-byte chunks per row
        constexpr int kRowsPer = 32 / kChunks;    // rows per warp instruction
        const int j = lane % kChunks;
#pragma unroll 1
        for (int i0 = 0; i0 < 32; i0 += kRowsPer) {
          const int i = i0 + lane / kChunks;      // row of the warp this lane stores
          const int ti = q4 * 32 + i;
          const int pos_i = __shfl_sync(0xffffffffu, pos, i);
          const int ok_i = __shfl_sync(0xffffffffu, in_seq ? 1 : 0, i);
          uint32_t w0, w1, w2, w3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                       : "r"(s_go + (j >> 3) * (128 * 128) + ti * 128 + (((j & 7) ^ (ti & 7)) << 4)));
          if (ok_i) st_stream_v4(out_row(args, it.bank, pos_i) + j * 8, make_uint4(w0, w1, w2, w3));
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          const int c0 = c * 32;  // first output column of this chunk
          float v[32];
          tmem_ld32(t_ox + c0, v);
          tmem_wait_ld();
          if (!in_seq) continue;
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16(v[8 * q + 0] * inv_l, v[8 * q + 1] * inv_l);
            w.y = pack_bf16(v[8 * q + 2] * inv_l, v[8 * q + 3] * inv_l);
            w.z = pack_bf16(v[8 * q + 4] * inv_l, v[8 * q + 5] * inv_l);
            w.w = pack_bf16(v[8 * q + 6] * inv_l, v[8 * q + 7] * inv_l);
            st_stream_v4(dst + q, w);
          }
        }
      }
      if (in_seq && args.lse) args.lse[bank_rows + pos] = lse_h;
    }
  }
  // Rows stored into other ranks' shards are made visible beyond this GPU before the kernel
  // ends (the ranks then meet at a collective before reading them).
  if (args.n_ranks > 1) __threadfence_system();
  // Nothing asynchronous is in flight past this barrier, on the normal path and after an
  // abort alike: the producer waited (bounded) for the completion of every TMA load it
  // issued - at most NST can be outstanding, since each load into a slot first waited for
  // that slot's previous load to be consumed - and the Q tiles; the MMA warp committed
  // every MMA it issued to `done` and waited (bounded) for it; the softmax warps' TMEM
  // loads and stores completed at their wait::ld / wait::st.  Only then is TMEM freed.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_fmha(const FmhaLaunch& L, cudaStream_t stream) {
  const FmhaArgs& a = L.args;
  if (a.NB > kMaxKeyBlocks || a.dense_start < 0 || a.dense_start > a.NB || a.dense_start > a.nB) return kErrShape;
  const int grid = fmha_grid(a.banks, a.NB, a.dense_start, a.all_blocks);
  if (grid <= 0) return kOk;
  if (L.D == 128) {
    const int smem = FmhaSmem<128>::kTotal + 1024;
    if (a.refresh) {
      cudaFuncSetAttribute(fmha_fwd_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      fmha_fwd_kernel<128, true><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.tm_go, L.tm_det, a);
    } else {
      cudaFuncSetAttribute(fmha_fwd_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      fmha_fwd_kernel<128, false><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.tm_go, L.tm_det, a);
    }
  } else if (L.D == 64) {
    // request enough shared memory for one CTA per SM (TMEM holds one CTA's 512 columns)
    int smem = FmhaSmem<64>::kTotal + 1024;
    if (smem < 120 * 1024) smem = 120 * 1024;
    if (a.refresh) {
      cudaFuncSetAttribute(fmha_fwd_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      fmha_fwd_kernel<64, true><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.tm_go, L.tm_det, a);
    } else {
      cudaFuncSetAttribute(fmha_fwd_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      fmha_fwd_kernel<64, false><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.tm_go, L.tm_det, a);
    }
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
