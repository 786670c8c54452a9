// Block-sparse attention forward on sm_100a: for every 128-row query block of
// every bank, exact softmax attention over the key blocks it keeps, with the
// natural-log log-sum-exp of each row.  Replaces the external block_sparse_attn
// call of recap/kernels/block_sparse.py:78-139 and the dense flash call of
// recap/operator.py:254-256 (the same kernel run with every key block kept).
//
// One CTA per (bank, query block); 12 warps:
//   warp 0      TMA producer: the Q tile once, then K and V^T tiles of every kept
//               key block through a ring of NST shared-memory slots;
//   warp 1      TMEM allocator and MMA issuer (one thread): S = Q K^T into one of
//               two TMEM S buffers, O += P V into the TMEM O accumulator;
//   warps 4-11  softmax, two warpgroups per query tile: each query row is shared by
//               one thread of each group (TMEM lane = row), group g taking key columns
//               [64g, 64g + 64) of S and output columns [D/2 g, D/2 (g+1)).  The groups
//               exchange row maxima each tile, so both rescale with the same running
//               max (log2 domain, lazy rescaling of O), write their half of P as bf16 to
//               shared memory, and split the epilogue.  Two softmax warps per SM
//               sub-partition hide each other's latency.
// The epilogue either writes O (bf16) and LSE, or applies the corrected merge of
// recap/kernels/detail_cache.py:188-301 (drift-weighted refinement + coarse
// tail, merged in log-mass space) and writes the result straight to the native
// token order (the Layout.restore gather of recap/sparse/layout.py:90-92).
#include "common.cuh"
#include "kernels.h"

namespace recap {

namespace {

constexpr int kThreads = 384;
constexpr int kSoftmaxWarp0 = 4;
constexpr int kMaxKeyBlocks = 2048;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when max grows by 2^8

template <int D>
struct FmhaSmem {
  static constexpr int kTileBytes = 128 * D * 2;  // Q, K (128 x D) and V^T (D x 128) tiles
  static constexpr int kNst = 4;
  static constexpr int kQ = 0;
  static constexpr int kP = kQ + kTileBytes;
  static constexpr int kKV = kP + 128 * 128 * 2;
  static constexpr int kBars = kKV + kNst * kTileBytes;
  // barriers: qfull, full[NST], empty[NST], sfull[2], sfree[2], pfull, ofull, done, xchg[2], xsum
  static constexpr int kNumBars = 1 + 2 * kNst + 2 + 2 + 3 + 3;
  static constexpr int kMisc = kBars + kNumBars * 8;  // tmem addr, abort flag, list length
  static constexpr int kList = kMisc + 16;
  static constexpr int kRowMax = kList + kMaxKeyBlocks * 4;  // [2 parity][2 halves][128] fp32
  static constexpr int kRowSum = kRowMax + 2 * 2 * 128 * 4;  // [2 halves][128] fp32
  static constexpr int kTotal = kRowSum + 2 * 128 * 4;
};

struct Bars {
  uint64_t* qfull;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* sfull;
  uint64_t* sfree;
  uint64_t* pfull;
  uint64_t* ofull;
  uint64_t* done;
  uint64_t* xchg;  // [2] row-max exchange between the two softmax warpgroups, by tile parity
  uint64_t* xsum;  // row-sum exchange at the end
};

template <int NST>
__device__ __forceinline__ Bars carve_bars(uint8_t* base) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  Bars r;
  r.qfull = b;
  r.full = b + 1;
  r.empty = b + 1 + NST;
  r.sfull = b + 1 + 2 * NST;
  r.sfree = b + 3 + 2 * NST;
  r.pfull = b + 5 + 2 * NST;
  r.ofull = b + 6 + 2 * NST;
  r.done = b + 7 + 2 * NST;
  r.xchg = b + 8 + 2 * NST;
  r.xsum = b + 10 + 2 * NST;
  return r;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_vt, const FmhaArgs args) {
  using L = FmhaSmem<D>;
  constexpr int NST = L::kNst;
  constexpr uint32_t kTileBytes = L::kTileBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sP = smem + L::kP;
  uint8_t* sKV = smem + L::kKV;
  Bars bars = carve_bars<NST>(smem + L::kBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  int* list_len = reinterpret_cast<int*>(smem + L::kMisc + 8);
  int* list = reinterpret_cast<int*>(smem + L::kList);
  float* rowmax = reinterpret_cast<float*>(smem + L::kRowMax);
  float* rowsum = reinterpret_cast<float*>(smem + L::kRowSum);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work item: bank-major; within a bank the long dense query blocks first
  const int NB = args.NB;
  const int bank = blockIdx.x / NB;
  const int item = blockIdx.x - bank * NB;
  const int n_dense_rows = NB - args.dense_start;
  int qblock = item < n_dense_rows ? args.dense_start + item : item - n_dense_rows;
  if (args.all_blocks) qblock = item;
  const bool dense_row = args.all_blocks || qblock >= args.dense_start;

  // ---- setup: barriers, TMEM, key-block list
  if (threadIdx.x == 0) {
    mbar_init(bars.qfull, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(bars.full + s, 1);
      mbar_init(bars.empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bars.sfull + b, 1);
      mbar_init(bars.sfree + b, 8);  // both softmax warpgroups read each S buffer
    }
    mbar_init(bars.pfull, 8);
    mbar_init(bars.ofull, 1);
    mbar_init(bars.done, 1);
    mbar_init(bars.xchg, 8);
    mbar_init(bars.xchg + 1, 8);
    mbar_init(bars.xsum, 8);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  if (warp == 0) {
    int count = 0;
    const uint8_t* prow =
        args.partition + (static_cast<size_t>(bank) * args.nB + (dense_row ? 0 : qblock)) * args.nB;
    for (int base = 0; base < NB; base += 32) {
      const int j = base + lane;
      bool keep = false;
      if (j < NB) keep = dense_row || j >= args.dense_start || prow[j] != 0;
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) list[count + __popc(m & ((1u << lane) - 1u))] = j;
      count += __popc(m);
    }
    if (lane == 0) *list_len = count;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_kv = *list_len;
  const uint32_t t_s = tmem;           // S buffers: columns [0,128) and [128,256)
  const uint32_t t_o = tmem + 256;     // O accumulator: columns [256, 256 + D)

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0 && n_kv > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_vt);
      const uint64_t keep = l2_evict_last();    // K and V tiles: re-read by many CTAs
      const uint64_t stream = l2_evict_first(); // the Q tile: read once
      const int qrow = bank * args.S_pad + qblock * 128;
      mbar_expect_tx(bars.qfull, kTileBytes);
#pragma unroll
      for (int a = 0; a < D / 64; ++a)
        tma_load_2d_hint(sQ + a * 128 * 128, &tm_q, bars.qfull, a * 64, qrow, stream);
      const int n_items = 2 * n_kv;
      int i = 0;
      for (; i < n_items; ++i) {
        const int slot = i % NST;
        if (i >= NST) {
          if (!mbar_wait(bars.empty + slot, ((i / NST) - 1) & 1, abort_flag, args.status,
                         kStatusTimeoutProducer))
            break;
        }
        uint8_t* dst = sKV + slot * kTileBytes;
        const int blk = list[i >> 1];
        mbar_expect_tx(bars.full + slot, kTileBytes);
        if ((i & 1) == 0) {
          const int krow = bank * args.S_pad + blk * 128;
#pragma unroll
          for (int a = 0; a < D / 64; ++a)
            tma_load_2d_hint(dst + a * 128 * 128, &tm_k, bars.full + slot, a * 64, krow, keep);
        } else {
#pragma unroll
          for (int a = 0; a < 2; ++a)
            tma_load_2d_hint(dst + a * D * 128, &tm_vt, bars.full + slot, blk * 128 + a * 64, bank * D, keep);
        }
      }
      // Leave no bulk copy in flight: wait for the last loads this thread issued.
      const int first = i > NST ? i - NST : 0;
      for (int k = first; k < i; ++k) {
        const int slot = k % NST;
        mbar_drain(bars.full + slot, (k / NST) & 1);
      }
      mbar_drain(bars.qfull, 0);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D);
      const uint32_t q_base = smem_u32(sQ);
      const uint32_t p_base = smem_u32(sP);
      const uint32_t kv_base = smem_u32(sKV);
      bool ok = mbar_wait(bars.qfull, 0, abort_flag, args.status, kStatusTimeoutTma);
      auto issue_s = [&](int j) -> bool {
        const int item_k = 2 * j;
        const int slot = item_k % NST;
        if (!mbar_wait(bars.full + slot, (item_k / NST) & 1, abort_flag, args.status,
                       kStatusTimeoutTma))
          return false;
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(bars.sfree + b, ((j >> 1) - 1) & 1, abort_flag, args.status,
                                 kStatusTimeoutMma))
          return false;
        tc_fence_after();
        const uint32_t k_base = kv_base + slot * kTileBytes;
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t off = (s >> 2) * (128 * 128) + (s & 3) * 32;
          mma_bf16_ss(t_s + b * 128, sdesc_k_sw128(q_base + off), sdesc_k_sw128(k_base + off),
                      idesc_s, s > 0);
        }
        mma_commit(bars.sfull + b);
        mma_commit(bars.empty + slot);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(bars.pfull, j & 1, abort_flag, args.status, kStatusTimeoutMma)) return false;
        const int item_v = 2 * j + 1;
        const int slot = item_v % NST;
        if (!mbar_wait(bars.full + slot, (item_v / NST) & 1, abort_flag, args.status,
                       kStatusTimeoutTma))
          return false;
        tc_fence_after();
        const uint32_t v_base = kv_base + slot * kTileBytes;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t off_p = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t off_v = (s >> 2) * (D * 128) + (s & 3) * 32;
          mma_bf16_ss(t_o, sdesc_k_sw128(p_base + off_p), sdesc_k_sw128(v_base + off_v), idesc_o,
                      (j > 0 || s > 0) ? 1u : 0u);
        }
        mma_commit(bars.empty + slot);
        mma_commit(bars.ofull);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 1; ok && j < n_kv; ++j) {
        ok = issue_s(j);
        if (ok) ok = issue_pv(j - 1);
      }
      if (ok) ok = issue_pv(n_kv - 1);
      // All MMAs issued by this thread complete before TMEM is released.
      mma_commit(bars.done);
      mbar_drain(bars.done, 0);
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ================================================================ softmax + epilogue
    // Two warpgroups share every query row: group g handles key columns [64g, 64g + 64)
    // of S and output columns [D/2 g, D/2 (g + 1)); the row max is exchanged through
    // shared memory each tile so both groups use the same running max.
    const int g = (warp - kSoftmaxWarp0) >> 2;   // column half
    const int q4 = (warp - kSoftmaxWarp0) & 3;   // TMEM lane quarter
    const int t = q4 * 32 + lane;                // query row within the block
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    const float scale_log2 = args.scale_log2;
    float m_run = -INFINITY;  // running max, log2 domain (scaled), identical in both groups
    float l_run = 0.f;        // this group's share of the row sum
    const uint32_t p_row = smem_u32(sP) + g * 16384 + t * 128;  // P columns [64g, 64g + 64)
    bool ok = n_kv > 0;
    for (int j = 0; ok && j < n_kv; ++j) {
      const int b = j & 1;
      ok = mbar_wait(bars.sfull + b, (j >> 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float x[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tmem_ld32(t_s + b * 128 + g * 64 + c * 32 + lane_base, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c * 32 + i] = v[i];
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.sfree + b);
      // keys past the end of the sequence (last, partial key block)
      const int valid = args.S - list[j] * 128 - g * 64;
      if (valid < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= valid) x[i] = -INFINITY;
      }
      float mxa[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mxa[k] = x[k];
#pragma unroll
      for (int i = 8; i < 64; ++i) mxa[i & 7] = fmaxf(mxa[i & 7], x[i]);
      float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                       fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
      // exchange the half-row maxima (double-buffered by tile parity); an mbarrier with a
      // bounded wait, so that a warpgroup that aborts cannot strand the other one
      rowmax[(b * 2 + g) * 128 + t] = mx;
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.xchg + b);
      ok = mbar_wait(bars.xchg + b, (j >> 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      mx = fmaxf(mx, rowmax[(b * 2 + (g ^ 1)) * 128 + t]);
      const float m_tile = mx * scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_run = m_tile;
      } else if (m_tile > m_run + kRescaleThreshold) {
        alpha = fast_exp2(m_run - m_tile);
        m_run = m_tile;
        rescale = true;
      }
      float sa[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = fast_exp2(fmaf(x[2 * i], scale_log2, -m_run));
        const float p1 = fast_exp2(fmaf(x[2 * i + 1], scale_log2, -m_run));
        sa[i & 3] += p0 + p1;
        pk[i] = pack_bf16(p0, p1);
      }
      l_run = l_run * alpha + ((sa[0] + sa[1]) + (sa[2] + sa[3]));
      // PV(j-1) must be complete before P is overwritten and O is rescaled.
      if (j > 0) {
        ok = mbar_wait(bars.ofull, (j - 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            float v[32];
            const uint32_t col = t_o + g * (D / 2) + c * 32 + lane_base;
            tmem_ld32(col, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tmem_st32(col, v);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        st_shared_v4(p_row + ((c ^ (t & 7)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.pfull);
    }
    if (ok) {
      ok = mbar_wait(bars.ofull, (n_kv - 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
    }
    // combine the two halves of the row sum
    float l_tot = l_run;
    if (ok) {
      rowsum[g * 128 + t] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.xsum);
      ok = mbar_wait(bars.xsum, 0, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) l_tot = l_run + rowsum[(g ^ 1) * 128 + t];
    }
    if (ok) {
      tc_fence_after();
      const int r = qblock * 128 + t;  // reordered row
      int pos = r < args.S ? (args.out_pos ? args.out_pos[r] : r) : -1;
      const bool in_seq = pos >= 0 && pos < args.S;  // a corrupt index writes nothing
      if (!in_seq) pos = 0;
      const float inv_l = 1.f / l_tot;
      const float lse_h = (m_run + __log2f(l_tot)) * 0.69314718055994531f;
      const size_t bank_rows = static_cast<size_t>(bank) * args.S;
      __nv_bfloat16* orow = args.o + (bank_rows + pos) * D;
      const bool video = args.epilogue == 1 && r < args.rows;
      float wh = 1.f, wt = 0.f, ms = 0.f, mc = 0.f, inv_td = 0.f, inv_den = 1.f;
      size_t vrow = 0;
      if (video) {
        // corrected merge (recap/kernels/detail_cache.py:267-292)
        vrow = static_cast<size_t>(bank) * args.rows + r;
        const float gl = args.gl[vrow];
        const float dl = args.dl[vrow];
        const float ogl = args.ogl[vrow];
        const float cshift = args.center[bank];
        const float admit = expf(-fabsf(gl - ogl - cshift));
        const float cl = gl + dl;
        const float tc = fmaxf(gl, cl);
        ms = (1.f - admit) * expf(gl - tc);
        mc = admit * expf(cl - tc);
        const float td = fmaxf(ms + mc, 1.0e-30f);
        inv_td = 1.f / td;
        const float tail_l = tc + logf(td);
        const float common = fmaxf(lse_h, tail_l);
        wh = expf(lse_h - common);
        wt = expf(tail_l - common);
        inv_den = 1.f / fmaxf(wh + wt, 1.0e-30f);
      }
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) {
        const int c0 = g * (D / 2) + c * 32;  // first output column of this chunk
        float v[32];
        tmem_ld32(t_o + c0 + lane_base, v);
        tmem_wait_ld();
        if (!in_seq) continue;
        float res[32];
        if (video) {
          const uint4* gsrc = reinterpret_cast<const uint4*>(args.go + vrow * D + c0);
          const uint4* dsrc = reinterpret_cast<const uint4*>(args.det + vrow * D + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 gw = ld_stream_v4(gsrc + q);
            const uint4 dw = ld_stream_v4(dsrc + q);
            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gw);
            const __half2* d2 = reinterpret_cast<const __half2*>(&dw);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 gf = __bfloat1622float2(g2[e]);
              const float2 df = __half22float2(d2[e]);
              const int i0 = 8 * q + 2 * e;
              const float oh0 = bf16_round(v[i0] * inv_l);
              const float oh1 = bf16_round(v[i0 + 1] * inv_l);
              const float to0 = (gf.x * ms + (gf.x + df.x) * mc) * inv_td;
              const float to1 = (gf.y * ms + (gf.y + df.y) * mc) * inv_td;
              res[i0] = (oh0 * wh + to0 * wt) * inv_den;
              res[i0 + 1] = (oh1 * wh + to1 * wt) * inv_den;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) res[i] = v[i] * inv_l;
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16(res[8 * q + 0], res[8 * q + 1]);
          w.y = pack_bf16(res[8 * q + 2], res[8 * q + 3]);
          w.z = pack_bf16(res[8 * q + 4], res[8 * q + 5]);
          w.w = pack_bf16(res[8 * q + 6], res[8 * q + 7]);
          st_stream_v4(dst + q, w);
        }
      }
      if (g == 0 && in_seq && args.lse) args.lse[bank_rows + pos] = lse_h;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_fmha(const FmhaLaunch& L, cudaStream_t stream) {
  if (L.args.NB > kMaxKeyBlocks) return kErrShape;
  const int grid = L.args.banks * L.args.NB;
  if (grid <= 0) return kOk;
  if (L.D == 128) {
    const int smem = FmhaSmem<128>::kTotal + 1024;
    cudaFuncSetAttribute(fmha_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fmha_fwd_kernel<128><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.args);
  } else if (L.D == 64) {
    // request enough shared memory for one CTA per SM (TMEM holds one CTA's 512 columns)
    int smem = FmhaSmem<64>::kTotal + 1024;
    if (smem < 120 * 1024) smem = 120 * 1024;
    cudaFuncSetAttribute(fmha_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fmha_fwd_kernel<64><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.args);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
