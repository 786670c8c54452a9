// Block-sparse attention forward on sm_100a: for every 128-row query block of
// every bank, exact softmax attention over the key blocks it keeps, with the
// natural-log log-sum-exp of each row.  Replaces the external block_sparse_attn
// call of recap/kernels/block_sparse.py:78-139 and the dense flash call of
// recap/operator.py:254-256 (the same kernel run with every key block kept).
//
// One CTA per (bank, pair of query blocks); 12 warps:
//   warp 0       TMA producer: both Q tiles, then the K and V^T tiles of both kept
//                lists, in the order the MMA warp consumes them, through a ring of
//                NST shared-memory slots;
//   warp 1       TMEM allocator and MMA issuer (one thread): S_x = Q_x K^T into the
//                tile's TMEM S buffer, O_x += P V into its TMEM O accumulator, the two
//                tiles interleaved so that the tensor core works on one tile while the
//                other tile's softmax runs;
//   warps 2-3    build the two kept lists, then idle;
//   warps 4-7    softmax of tile A, warps 8-11 softmax of tile B: one query row per
//                thread (TMEM lane = row), online softmax in the log2 domain with lazy
//                rescaling of O, P written as bf16 into the shared P buffer, then the
//                epilogue.
// The epilogue either writes O (bf16) and LSE, or applies the corrected merge of
// recap/kernels/detail_cache.py:188-301 (drift-weighted refinement + coarse tail,
// merged in log-mass space) and writes the result straight to the native token
// order (the Layout.restore gather of recap/sparse/layout.py:90-92).
//
// Op order (both the producer and the MMA warp walk it; each op takes one ring slot):
//   S_A(0) S_B(0), then for j = 0, 1, ...:  S_A(j+1) PV_A(j) S_B(j+1) PV_B(j)
// with the ops of a tile dropped once its list is exhausted.  P uses follow the PV
// order; the writer of P use u waits until PV use u-1 has completed.
#include "common.cuh"
#include "kernels.h"

namespace recap {

namespace {

constexpr int kThreads = 384;
constexpr int kMaxKeyBlocks = 2048;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by 2^8

template <int D>
struct FmhaSmem {
  static constexpr int kTileBytes = 128 * D * 2;  // Q, K (128 x D) and V^T (D x 128) tiles
  static constexpr int kNst = 3;
  static constexpr int kQ = 0;                     // two Q tiles
  static constexpr int kP = kQ + 2 * kTileBytes;   // one P buffer, 128 x 128 bf16
  static constexpr int kKV = kP + 128 * 128 * 2;
  static constexpr int kList = kKV + kNst * kTileBytes;  // two uint16 key-block lists
  static constexpr int kBars = kList + 2 * kMaxKeyBlocks * 2;
  // qfull, full[NST], empty[NST], sfull[2], sfree[2], pfull[2], ofull[2], pdone, done
  static constexpr int kNumBars = 1 + 2 * kNst + 8 + 2;
  static constexpr int kMisc = kBars + kNumBars * 8;  // tmem addr, abort flag, list lengths
  static constexpr int kTotal = kMisc + 16;
};

struct Bars {
  uint64_t *qfull, *full, *empty, *sfull, *sfree, *pfull, *ofull, *pdone, *done;
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
  r.ofull = b + 7 + 2 * NST;
  r.pdone = b + 9 + 2 * NST;
  r.done = b + 10 + 2 * NST;
  return r;
}

// Global index of PV_x(j) in the op order (number of PV ops before it).
__device__ __forceinline__ int pv_index(int tile, int j, int LA, int LB) {
  return tile == 0 ? j + min(j, LB) : j + min(j + 1, LA);
}

// Walk the op order, calling f(tile, is_pv, j) for every op; stops when f returns false.
template <typename F>
__device__ __forceinline__ bool walk_ops(int LA, int LB, F&& f) {
  if (LA > 0 && !f(0, false, 0)) return false;
  if (LB > 0 && !f(1, false, 0)) return false;
  const int n = max(LA, LB);
  for (int j = 0; j < n; ++j) {
    if (j + 1 < LA && !f(0, false, j + 1)) return false;
    if (j < LA && !f(0, true, j)) return false;
    if (j + 1 < LB && !f(1, false, j + 1)) return false;
    if (j < LB && !f(1, true, j)) return false;
  }
  return true;
}

template <int D>
__device__ __forceinline__ void epilogue(const FmhaArgs& args, int bank, int qblock, int t, uint32_t t_o,
                                         uint32_t lane_base, float m_run, float l_run) {
  const int r = qblock * 128 + t;  // reordered row
  int pos = r < args.S ? (args.out_pos ? args.out_pos[r] : r) : -1;
  const bool in_seq = pos >= 0 && pos < args.S;  // a corrupt index writes nothing
  if (!in_seq) pos = 0;
  const float inv_l = 1.f / l_run;
  const float lse_h = (m_run + __log2f(l_run)) * 0.69314718055994531f;
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
  for (int c = 0; c < D / 32; ++c) {
    float v[32];
    tmem_ld32(t_o + c * 32 + lane_base, v);
    tmem_wait_ld();
    if (!in_seq) continue;
    float res[32];
    if (video) {
      const uint4* gsrc = reinterpret_cast<const uint4*>(args.go + vrow * D + c * 32);
      const uint4* dsrc = reinterpret_cast<const uint4*>(args.det + vrow * D + c * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 gw = gsrc[q];
        const uint4 dw = dsrc[q];
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
    uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack_bf16(res[8 * q + 0], res[8 * q + 1]);
      w.y = pack_bf16(res[8 * q + 2], res[8 * q + 3]);
      w.z = pack_bf16(res[8 * q + 4], res[8 * q + 5]);
      w.w = pack_bf16(res[8 * q + 6], res[8 * q + 7]);
      dst[q] = w;
    }
  }
  if (in_seq && args.lse) args.lse[bank_rows + pos] = lse_h;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_vt, const FmhaArgs args) {
  using L = FmhaSmem<D>;
  constexpr int NST = L::kNst;
  constexpr uint32_t kTileBytes = L::kTileBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sP = smem + L::kP;
  uint8_t* sKV = smem + L::kKV;
  uint16_t* lists = reinterpret_cast<uint16_t*>(smem + L::kList);
  Bars bars = carve_bars<NST>(smem + L::kBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  int* list_len = reinterpret_cast<int*>(smem + L::kMisc + 8);  // [2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work: bank-major; within a bank the long dense query blocks first, in pairs
  const int NB = args.NB;
  const int pairs = (NB + 1) / 2;
  const int bank = blockIdx.x / pairs;
  const int pair = blockIdx.x - bank * pairs;
  const int n_dense_rows = NB - args.dense_start;
  int qblock[2];
  bool dense_row[2];
  bool has_tile[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int item = 2 * pair + x;
    has_tile[x] = item < NB;
    int qb = item < n_dense_rows ? args.dense_start + item : item - n_dense_rows;
    if (args.all_blocks) qb = item;
    qblock[x] = has_tile[x] ? qb : 0;
    dense_row[x] = args.all_blocks || qb >= args.dense_start;
  }

  // ---- setup: barriers, TMEM, key-block lists
  if (threadIdx.x == 0) {
    mbar_init(bars.qfull, 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(bars.full + s, 1);
      mbar_init(bars.empty + s, 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bars.sfull + x, 1);
      mbar_init(bars.sfree + x, 4);
      mbar_init(bars.pfull + x, 4);
      mbar_init(bars.ofull + x, 1);
    }
    mbar_init(bars.pdone, 1);
    mbar_init(bars.done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  if (warp == 2 || warp == 3) {
    const int x = warp - 2;
    int count = 0;
    if (has_tile[x]) {
      const uint8_t* prow =
          args.partition + (static_cast<size_t>(bank) * args.nB + (dense_row[x] ? 0 : qblock[x])) * args.nB;
      for (int base = 0; base < NB; base += 32) {
        const int j = base + lane;
        bool keep = false;
        if (j < NB) keep = dense_row[x] || j >= args.dense_start || prow[j] != 0;
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        if (keep) lists[x * kMaxKeyBlocks + count + __popc(m & ((1u << lane) - 1u))] = static_cast<uint16_t>(j);
        count += __popc(m);
      }
    }
    if (lane == 0) list_len[x] = count;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int LA = list_len[0];
  const int LB = list_len[1];
  // TMEM: tile x uses S in columns [256x, 256x + 128) and O in [256x + 128, 256x + 128 + D)

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0 && LA + LB > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_vt);
      mbar_expect_tx(bars.qfull, (LB > 0 ? 2u : 1u) * kTileBytes);
      for (int x = 0; x < 2; ++x) {
        if ((x == 0 ? LA : LB) == 0) continue;
        const int qrow = bank * args.S_pad + qblock[x] * 128;
#pragma unroll
        for (int a = 0; a < D / 64; ++a)
          tma_load_2d(sQ + x * kTileBytes + a * 128 * 128, &tm_q, bars.qfull, a * 64, qrow);
      }
      int i = 0;
      walk_ops(LA, LB, [&](int x, bool is_pv, int j) -> bool {
        const int slot = i % NST;
        if (i >= NST && !mbar_wait(bars.empty + slot, ((i / NST) - 1) & 1, abort_flag, args.status,
                                   kStatusTimeoutProducer))
          return false;
        uint8_t* dst = sKV + slot * kTileBytes;
        const int blk = lists[x * kMaxKeyBlocks + j];
        mbar_expect_tx(bars.full + slot, kTileBytes);
        if (!is_pv) {
          const int krow = bank * args.S_pad + blk * 128;
#pragma unroll
          for (int a = 0; a < D / 64; ++a) tma_load_2d(dst + a * 128 * 128, &tm_k, bars.full + slot, a * 64, krow);
        } else {
#pragma unroll
          for (int a = 0; a < 2; ++a)
            tma_load_2d(dst + a * D * 128, &tm_vt, bars.full + slot, blk * 128 + a * 64, bank * D);
        }
        ++i;
        return true;
      });
      // leave no bulk copy in flight
      const int first = i > NST ? i - NST : 0;
      for (int k = first; k < i; ++k) mbar_drain(bars.full + (k % NST), (k / NST) & 1);
      mbar_drain(bars.qfull, 0);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0 && LA + LB > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D);
      const uint32_t q_base = smem_u32(sQ);
      const uint32_t p_base = smem_u32(sP);
      const uint32_t kv_base = smem_u32(sKV);
      bool ok = mbar_wait(bars.qfull, 0, abort_flag, args.status, kStatusTimeoutTma);
      int i = 0;
      if (ok) {
        walk_ops(LA, LB, [&](int x, bool is_pv, int j) -> bool {
          const int slot = i % NST;
          const uint32_t t_s = tmem + 256 * x;
          const uint32_t t_o = t_s + 128;
          if (!is_pv) {
            if (j >= 1 && !mbar_wait(bars.sfree + x, (j - 1) & 1, abort_flag, args.status, kStatusTimeoutMma))
              return false;
          } else {
            if (!mbar_wait(bars.pfull + x, j & 1, abort_flag, args.status, kStatusTimeoutMma)) return false;
          }
          if (!mbar_wait(bars.full + slot, (i / NST) & 1, abort_flag, args.status, kStatusTimeoutTma)) return false;
          tc_fence_after();
          const uint32_t op_base = kv_base + slot * kTileBytes;
          if (!is_pv) {
            const uint32_t qb = q_base + x * kTileBytes;
#pragma unroll
            for (int s = 0; s < D / 16; ++s) {
              const uint32_t off = (s >> 2) * (128 * 128) + (s & 3) * 32;
              mma_bf16_ss(t_s, sdesc_k_sw128(qb + off), sdesc_k_sw128(op_base + off), idesc_s, s > 0);
            }
            mma_commit(bars.sfull + x);
          } else {
#pragma unroll
            for (int s = 0; s < 8; ++s) {
              const uint32_t off_p = (s >> 2) * (128 * 128) + (s & 3) * 32;
              const uint32_t off_v = (s >> 2) * (D * 128) + (s & 3) * 32;
              mma_bf16_ss(t_o, sdesc_k_sw128(p_base + off_p), sdesc_k_sw128(op_base + off_v), idesc_o,
                          (j > 0 || s > 0) ? 1u : 0u);
            }
            mma_commit(bars.ofull + x);
            mma_commit(bars.pdone);
          }
          mma_commit(bars.empty + slot);
          ++i;
          return true;
        });
      }
      // all MMAs issued by this thread complete before TMEM is released
      mma_commit(bars.done);
      mbar_drain(bars.done, 0);
    }
  } else if (warp >= 4) {
    // ================================================================ softmax + epilogue
    const int x = (warp - 4) >> 2;          // tile
    const int q4 = (warp - 4) & 3;          // warp within the tile's warpgroup = TMEM lane quarter
    const int t = q4 * 32 + lane;           // query row within the block
    const int Lx = x == 0 ? LA : LB;
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    const uint32_t t_s = tmem + 256 * x;
    const uint32_t t_o = t_s + 128;
    const float scale_log2 = args.scale_log2;
    const uint16_t* list = lists + x * kMaxKeyBlocks;
    float m_run = -INFINITY;  // running max, log2 domain (scaled)
    float l_run = 0.f;
    const uint32_t p_row = smem_u32(sP) + t * 128;
    bool ok = Lx > 0;
    for (int j = 0; ok && j < Lx; ++j) {
      ok = mbar_wait(bars.sfull + x, j & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int valid = args.S - static_cast<int>(list[j]) * 128;  // keys past the sequence end
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(t_s + c * 32 + lane_base, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c * 32 + i < valid) mx = fmaxf(mx, v[i]);
      }
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
      // pass 2: probabilities, packed to bf16
      float sum = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(t_s + c * 32 + lane_base, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k0 = c * 32 + 2 * i;
          const float p0 = k0 < valid ? fast_exp2(fmaf(v[2 * i], scale_log2, -m_run)) : 0.f;
          const float p1 = k0 + 1 < valid ? fast_exp2(fmaf(v[2 * i + 1], scale_log2, -m_run)) : 0.f;
          sum += p0 + p1;
          pk[c * 16 + i] = pack_bf16(p0, p1);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.sfree + x);
      l_run = l_run * alpha + sum;
      // This tile's previous PV (P use u_x(j-1) >= u-2) completes first: O may then be
      // rescaled, and the global P-use barrier is at most one phase short of use u-1, the
      // range a parity wait can tell apart.  Then the shared P buffer is free once P use
      // u-1 (the other tile's, or this tile's own) has been consumed.
      const int u = pv_index(x, j, LA, LB);
      if (j > 0) {
        ok = mbar_wait(bars.ofull + x, (j - 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
      if (u > 0) {
        ok = mbar_wait(bars.pdone, (u - 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          tmem_ld32(t_o + c * 32 + lane_base, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(t_o + c * 32 + lane_base, v);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int atom = c >> 3;
        const int cc = c & 7;
        st_shared_v4(p_row + atom * 16384 + ((cc ^ (t & 7)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                     pk[4 * c + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.pfull + x);
    }
    if (ok) {
      ok = mbar_wait(bars.ofull + x, (Lx - 1) & 1, abort_flag, args.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      epilogue<D>(args, bank, qblock[x], t, t_o, lane_base, m_run, l_run);
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
  const int grid = L.args.banks * ((L.args.NB + 1) / 2);
  if (grid <= 0) return kOk;
  if (L.D == 128) {
    const int smem = FmhaSmem<128>::kTotal + 1024;
    cudaFuncSetAttribute(fmha_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fmha_fwd_kernel<128><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.args);
  } else if (L.D == 64) {
    // at least ~115 KB so that one CTA runs per SM (it holds all 512 TMEM columns)
    int smem = FmhaSmem<64>::kTotal + 1024;
    if (smem < 116 * 1024) smem = 116 * 1024;
    cudaFuncSetAttribute(fmha_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fmha_fwd_kernel<64><<<grid, kThreads, smem, stream>>>(L.tm_q, L.tm_k, L.tm_vt, L.args);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
