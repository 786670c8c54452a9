// Corrected coarse tail on sm_100a tensor cores.
//
// For a 128-row query block i of bank b (rows < rows), every omitted key block j
// (partition[b][i][j] == 0, j < nB) enters a softmax with the logit
//     s q.kbar_j + ln n_j + [ s^2/2 (qsq . w_j)  if s^2 (qsq . w_j) <= theta^2 ]
// and the output is  o + g * drift,  with g the gated share of the mass
// (_coarse_tail_kernel, recap/kernels/coarse_tail.py:36-186, and its wrapper
// 194-312).  qsq = (Q U)^2 and drift = s Q C_vk^T (rotated_query_square and
// value_drift, recap/sparse/closure.py:84-93) are computed here from the Q tile
// with two tcgen05 MMAs and never reach HBM.  Rounding follows the reference:
// kbar, vbar, w, U and C_vk in bf16, qsq and drift rounded to bf16 as the bf16
// bmm outputs they replace, P rounded to bf16 before P vbar, the output rounded
// to bf16 and the drift added in bf16 arithmetic.
//
// The omitted set is a mask over all nB block means, processed in 64-column tiles
// (kbar, w and vbar^T of a bank stay in L2).  One CTA per (query block, bank), 8 warps:
//   warp 0      TMA producer: Q, U^T and C_vk once, then (kbar, w, vbar^T) tiles
//               through a 2-stage ring;
//   warp 1      TMEM allocator and MMA issuer: Q U and Q C_vk^T, then per tile
//               S1 = Q kbar^T and S2 = qsq w^T into one of two TMEM buffer pairs,
//               and O += P vbar;
//   warps 4-7   one query row per thread: qsq, the gated online softmax (log2 domain,
//               lazy rescaling of O), P in shared memory, the epilogue.
// The epilogue also writes the per-block sum of (lse - old_lse) for the drift centre
// (recap/operator.py:148-150).
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

constexpr int kThreads = 256;
constexpr int kSoftmaxWarp0 = 4;
constexpr int kTileN = 64;          // block means per tile
constexpr int kStages = 2;
constexpr int kMaxBlocks = 4096;    // nB_pad limit (column terms in shared memory)
constexpr float kRescaleThreshold = 8.0f;

template <int D>
struct CoarseSmem {
  static constexpr int kTileQ = 128 * D * 2;
  static constexpr int kOpK = kTileN * D * 2;      // kbar tile: 64 rows x D
  static constexpr int kOpW = kTileN * D * 2;      // w tile
  static constexpr int kOpV = D * kTileN * 2;      // vbar^T tile: D rows x 64
  static constexpr int kStage = kOpK + kOpW + kOpV;
  static constexpr int kQ = 0;
  static constexpr int kQsq = kQ + kTileQ;
  static constexpr int kP = kQsq + kTileQ;         // 128 x 64 bf16, one swizzle atom
  static constexpr int kRing = kP + 128 * kTileN * 2;
  // U^T (D x D) and C_vk (D x D) share the ring before the first tile
  static constexpr int kRingBytes = (kStages * kStage > 2 * D * D * 2) ? kStages * kStage : 2 * D * D * 2;
  static constexpr int kCol = kRing + kRingBytes;  // fp32 column terms [kMaxBlocks]
  static constexpr int kBars = kCol + kMaxBlocks * 4;
  // bars: pro_full, pro_done, qsq_ready, full[2], empty[2], sfull[2], sfree[2], pfull, ofull, done
  static constexpr int kNumBars = 3 + 4 * kStages + 3 + 2;
  static constexpr int kMisc = kBars + kNumBars * 8;
  static constexpr int kTotal = kMisc + 16 + 4 * 4;
};

struct CoarseBars {
  uint64_t *pro_full, *pro_done, *qsq_ready, *full, *empty, *sfull, *sfree, *pfull, *ofull, *done;
};

__device__ __forceinline__ CoarseBars carve(uint8_t* base) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  CoarseBars r;
  r.pro_full = b;
  r.pro_done = b + 1;
  r.qsq_ready = b + 2;
  r.full = b + 3;
  r.empty = b + 3 + kStages;
  r.sfull = b + 3 + 2 * kStages;
  r.sfree = b + 3 + 3 * kStages;
  r.pfull = b + 3 + 4 * kStages;
  r.ofull = b + 4 + 4 * kStages;
  r.done = b + 5 + 4 * kStages;
  return r;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    coarse_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_ut,
                  const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_kbar,
                  const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_vbt,
                  const CoarseArgs a) {
  using L = CoarseSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sQsq = smem + L::kQsq;
  uint8_t* sP = smem + L::kP;
  uint8_t* sRing = smem + L::kRing;
  float* colterm = reinterpret_cast<float*>(smem + L::kCol);
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

  if (threadIdx.x == 0) {
    mbar_init(bars.pro_full, 1);
    mbar_init(bars.pro_done, 1);
    mbar_init(bars.qsq_ready, 4);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bars.full + s, 1);
      mbar_init(bars.empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bars.sfull + b, 1);
      mbar_init(bars.sfree + b, 4);
    }
    mbar_init(bars.pfull, 4);
    mbar_init(bars.ofull, 1);
    mbar_init(bars.done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  {
    // per-column term: ln n_j for omitted blocks, -inf for selected or padding ones
    const uint8_t* prow = a.partition + (static_cast<size_t>(bank) * nB + qb) * nB;
    for (int j = threadIdx.x; j < a.nB_pad; j += kThreads)
      colterm[j] = (j < nB && prow[j] == 0) ? a.counts_log[j] : -INFINITY;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s1 = tmem;          // S1 buffers: columns [0,64) and [64,128); Q U in [0, D)
  const uint32_t t_s2 = tmem + 128;    // S2 buffers: columns [128,192) and [192,256)
  const uint32_t t_o = tmem + 256;     // O: columns [256, 256 + D)
  const uint32_t t_x = tmem + 384;     // Q C_vk^T: columns [384, 384 + D)
  constexpr uint32_t kTileQ = L::kTileQ;

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0) {
      const uint64_t keep = l2_evict_last();    // per-bank operands: read by every query block
      const uint64_t stream = l2_evict_first(); // the Q tile: read once here
      const int qrow = bank * a.S_pad + qb * 128;
      mbar_expect_tx(bars.pro_full, kTileQ + 2 * D * D * 2);
#pragma unroll
      for (int at = 0; at < D / 64; ++at) {
        tma_load_2d_hint(sQ + at * 128 * 128, &tm_q, bars.pro_full, at * 64, qrow, stream);
        tma_load_2d(sRing + at * D * 128, &tm_ut, bars.pro_full, at * 64, bank * D);
        tma_load_2d(sRing + D * D * 2 + at * D * 128, &tm_c, bars.pro_full, at * 64, bank * D);
      }
      // the ring holds U^T and C_vk until the prologue MMAs have read them
      bool ok = mbar_wait(bars.pro_done, 0, abort_flag, a.status, kStatusTimeoutProducer);
      int j = 0;
      for (; ok && j < n_tiles; ++j) {
        const int st = j % kStages;
        if (j >= kStages &&
            !mbar_wait(bars.empty + st, ((j / kStages) - 1) & 1, abort_flag, a.status, kStatusTimeoutProducer))
          break;
        uint8_t* base = sRing + st * L::kStage;
        const int brow = bank * a.nB_pad + j * kTileN;
        mbar_expect_tx(bars.full + st, L::kStage);
#pragma unroll
        for (int at = 0; at < D / 64; ++at) {
          tma_load_2d_hint(base + at * kTileN * 128, &tm_kbar, bars.full + st, at * 64, brow, keep);
          tma_load_2d_hint(base + L::kOpK + at * kTileN * 128, &tm_w, bars.full + st, at * 64, brow, keep);
        }
        tma_load_2d_hint(base + L::kOpK + L::kOpW, &tm_vbt, bars.full + st, j * kTileN, bank * D, keep);
      }
      const int first = j > kStages ? j - kStages : 0;
      for (int k = first; k < j; ++k) mbar_drain(bars.full + (k % kStages), (k / kStages) & 1);
      mbar_drain(bars.pro_full, 0);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      const uint32_t q0 = smem_u32(sQ), qs0 = smem_u32(sQsq), p0 = smem_u32(sP), ring = smem_u32(sRing);
      bool ok = mbar_wait(bars.pro_full, 0, abort_flag, a.status, kStatusTimeoutTma);
      if (ok) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, D);
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t offb = (s >> 2) * (D * 128) + (s & 3) * 32;
          mma_bf16_ss(t_s1, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(ring + offb), idesc, s > 0);
          mma_bf16_ss(t_x, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(ring + D * D * 2 + offb), idesc, s > 0);
        }
        mma_commit(bars.pro_done);
        ok = mbar_wait(bars.qsq_ready, 0, abort_flag, a.status, kStatusTimeoutMma);
      }
      auto issue_s = [&](int j) -> bool {
        const int st = j % kStages;
        if (!mbar_wait(bars.full + st, (j / kStages) & 1, abort_flag, a.status, kStatusTimeoutTma)) return false;
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(bars.sfree + b, ((j >> 1) - 1) & 1, abort_flag, a.status, kStatusTimeoutMma))
          return false;
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, kTileN);
        const uint32_t kb = ring + st * L::kStage;
        const uint32_t wb = kb + L::kOpK;
#pragma unroll
        for (int s = 0; s < D / 16; ++s) {
          const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
          const uint32_t offb = (s >> 2) * (kTileN * 128) + (s & 3) * 32;
          mma_bf16_ss(t_s1 + b * kTileN, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(kb + offb), idesc, s > 0);
          mma_bf16_ss(t_s2 + b * kTileN, sdesc_k_sw128(qs0 + offq), sdesc_k_sw128(wb + offb), idesc, s > 0);
        }
        mma_commit(bars.sfull + b);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(bars.pfull, j & 1, abort_flag, a.status, kStatusTimeoutMma)) return false;
        tc_fence_after();
        const int st = j % kStages;
        constexpr uint32_t idesc = idesc_bf16_f32(128, D);
        const uint32_t vb = ring + st * L::kStage + L::kOpK + L::kOpW;
#pragma unroll
        for (int s = 0; s < kTileN / 16; ++s)
          mma_bf16_ss(t_o, sdesc_k_sw128(p0 + s * 32), sdesc_k_sw128(vb + s * 32), idesc, (j > 0 || s > 0) ? 1u : 0u);
        mma_commit(bars.empty + st);
        mma_commit(bars.ofull);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 1; ok && j < n_tiles; ++j) {
        ok = issue_s(j);
        if (ok) ok = issue_pv(j - 1);
      }
      if (ok) ok = issue_pv(n_tiles - 1);
      mma_commit(bars.done);
      mbar_drain(bars.done, 0);
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ================================================================ softmax + epilogue
    const int t = threadIdx.x - kSoftmaxWarp0 * 32;
    const int q4 = warp - kSoftmaxWarp0;
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    constexpr float kLog2e = 1.4426950408889634f;
    const float scale = a.scale;
    const float s2 = scale * scale;
    const float half_s2 = 0.5f * s2;
    const float th2 = a.theta * a.theta;
    bool ok = mbar_wait(bars.pro_done, 0, abort_flag, a.status, kStatusTimeoutSoftmax);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      // qsq = bf16(bf16(q U)^2), written as the K-major A operand of qsq . w^T
      const uint32_t qsq_row = smem_u32(sQsq) + t * 128;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(t_s1 + c * 32 + lane_base, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float x0 = bf16_round(v[2 * e]);
          const float x1 = bf16_round(v[2 * e + 1]);
          pk[e] = pack_bf16(x0 * x0, x1 * x1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = c * 32 + q * 8;
          st_shared_v4(qsq_row + (k >> 6) * 16384 + ((((k & 63) >> 3) ^ (t & 7)) << 4), pk[4 * q], pk[4 * q + 1],
                       pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.qsq_ready);
    }
    float m_run = -INFINITY;  // running max (log2 domain)
    float l_run = 0.f, g_run = 0.f;
    const uint32_t p_row = smem_u32(sP) + t * 128;
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int b = j & 1;
      ok = mbar_wait(bars.sfull + b, (j >> 1) & 1, abort_flag, a.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float x[kTileN];
      uint32_t gate[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v1[32], v2[32];
        tmem_ld32(t_s1 + b * kTileN + c * 32 + lane_base, v1);
        tmem_ld32(t_s2 + b * kTileN + c * 32 + lane_base, v2);
        tmem_wait_ld();
        uint32_t gm = 0;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float quad = v2[e];
          const bool gt = quad * s2 <= th2;
          gm |= gt ? (1u << e) : 0u;
          const float term = colterm[j * kTileN + c * 32 + e];
          // natural-log logit, then into the log2 domain
          const float sc = v1[e] * scale + term + (gt ? quad * half_s2 : 0.f);
          x[c * 32 + e] = sc * kLog2e;
        }
        gate[c] = gm;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.sfree + b);
      float mxa[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mxa[k] = x[k];
#pragma unroll
      for (int i = 8; i < kTileN; ++i) mxa[i & 7] = fmaxf(mxa[i & 7], x[i]);
      const float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                             fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
      float alpha = 1.f;
      bool rescale = false;
      if (mx != -INFINITY) {
        if (m_run == -INFINITY) {
          m_run = mx;
        } else if (mx > m_run + kRescaleThreshold) {
          alpha = fast_exp2(m_run - mx);
          m_run = mx;
          rescale = true;
        }
      }
      float ls[4] = {0.f, 0.f, 0.f, 0.f}, gs[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[kTileN / 2];
#pragma unroll
      for (int e = 0; e < kTileN / 2; ++e) {
        const int c0 = 2 * e, c1 = 2 * e + 1;
        const float p0 = x[c0] == -INFINITY ? 0.f : fast_exp2(x[c0] - m_run);
        const float p1 = x[c1] == -INFINITY ? 0.f : fast_exp2(x[c1] - m_run);
        ls[e & 3] += p0 + p1;
        gs[e & 3] += (((gate[c0 >> 5] >> (c0 & 31)) & 1u) ? p0 : 0.f) + (((gate[c1 >> 5] >> (c1 & 31)) & 1u) ? p1 : 0.f);
        pk[e] = pack_bf16(p0, p1);
      }
      const float lsum = (ls[0] + ls[1]) + (ls[2] + ls[3]);
      const float gsum = (gs[0] + gs[1]) + (gs[2] + gs[3]);
      l_run = l_run * alpha + lsum;
      g_run = g_run * alpha + gsum;
      if (j > 0) {
        ok = mbar_wait(bars.ofull, (j - 1) & 1, abort_flag, a.status, kStatusTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
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
      }
#pragma unroll
      for (int c = 0; c < kTileN / 8; ++c)
        st_shared_v4(p_row + ((c ^ (t & 7)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.pfull);
    }
    if (ok) {
      ok = mbar_wait(bars.ofull, (n_tiles - 1) & 1, abort_flag, a.status, kStatusTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const bool has_tail = l_run > 0.f;
      const float safe_l = fmaxf(l_run, 1.0e-30f);
      const float inv_l = 1.f / safe_l;
      const float lse = has_tail ? (m_run + __log2f(l_run)) * 0.69314718055994531f : -INFINITY;
      const float g_bf = bf16_round(has_tail ? g_run * inv_l : 0.f);
      const int r = qb * 128 + t;
      const size_t orow = static_cast<size_t>(bank) * a.rows + r;
      __nv_bfloat16* dst = a.out + orow * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float ov[32], xv[32];
        tmem_ld32(t_o + c * 32 + lane_base, ov);
        tmem_ld32(t_x + c * 32 + lane_base, xv);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float res[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float o = has_tail ? bf16_round(ov[2 * e + h] * inv_l) : 0.f;
            const float drift = bf16_round(scale * bf16_round(xv[2 * e + h]));
            res[h] = o + bf16_round(g_bf * drift);
          }
          w[e] = pack_bf16(res[0], res[1]);
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) st_stream_v4(d4 + q, make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]));
      }
      a.lse[orow] = lse;
      if (a.center_partial != nullptr) {
        float dv = lse - a.old_lse[orow];
        for (int o = 16; o > 0; o >>= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
        if (lane == 0) row_part[q4] = dv;
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

}  // namespace

int launch_coarse(const CoarseLaunch& L, cudaStream_t s) {
  const CoarseArgs& a = L.args;
  if (a.rows % 128 || a.nB_pad % 128 || a.nB_pad > kMaxBlocks) return kErrShape;
  if (a.rows == 0) return kOk;
  dim3 grid(a.rows / 128, a.banks);
  if (L.D == 128) {
    const int smem = CoarseSmem<128>::kTotal + 1024;
    cudaFuncSetAttribute(coarse_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    coarse_kernel<128><<<grid, kThreads, smem, s>>>(L.tm_q, L.tm_basis_t, L.tm_cvk, L.tm_kmean, L.tm_var,
                                                    L.tm_vmean_t, a);
  } else if (L.D == 64) {
    int smem = CoarseSmem<64>::kTotal + 1024;
    if (smem < 120 * 1024) smem = 120 * 1024;  // one CTA per SM: it holds all 512 TMEM columns
    cudaFuncSetAttribute(coarse_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    coarse_kernel<64><<<grid, kThreads, smem, s>>>(L.tm_q, L.tm_basis_t, L.tm_cvk, L.tm_kmean, L.tm_var,
                                                   L.tm_vmean_t, a);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
