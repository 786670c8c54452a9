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
// The omitted set is taken as a mask over all nB block means, processed in
// 128-column tiles (kbar, w and vbar^T of a bank stay in L2).  One thread issues
// the TMA loads and MMAs; all 128 threads (one per query row) run the softmax.
// The epilogue also writes the per-block sum of (lse - old_lse) used for the
// drift centre (recap/operator.py:148-150).
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

template <int D>
struct CoarseSmem {
  static constexpr int kTileQ = 128 * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kQsq = kQ + kTileQ;
  static constexpr int kP = kQsq + kTileQ;
  static constexpr int kA = kP + 128 * 128 * 2;  // kbar tile (or U^T)
  static constexpr int kB = kA + kTileQ;         // w tile (or C_vk)
  static constexpr int kC = kB + kTileQ;         // vbar^T tile
  static constexpr int kBars = kC + 128 * D * 2;
  static constexpr int kMisc = kBars + 16;
  static constexpr int kOmit = kMisc + 16 + 128 * 4;  // tmem addr, abort, row partials
  static constexpr int kMaxBlocks = 4096;
  static constexpr int kTotal = kOmit + kMaxBlocks;
};

template <int D>
__global__ void __launch_bounds__(128, 1)
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
  uint8_t* sA = smem + L::kA;
  uint8_t* sB = smem + L::kB;
  uint8_t* sC = smem + L::kC;
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  float* row_part = reinterpret_cast<float*>(smem + L::kMisc + 16);
  uint8_t* omit = smem + L::kOmit;

  const int qb = blockIdx.x;
  const int bank = blockIdx.y;
  const int t = threadIdx.x;
  const int warp = t >> 5;
  const int lane = t & 31;
  const int nB = a.nB;

  if (t == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  const uint8_t* prow = a.partition + (static_cast<size_t>(bank) * nB + qb) * nB;
  for (int j = t; j < a.nB_pad; j += 128) omit[j] = (j < nB && prow[j] == 0) ? 1 : 0;
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s1 = tmem;        // also Q U in the prologue
  const uint32_t t_s2 = tmem + 128;
  const uint32_t t_o = tmem + 256;
  const uint32_t t_x = tmem + 384;   // Q C_vk^T
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  constexpr uint32_t kTileQ = L::kTileQ;
  uint32_t tma_phase = 0, mma_phase = 0;
  bool ok = true;

  // ---- prologue: Q tile, U^T and C_vk; Q U and Q C_vk^T
  if (t == 0) {
    prefetch_tmap(&tm_q);
    mbar_expect_tx(bar_tma, kTileQ + 2 * D * D * 2);
    const int qrow = bank * a.S_pad + qb * 128;
#pragma unroll
    for (int at = 0; at < D / 64; ++at) {
      tma_load_2d(sQ + at * 128 * 128, &tm_q, bar_tma, at * 64, qrow);
      tma_load_2d(sA + at * D * 128, &tm_ut, bar_tma, at * 64, bank * D);
      tma_load_2d(sB + at * D * 128, &tm_c, bar_tma, at * 64, bank * D);
    }
  }
  ok = mbar_wait(bar_tma, tma_phase, abort_flag, a.status, kStatusTimeoutTma);
  tma_phase ^= 1;
  if (t == 0 && ok) {
    tc_fence_after();
    constexpr uint32_t idesc = idesc_bf16_f32(128, D);
    const uint32_t q0 = smem_u32(sQ), a0 = smem_u32(sA), b0 = smem_u32(sB);
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
      const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
      const uint32_t offb = (s >> 2) * (D * 128) + (s & 3) * 32;
      mma_bf16_ss(t_s1, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(a0 + offb), idesc, s > 0);
    }
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
      const uint32_t offq = (s >> 2) * (128 * 128) + (s & 3) * 32;
      const uint32_t offb = (s >> 2) * (D * 128) + (s & 3) * 32;
      mma_bf16_ss(t_x, sdesc_k_sw128(q0 + offq), sdesc_k_sw128(b0 + offb), idesc, s > 0);
    }
    mma_commit(bar_mma);
  }
  ok = ok && mbar_wait(bar_mma, mma_phase, abort_flag, a.status, kStatusTimeoutMma);
  mma_phase ^= 1;
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
        const int k = c * 32 + q * 8;  // first element of this 16-byte chunk
        const int atom = k >> 6;
        const int chunk = (k & 63) >> 3;
        st_shared_v4(qsq_row + atom * 16384 + ((chunk ^ (t & 7)) << 4), pk[4 * q], pk[4 * q + 1],
                     pk[4 * q + 2], pk[4 * q + 3]);
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();

  // ---- main loop over 128-column tiles of block means
  const float scale = a.scale;
  const float half_s2 = 0.5f * scale * scale;
  const float s2 = scale * scale;
  const float th2 = a.theta * a.theta;
  constexpr float kLog2e = 1.4426950408889634f;
  float m_i = -INFINITY, l_i = 0.f, g_i = 0.f;
  const int n_tiles = a.nB_pad / 128;
  const uint32_t p_row = smem_u32(sP) + t * 128;
  for (int tt = 0; ok && tt < n_tiles; ++tt) {
    if (t == 0) {
      mbar_expect_tx(bar_tma, 3 * kTileQ);
      const int brow = bank * a.nB_pad + tt * 128;
#pragma unroll
      for (int at = 0; at < D / 64; ++at) {
        tma_load_2d(sA + at * 128 * 128, &tm_kbar, bar_tma, at * 64, brow);
        tma_load_2d(sB + at * 128 * 128, &tm_w, bar_tma, at * 64, brow);
      }
#pragma unroll
      for (int at = 0; at < 2; ++at)
        tma_load_2d(sC + at * D * 128, &tm_vbt, bar_tma, tt * 128 + at * 64, bank * D);
    }
    ok = mbar_wait(bar_tma, tma_phase, abort_flag, a.status, kStatusTimeoutTma);
    tma_phase ^= 1;
    if (t == 0 && ok) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_bf16_f32(128, 128);
      const uint32_t q0 = smem_u32(sQ), qs0 = smem_u32(sQsq), a0 = smem_u32(sA), b0 = smem_u32(sB);
#pragma unroll
      for (int s = 0; s < D / 16; ++s) {
        const uint32_t off = (s >> 2) * (128 * 128) + (s & 3) * 32;
        mma_bf16_ss(t_s1, sdesc_k_sw128(q0 + off), sdesc_k_sw128(a0 + off), idesc, s > 0);
      }
#pragma unroll
      for (int s = 0; s < D / 16; ++s) {
        const uint32_t off = (s >> 2) * (128 * 128) + (s & 3) * 32;
        mma_bf16_ss(t_s2, sdesc_k_sw128(qs0 + off), sdesc_k_sw128(b0 + off), idesc, s > 0);
      }
      mma_commit(bar_mma);
    }
    ok = ok && mbar_wait(bar_mma, mma_phase, abort_flag, a.status, kStatusTimeoutMma);
    mma_phase ^= 1;
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    tc_fence_after();
    float x[128];
    uint32_t gate[4];  // bit e of gate[c]: column c*32+e passed the variance gate
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v1[32], v2[32];
      tmem_ld32(t_s1 + c * 32 + lane_base, v1);
      tmem_ld32(t_s2 + c * 32 + lane_base, v2);
      tmem_wait_ld();
      uint32_t gm = 0;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int col = c * 32 + e;
        const int j = tt * 128 + col;
        const float quad = v2[e];
        const bool gt = quad * s2 <= th2;
        float sc = v1[e] * scale + a.counts_log[min(j, nB - 1)];
        sc += gt ? quad * half_s2 : 0.f;
        gm |= gt ? (1u << e) : 0u;
        x[col] = omit[j] ? sc : -INFINITY;
      }
      gate[c] = gm;
    }
    float m_ij = -INFINITY;
#pragma unroll
    for (int c = 0; c < 128; ++c) m_ij = fmaxf(m_ij, x[c]);
    const bool tile_valid = m_ij != -INFINITY;
    const float m_new = tile_valid ? fmaxf(m_i, m_ij) : m_i;
    const float alpha = tile_valid ? fast_exp2((m_i - m_new) * kLog2e) : 1.f;
    float lsum = 0.f, gsum = 0.f;
    uint32_t pk[64];
#pragma unroll
    for (int e = 0; e < 64; ++e) {
      const int c0 = 2 * e, c1 = 2 * e + 1;
      const float p0 = x[c0] == -INFINITY ? 0.f : fast_exp2((x[c0] - m_new) * kLog2e);
      const float p1 = x[c1] == -INFINITY ? 0.f : fast_exp2((x[c1] - m_new) * kLog2e);
      lsum += p0 + p1;
      gsum += (((gate[c0 >> 5] >> (c0 & 31)) & 1u) ? p0 : 0.f) +
              (((gate[c1 >> 5] >> (c1 & 31)) & 1u) ? p1 : 0.f);
      pk[e] = pack_bf16(p0, p1);
    }
    l_i = alpha * l_i + lsum;
    g_i = alpha * g_i + gsum;
    m_i = m_new;
    if (tt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(t_o + c * 32 + lane_base, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= alpha;
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
    __syncthreads();
    if (t == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_bf16_f32(128, D);
      const uint32_t p0 = smem_u32(sP), c0 = smem_u32(sC);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t offp = (s >> 2) * (128 * 128) + (s & 3) * 32;
        const uint32_t offc = (s >> 2) * (D * 128) + (s & 3) * 32;
        mma_bf16_ss(t_o, sdesc_k_sw128(p0 + offp), sdesc_k_sw128(c0 + offc), idesc,
                    (tt > 0 || s > 0) ? 1u : 0u);
      }
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase, abort_flag, a.status, kStatusTimeoutMma);
    mma_phase ^= 1;
    ok = __all_sync(0xffffffffu, ok);
  }

  // ---- epilogue
  if (ok) {
    tc_fence_after();
    const bool has_tail = l_i > 0.f;
    const float safe_l = fmaxf(l_i, 1.0e-30f);
    const float lse = has_tail ? m_i + logf(l_i) : -INFINITY;
    const float gfrac = has_tail ? g_i / safe_l : 0.f;
    const float g_bf = bf16_round(gfrac);
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
          const float o = has_tail ? bf16_round(ov[2 * e + h] / safe_l) : 0.f;
          const float drift = bf16_round(scale * bf16_round(xv[2 * e + h]));
          res[h] = o + bf16_round(g_bf * drift);
        }
        w[e] = pack_bf16(res[0], res[1]);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) d4[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
    a.lse[orow] = lse;
    if (a.center_partial != nullptr) {
      float dv = lse - a.old_lse[orow];
      for (int o = 16; o > 0; o >>= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
      if (lane == 0) row_part[warp] = dv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ok && t == 0 && a.center_partial != nullptr)
    a.center_partial[static_cast<size_t>(bank) * (a.rows / 128) + qb] =
        ((row_part[0] + row_part[1]) + (row_part[2] + row_part[3]));
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_coarse(const CoarseLaunch& L, cudaStream_t s) {
  const CoarseArgs& a = L.args;
  if (a.rows % 128 || a.nB_pad % 128 || a.nB_pad > CoarseSmem<128>::kMaxBlocks) return kErrShape;
  if (a.rows == 0) return kOk;
  dim3 grid(a.rows / 128, a.banks);
  if (L.D == 128) {
    const int smem = CoarseSmem<128>::kTotal + 1024;
    cudaFuncSetAttribute(coarse_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    coarse_kernel<128><<<grid, 128, smem, s>>>(L.tm_q, L.tm_basis_t, L.tm_cvk, L.tm_kmean, L.tm_var,
                                               L.tm_vmean_t, a);
  } else if (L.D == 64) {
    int smem = CoarseSmem<64>::kTotal + 1024;
    if (smem < 120 * 1024) smem = 120 * 1024;  // one CTA per SM: it holds all 512 TMEM columns
    cudaFuncSetAttribute(coarse_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    coarse_kernel<64><<<grid, 128, smem, s>>>(L.tm_q, L.tm_basis_t, L.tm_cvk, L.tm_kmean, L.tm_var,
                                              L.tm_vmean_t, a);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
