// Pooled value-key covariance C_vk = sum_t v_t (k_t - kbar_blk(t))^T / N on tensor cores
// (_batched_centered_cross_fp32_kernel and pooled_cross_centered_triton_fp32,
// recap/kernels/closure_stats.py:27-94, 245-290).
//
// A split-K GEMM over the video tokens: CTA (chunk, bank) accumulates
//     P[bank][chunk] = V^T[:, chunk] * Kc[:, chunk]^T          (D x D, fp32 in TMEM)
// from the two K-major operands the layout pass writes: V^T [banks, D, S_pad] and the
// block-centred keys Kc^T [banks, D, S_pad] (bf16, zero outside the video tokens).  The
// chunk partials are then added in a fixed order and divided by N.  The reference keeps
// the centred keys in fp32 (split into two bf16 terms); here they are rounded once to
// bf16, an unbiased per-element rounding whose effect on the sum is far below the bf16
// rounding C_vk itself gets before use (recap/sparse/closure.py:93).
//
// Warp 0 streams 64-token slices of both operands through a 4-slot TMA ring, warp 1 issues
// tcgen05.mma (M = 128: for D = 64 the upper 64 rows belong to the next bank and are
// discarded), warps 2-5 read the accumulator out of TMEM.
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

constexpr int kNst = 4;
constexpr int kStepTokens = 64;
constexpr int kStepsPerChunk = 64;  // 4096 tokens per CTA

template <int D>
struct CvkSmem {
  static constexpr int kA = 128 * kStepTokens * 2;  // V^T slice, 128 rows
  static constexpr int kB = D * kStepTokens * 2;    // Kc^T slice, D rows
  static constexpr int kStage = kA + kB;
  static constexpr int kBars = kNst * kStage;
  static constexpr int kMisc = kBars + (2 * kNst + 1) * 8;
  static constexpr int kTotal = kMisc + 16;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    cvk_kernel(const __grid_constant__ CUtensorMap tm_vt, const __grid_constant__ CUtensorMap tm_kct,
               const CvkArgs a) {
  using L = CvkSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* empty = full + kNst;
  uint64_t* done = empty + kNst;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int chunk = blockIdx.x;
  const int bank = blockIdx.y;
  const int step0 = chunk * kStepsPerChunk;
  const int n_steps = min(kStepsPerChunk, a.video_steps - step0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNst; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, D < 32 ? 32 : D);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n_steps > 0) {
      int i = 0;
      for (; i < n_steps; ++i) {
        const int slot = i % kNst;
        if (i >= kNst &&
            !mbar_wait(empty + slot, ((i / kNst) - 1) & 1, abort_flag, a.status, kStatusTimeoutProducer))
          break;
        uint8_t* st = smem + slot * L::kStage;
        const int x = (step0 + i) * kStepTokens;
        mbar_expect_tx(full + slot, L::kStage);
        tma_load_2d(st, &tm_vt, full + slot, x, bank * D);
        tma_load_2d(st + L::kA, &tm_kct, full + slot, x, bank * D);
      }
      const int first = i > kNst ? i - kNst : 0;
      for (int k = first; k < i; ++k) mbar_drain(full + (k % kNst), (k / kNst) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_steps > 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, D);
      const uint32_t base = smem_u32(smem);
      for (int i = 0; i < n_steps; ++i) {
        const int slot = i % kNst;
        if (!mbar_wait(full + slot, (i / kNst) & 1, abort_flag, a.status, kStatusTimeoutTma)) break;
        tc_fence_after();
        const uint32_t sa = base + slot * L::kStage;
        const uint32_t sb = sa + L::kA;
#pragma unroll
        for (int k = 0; k < kStepTokens / 16; ++k)
          mma_bf16_ss(tmem, sdesc_k_sw128(sa + k * 32), sdesc_k_sw128(sb + k * 32), idesc, (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(empty + slot);
      }
      mma_commit(done);
    }
  } else {
    // epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. +31
    const int quarter = warp & 3;
    const int m = quarter * 32 + lane;  // row of C_vk (value dimension)
    bool ok = n_steps > 0;
    if (ok) ok = mbar_wait(done, 0, abort_flag, a.status, kStatusTimeoutMma);
    ok = __all_sync(0xffffffffu, ok);
    float* out = a.partial + ((static_cast<size_t>(bank) * gridDim.x + chunk) * D) * D;
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, v);
        tmem_wait_ld();
        if (m < D) {
          float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(m) * D + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
      }
    } else if (n_steps <= 0 && m < D) {
      for (int n = 0; n < D; ++n) out[static_cast<size_t>(m) * D + n] = 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, D < 32 ? 32 : D);
  }
}

}  // namespace

int cvk_chunks(int n_video) {
  const int steps = (n_video + kStepTokens - 1) / kStepTokens;
  return (steps + kStepsPerChunk - 1) / kStepsPerChunk;
}

int launch_cvk(const CvkLaunch& L, cudaStream_t s) {
  const CvkArgs& a = L.args;
  const int nch = cvk_chunks(a.n_video);
  if (nch <= 0 || a.banks <= 0) return kErrShape;
  dim3 grid(nch, a.banks);
  if (L.D == 128) {
    const int smem = CvkSmem<128>::kTotal + 1024;
    cudaFuncSetAttribute(cvk_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cvk_kernel<128><<<grid, 192, smem, s>>>(L.tm_vt, L.tm_kct, a);
  } else if (L.D == 64) {
    // at least ~115 KB so that one CTA runs per SM
    int smem = CvkSmem<64>::kTotal + 1024;
    if (smem < 116 * 1024) smem = 116 * 1024;
    cudaFuncSetAttribute(cvk_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cvk_kernel<64><<<grid, 192, smem, s>>>(L.tm_vt, L.tm_kct, a);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
