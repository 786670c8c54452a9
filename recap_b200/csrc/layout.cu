// Layout gather fused with block pooling and the per-call closure statistics of K.
//
// One pass over the native-order Q, K and V of a layer call, one CTA per 128-token block:
//  * reorders the tokens into [Hilbert-ordered video | text] (Layout.reorder,
//    recap/sparse/layout.py:86-90), writing Q and K as [banks, S_pad, D] and V
//    transposed as [banks, D, S_pad] (the K-major operand layout of P V);
//  * sums each block over its video tokens in fp32 and divides by the token count
//    (pool_blocks, recap/sparse/pooling.py:10-34): fp32 means plus the bf16 copies the
//    coarse tail reads;
//  * writes the block-centred video keys k - kbar, transposed and rounded to bf16, as
//    the K-major B operand of the C_vk GEMM (recap/kernels/closure_stats.py:27-94);
//  * with a basis U and 0 < rank < D, the rank-folded per-block key variances in U
//    (rotated_leaf_moments_triton + fold_rank, recap/kernels/closure_stats.py:96-189,
//    recap/sparse/closure.py:96-104): the leading `rank` columns are the two-pass
//    population variances of K U[:, c]; every other column is their mean, which for an
//    orthonormal U equals (trace of the block covariance - the leading variances) /
//    (D - rank), so only K U[:, :rank] is formed.
//  * the norm bounds the softmax kernels use to skip their running-max work: the
//    largest |k| over each block's tokens and |bf16(kbar)| of each video block.
// Rows past S (up to S_pad) are written as zeros.  HBM-bound.
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRank = 8;

__device__ __forceinline__ void add8(float (&acc)[8], const uint4& w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(h[e]);
    acc[2 * e] += f.x;
    acc[2 * e + 1] += f.y;
  }
}

// Staged 128 x D bf16 tiles: rows of D * 2 bytes, the 16-byte chunks of row r stored at
// chunk ^ ((r / 8) mod (D / 8)).  Lanes that read eight consecutive rows of one column
// (the transposed stores) then see distinct chunks; lanes that read a row see a
// permutation of its chunks.
template <int D>
__device__ __forceinline__ uint32_t stage_off(int r, int chunk) {
  constexpr int CPR = D / 8;
  return static_cast<uint32_t>(r * (D * 2) + ((chunk ^ ((r >> 3) & (CPR - 1))) << 4));
}
template <int D>
__device__ __forceinline__ __nv_bfloat16 stage_elem(const uint8_t* tile, int r, int d) {
  return *reinterpret_cast<const __nv_bfloat16*>(tile + stage_off<D>(r, d >> 3) + (d & 7) * 2);
}

template <int D>
struct GatherSmem {
  static constexpr int kV = 0;
  static constexpr int kK = kV + 128 * D * 2;
  static constexpr int kRed = kK + 128 * D * 2;              // [RPP][D] fp32
  static constexpr int kMean = kRed + 32 * D * 4;            // [D] fp32 key means
  static constexpr int kRot = kMean + D * 4;                 // [2 halves][128][kMaxRank] fp32
  static constexpr int kUs = kRot + 2 * 128 * kMaxRank * 4;  // [D][kMaxRank] leading basis columns
  static constexpr int kStat = kUs + D * kMaxRank * 4;       // [2*kMaxRank + 1]
  static constexpr int kTotal = kStat + 64 * 4;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 2) gather_kernel(const GatherArgs a) {
  using L = GatherSmem<D>;
  constexpr int CPR = D / 8;              // 16-byte chunks per row
  constexpr int RPP = kThreads / CPR;     // rows per pass
  constexpr int PASSES = 128 / RPP;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* vtile = smem + L::kV;
  uint8_t* ktile = smem + L::kK;
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* kmean_s = reinterpret_cast<float*>(smem + L::kMean);
  float* rot = reinterpret_cast<float*>(smem + L::kRot);
  float* us = reinterpret_cast<float*>(smem + L::kUs);
  float* stat = reinterpret_cast<float*>(smem + L::kStat);

  const int blk = blockIdx.x;
  const int bank = blockIdx.y;
  const int bi = bank / a.heads;
  const int hi = bank - bi * a.heads;
  const int tid = threadIdx.x;
  const int ch = tid % CPR;
  const int rsub = tid / CPR;
  const int row0 = blk * 128;
  const int video_rows = min(128, a.n_video - row0);  // <= 0 for text-only blocks
  const bool need_k_tile = (a.kct != nullptr || a.variance != nullptr) && video_rows > 0;

  // The variance pass's leading basis columns U[d][0 .. rank), staged now: their loads
  // overlap the gathers (us is read only after the later barriers).
  if (a.variance != nullptr && blk < a.nB && video_rows > 0 && tid < D) {
    const float* U = a.basis + (static_cast<size_t>(bank) * D + tid) * D;
    for (int c = 0; c < a.rank; ++c) us[tid * kMaxRank + c] = U[c];
  }

  // Native rows of this thread's PASSES rows, then each tensor's PASSES row chunks in
  // one burst of independent loads (two tensors in flight): the pass is bound by the
  // latency of these gathers.
  int nat[PASSES];
#pragma unroll
  for (int p = 0; p < PASSES; ++p) {
    const int r = row0 + p * RPP + rsub;
    int n = -1;
    if (r < a.S) {
      n = a.src_row[r];
      if (n < 0 || n >= a.S) n = -1;  // a corrupt index reads nothing out of bounds
    }
    nat[p] = n;
  }
  auto load_rows = [&](int t, uint4 (&v)[PASSES]) {
    const __nv_bfloat16* src = a.src[t];
    if (src == nullptr) return;
    const __nv_bfloat16* base = src + bi * a.stride_b[t] + hi * a.stride_h[t] + ch * 8;
#pragma unroll
    for (int p = 0; p < PASSES; ++p)
      v[p] = nat[p] >= 0 ? ld_stream_v4(base + static_cast<int64_t>(nat[p]) * a.stride_s[t]) : make_uint4(0, 0, 0, 0);
  };
  float knorm2 = 0.f;  // largest |k|^2 over this thread's rows
  auto process = [&](int t, const uint4 (&v)[PASSES]) {
    if (a.src[t] == nullptr) return;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int p = 0; p < PASSES; ++p) {
      const int rl = p * RPP + rsub;
      const int r = row0 + rl;
      const uint4 val = v[p];
      if (t == 0 && a.qr) {
        *reinterpret_cast<uint4*>(a.qr + (static_cast<size_t>(bank) * a.S_pad + r) * D + ch * 8) = val;
      } else if (t == 1) {
        if (a.kr)
          *reinterpret_cast<uint4*>(a.kr + (static_cast<size_t>(bank) * a.S_pad + r) * D + ch * 8) = val;
        if (need_k_tile) *reinterpret_cast<uint4*>(ktile + stage_off<D>(rl, ch)) = val;
      } else if (t == 2) {
        *reinterpret_cast<uint4*>(vtile + stage_off<D>(rl, ch)) = val;
      }
      if (rl < video_rows) add8(acc, val);
      if (t == 1 && a.k_norm_max) {
        // |k|^2 of row rl: this lane's 8 dims, summed over the 16 lanes of the row
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&val);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
        }
#pragma unroll
        for (int o = CPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        knorm2 = fmaxf(knorm2, ss);
      }
    }
    const bool want_mean = blk < a.nB && (a.mean[t] != nullptr || (t == 1 && (need_k_tile || a.k_mean_norm)));
    if (want_mean) {
#pragma unroll
      for (int e = 0; e < 8; ++e) red[rsub * D + ch * 8 + e] = acc[e];
      __syncthreads();
      if (tid < D) {
        float sum = 0.f;
#pragma unroll 4
        for (int g = 0; g < RPP; ++g) sum += red[g * D + tid];
        const float m = sum / static_cast<float>(video_rows);
        if (t == 1) {
          kmean_s[tid] = m;
          if (a.k_mean_norm) {
            // |bf16(kbar)|^2 over the D columns (threads 0 .. D-1, whole warps)
            const float mb = __bfloat162float(__float2bfloat16_rn(m));
            float q = mb * mb;
            for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            if ((tid & 31) == 0) stat[32 + (tid >> 5)] = q;
          }
        }
        if (a.mean[t]) a.mean[t][(static_cast<size_t>(bank) * a.nB + blk) * D + tid] = m;
        if (t == 1 && a.kmean_bf16)
          a.kmean_bf16[(static_cast<size_t>(bank) * a.nB_pad + blk) * D + tid] = __float2bfloat16_rn(m);
        if (t == 2 && a.vmean_t_bf16)
          a.vmean_t_bf16[(static_cast<size_t>(bank) * D + tid) * a.nB_pad + blk] = __float2bfloat16_rn(m);
      }
      __syncthreads();
      if (t == 1 && a.k_mean_norm && tid == 0) {
        float q = 0.f;
        for (int w = 0; w < D / 32; ++w) q += stat[32 + w];
        a.k_mean_norm[static_cast<size_t>(bank) * a.nB + blk] = sqrtf(q);
      }
    }
  };
  {
    uint4 va[PASSES], vb[PASSES];
    load_rows(0, va);
    load_rows(1, vb);
    process(0, va);
    load_rows(2, va);
    process(1, vb);
    process(2, va);
  }
  if (a.k_norm_max) {
    // block maximum of the row norms: warp maxima, then one thread
    float m2 = knorm2;
    for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
    if ((tid & 31) == 0) stat[48 + (tid >> 5)] = m2;
    __syncthreads();
    if (tid == 0) {
      float mm = 0.f;
      for (int w = 0; w < kThreads / 32; ++w) mm = fmaxf(mm, stat[48 + w]);
      a.k_norm_max[static_cast<size_t>(bank) * (a.S_pad / 128) + blk] = sqrtf(mm);
    }
  }

  __syncthreads();  // the staged V and K tiles are complete before anyone reads them back
  // Transposed stores (V^T and the centred K^T): for each head dimension d this block
  // owns 128 contiguous bf16 (256 bytes) of row d.  A half-warp writes one such row, each
  // lane 8 consecutive tokens (16 bytes); a warp covers two dimensions per step.
  {
    const int lane = tid & 31;
    const int g = lane & 15;   // tokens 8g .. 8g + 7
    const int dd = lane >> 4;  // which of the warp's two dimensions
    constexpr int kWarps = kThreads / 32;
    if (a.vt != nullptr && a.src[2] != nullptr) {
      for (int d0 = 2 * (tid >> 5); d0 < D; d0 += 2 * kWarps) {
        const int d = d0 + dd;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat16 lo = stage_elem<D>(vtile, 8 * g + 2 * e, d);
          const __nv_bfloat16 hi = stage_elem<D>(vtile, 8 * g + 2 * e + 1, d);
          w[e] = static_cast<uint32_t>(__bfloat16_as_ushort(lo)) |
                 (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
        }
        *reinterpret_cast<uint4*>(a.vt + (static_cast<size_t>(bank) * D + d) * a.S_pad + row0 + 8 * g) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    if (a.kct != nullptr) {
      // centred video keys, bf16; zero outside the video tokens
      for (int d0 = 2 * (tid >> 5); d0 < D; d0 += 2 * kWarps) {
        const int d = d0 + dd;
        const float m = video_rows > 0 ? kmean_s[d] : 0.f;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r0 = 8 * g + 2 * e;
          const float x0 = r0 < video_rows ? __bfloat162float(stage_elem<D>(ktile, r0, d)) - m : 0.f;
          const float x1 = r0 + 1 < video_rows ? __bfloat162float(stage_elem<D>(ktile, r0 + 1, d)) - m : 0.f;
          const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
          w[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(a.kct + (static_cast<size_t>(bank) * D + d) * a.S_pad + row0 + 8 * g) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }

  if (a.variance != nullptr && blk < a.nB && video_rows > 0) {
    const int rank = a.rank;
    // rotated values of the leading columns: rot[r][c] = sum_d k[r][d] U[d][c], thread
    // (half, r) summing its half of the head dimension; and the trace of the block
    // covariance, sum_d sum_r (k[r][d] - m_d)^2, thread (half, d) over its half of the rows
    const int r = tid & 127;
    const int half = tid >> 7;
    {
      float acc[kMaxRank];
#pragma unroll
      for (int c = 0; c < kMaxRank; ++c) acc[c] = 0.f;
      if (r < video_rows) {
#pragma unroll 2
        for (int j = half * (CPR / 2); j < (half + 1) * (CPR / 2); ++j) {
          const uint4 w = *reinterpret_cast<const uint4*>(ktile + stage_off<D>(r, j));
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            const int d = j * 8 + 2 * e;
            const float4 u0a = *reinterpret_cast<const float4*>(us + d * kMaxRank);
            const float4 u0b = *reinterpret_cast<const float4*>(us + d * kMaxRank + 4);
            const float4 u1a = *reinterpret_cast<const float4*>(us + (d + 1) * kMaxRank);
            const float4 u1b = *reinterpret_cast<const float4*>(us + (d + 1) * kMaxRank + 4);
            const float ua[8] = {u0a.x, u0a.y, u0a.z, u0a.w, u0b.x, u0b.y, u0b.z, u0b.w};
            const float ub[8] = {u1a.x, u1a.y, u1a.z, u1a.w, u1b.x, u1b.y, u1b.z, u1b.w};
#pragma unroll
            for (int c = 0; c < kMaxRank; ++c)
              if (c < rank) acc[c] = fmaf(f.y, ub[c], fmaf(f.x, ua[c], acc[c]));
          }
        }
      }
#pragma unroll
      for (int c = 0; c < kMaxRank; ++c) rot[(half * 128 + r) * kMaxRank + c] = acc[c];
    }
    float tr = 0.f;
    {
      const int d = tid & (D - 1);
      const int rows_per = 128 * D / kThreads;  // rows per thread: D threads per row
      const int part = tid / D;
      const float m = kmean_s[d];
      float t4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int i = 0; i < rows_per; ++i) {
        const int rr = part * rows_per + i;
        const float x = rr < video_rows ? __bfloat162float(stage_elem<D>(ktile, rr, d)) - m : 0.f;
        t4[i & 3] = fmaf(x, x, t4[i & 3]);
      }
      tr = (t4[0] + t4[1]) + (t4[2] + t4[3]);
    }
    for (int o = 16; o > 0; o >>= 1) tr += __shfl_xor_sync(0xffffffffu, tr, o);
    __syncthreads();  // red (the pooling scratch) is free for the trace partial sums
    if ((tid & 31) == 0) red[tid >> 5] = tr;
    // combine the two halves of rot
    if (tid < 128) {
#pragma unroll
      for (int c = 0; c < kMaxRank; ++c) rot[tid * kMaxRank + c] += rot[(128 + tid) * kMaxRank + c];
    }
    __syncthreads();
    if ((tid >> 5) < rank) {
      // two-pass population variance of column c of K U, one warp per column
      const int c = tid >> 5;
      const int lane = tid & 31;
      float sum = 0.f;
      for (int r = lane; r < video_rows; r += 32) sum += rot[r * kMaxRank + c];
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float m = sum / static_cast<float>(video_rows);
      float ss = 0.f;
      for (int r = lane; r < video_rows; r += 32) {
        const float x = rot[r * kMaxRank + c] - m;
        ss = fmaf(x, x, ss);
      }
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) stat[c] = fmaxf(ss / static_cast<float>(video_rows), 0.f);
    }
    __syncthreads();
    if (tid < D) {
      float v;
      if (tid < rank) {
        v = stat[tid];
      } else {
        float total = 0.f;
        for (int q = 0; q < kThreads / 32; ++q) total += red[q];
        total /= static_cast<float>(video_rows);
        float lead = 0.f;
        for (int c = 0; c < rank; ++c) lead += stat[c];
        v = fmaxf(total - lead, 0.f) / static_cast<float>(D - rank);
      }
      a.variance[(static_cast<size_t>(bank) * a.nB + blk) * D + tid] = v;
      if (a.variance_bf16)
        a.variance_bf16[(static_cast<size_t>(bank) * a.nB_pad + blk) * D + tid] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace

int launch_gather(const GatherArgs& a, cudaStream_t s) {
  if (a.S_pad % 128 || a.S > a.S_pad || a.n_video > a.S || a.n_video <= 0) return kErrShape;
  if (a.variance != nullptr && (a.basis == nullptr || a.rank <= 0 || a.rank >= a.D || a.rank > kMaxRank))
    return kErrShape;
  dim3 grid(a.S_pad / 128, a.batch * a.heads);
  if (a.D == 128) {
    const int smem = GatherSmem<128>::kTotal;
    cudaFuncSetAttribute(gather_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    gather_kernel<128><<<grid, kThreads, smem, s>>>(a);
  } else if (a.D == 64) {
    const int smem = GatherSmem<64>::kTotal;
    cudaFuncSetAttribute(gather_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    gather_kernel<64><<<grid, kThreads, smem, s>>>(a);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int gather_max_rank() { return kMaxRank; }

}  // namespace recap
