// Moment statistics of the coarse tail (recap/sparse/closure.py, recap/kernels/closure_stats.py).
//
// moments_kernel   pooled within-block key scatter  sum_t (k_t - kbar_b)(k_t - kbar_b)^T / N
//                  (pooled_within_block_scatter, recap/sparse/closure.py:42-73) and the pooled
//                  value-key covariance  sum_t v_t (k_t - kbar_b)^T / N
//                  (_batched_centered_cross_fp32_kernel, recap/kernels/closure_stats.py:27-94,
//                  246-290), over the video tokens, in fp32.  Each CTA accumulates a D x D tile
//                  over a chunk of blocks; a second kernel adds the chunks in a fixed order.
// variance_kernel  per-block population variance of K U, two-pass, clamped at 0
//                  (_rotated_leaf_variance_kernel, recap/kernels/closure_stats.py:96-189, 242),
//                  then fold_rank (recap/sparse/closure.py:96-104) in the epilogue.
// basis_prep       U^T in bf16, the K-major B operand of Q U in the coarse-tail kernel.
#include "kernels.h"

namespace recap {
namespace {

constexpr int kChunkBlocks = 32;  // 128-token blocks per moments CTA
constexpr int kTok = 32;          // tokens staged per step

template <int D>
__global__ void __launch_bounds__(256) moments_kernel(const ClosureArgs a, float* ws_scatter,
                                                       float* ws_cross, int nchunks) {
  constexpr int TI = D / 16;  // output rows per thread
  constexpr int TJ = D / 16;  // output cols per thread
  __shared__ __align__(16) float kc[kTok][D];
  __shared__ float vT[D][kTok + 1];
  const int chunk = blockIdx.x;
  const int bank = blockIdx.y;
  const int tid = threadIdx.x;
  const int i0 = (tid / 16) * TI;
  const int j0 = (tid % 16) * TJ;
  const bool do_scatter = ws_scatter != nullptr;
  const bool do_cross = ws_cross != nullptr;
  float acc_s[TI][TJ];
  float acc_c[TI][TJ];
#pragma unroll
  for (int x = 0; x < TI; ++x)
#pragma unroll
    for (int y = 0; y < TJ; ++y) acc_s[x][y] = acc_c[x][y] = 0.f;

  const int t_begin = chunk * kChunkBlocks * 128;
  const int t_end = min(t_begin + kChunkBlocks * 128, a.n_video);
  const __nv_bfloat16* kb = a.kr + static_cast<size_t>(bank) * a.S_pad * D;
  const __nv_bfloat16* vb = a.vt + static_cast<size_t>(bank) * D * a.S_pad;
  const float* mb = a.kmean + static_cast<size_t>(bank) * a.nB * D;
  for (int t0 = t_begin; t0 < t_end; t0 += kTok) {
    __syncthreads();
    for (int idx = tid; idx < kTok * D; idx += 256) {
      const int tt = idx / D;
      const int d = idx % D;
      const int t = t0 + tt;
      float v = 0.f;
      if (t < t_end) v = __bfloat162float(kb[static_cast<size_t>(t) * D + d]) - mb[(t >> 7) * D + d];
      kc[tt][d] = v;
    }
    if (do_cross) {
      for (int idx = tid; idx < kTok * D; idx += 256) {
        const int d = idx / kTok;
        const int tt = idx % kTok;
        const int t = t0 + tt;
        vT[d][tt] = t < t_end ? __bfloat162float(vb[static_cast<size_t>(d) * a.S_pad + t]) : 0.f;
      }
    }
    __syncthreads();
#pragma unroll 2
    for (int tt = 0; tt < kTok; ++tt) {
      float bv[TJ];
#pragma unroll
      for (int y = 0; y < TJ; y += 4) {
        const float4 q = *reinterpret_cast<const float4*>(&kc[tt][j0 + y]);
        bv[y] = q.x;
        bv[y + 1] = q.y;
        bv[y + 2] = q.z;
        bv[y + 3] = q.w;
      }
      if (do_scatter) {
#pragma unroll
        for (int x = 0; x < TI; ++x) {
          const float av = kc[tt][i0 + x];
#pragma unroll
          for (int y = 0; y < TJ; ++y) acc_s[x][y] = fmaf(av, bv[y], acc_s[x][y]);
        }
      }
      if (do_cross) {
#pragma unroll
        for (int x = 0; x < TI; ++x) {
          const float av = vT[i0 + x][tt];
#pragma unroll
          for (int y = 0; y < TJ; ++y) acc_c[x][y] = fmaf(av, bv[y], acc_c[x][y]);
        }
      }
    }
  }
  const size_t base = (static_cast<size_t>(bank) * nchunks + chunk) * D * D;
#pragma unroll
  for (int x = 0; x < TI; ++x)
#pragma unroll
    for (int y = 0; y < TJ; ++y) {
      if (do_scatter) ws_scatter[base + (i0 + x) * D + j0 + y] = acc_s[x][y];
      if (do_cross) ws_cross[base + (i0 + x) * D + j0 + y] = acc_c[x][y];
    }
}

__global__ void moments_reduce_kernel(const float* ws, int nchunks, int D, float inv_n, float* out,
                                      __nv_bfloat16* out_bf16) {
  const int bank = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= D * D) return;
  float s = 0.f;
  for (int c = 0; c < nchunks; ++c) s += ws[(static_cast<size_t>(bank) * nchunks + c) * D * D + e];
  const float v = s * inv_n;
  out[static_cast<size_t>(bank) * D * D + e] = v;
  if (out_bf16) out_bf16[static_cast<size_t>(bank) * D * D + e] = __float2bfloat16_rn(v);
}

template <int D>
__global__ void __launch_bounds__(256) variance_kernel(const ClosureArgs a) {
  constexpr int TR = 8;       // rows per thread (128 rows / 16)
  constexpr int TC = D / 16;  // cols per thread
  constexpr int KS = D + 1;   // padded key row
  extern __shared__ __align__(16) float sm[];
  float* kblk = sm;                // [128][D+1]
  float* ub = kblk + 128 * KS;     // [D][D]
  float* red = ub + D * D;         // [16][D]
  float* var = red + 16 * D;       // [D]
  const int blk = blockIdx.x;
  const int bank = blockIdx.y;
  const int tid = threadIdx.x;
  const int r0 = (tid / 16) * TR;
  const int c0 = (tid % 16) * TC;
  const int count = min(128, a.n_video - blk * 128);
  const __nv_bfloat16* kb = a.kr + (static_cast<size_t>(bank) * a.S_pad + blk * 128) * D;
  for (int idx = tid; idx < 128 * D; idx += 256) {
    const int r = idx / D, d = idx % D;
    kblk[r * KS + d] = r < count ? __bfloat162float(kb[static_cast<size_t>(r) * D + d]) : 0.f;
  }
  const float* U = a.basis + static_cast<size_t>(bank) * D * D;
  for (int idx = tid; idx < D * D; idx += 256) ub[idx] = U[idx];
  __syncthreads();
  float acc[TR][TC];
#pragma unroll
  for (int x = 0; x < TR; ++x)
#pragma unroll
    for (int y = 0; y < TC; ++y) acc[x][y] = 0.f;
#pragma unroll 4
  for (int k = 0; k < D; ++k) {
    float uv[TC];
#pragma unroll
    for (int y = 0; y < TC; ++y) uv[y] = ub[k * D + c0 + y];
#pragma unroll
    for (int x = 0; x < TR; ++x) {
      const float kv = kblk[(r0 + x) * KS + k];
#pragma unroll
      for (int y = 0; y < TC; ++y) acc[x][y] = fmaf(kv, uv[y], acc[x][y]);
    }
  }
  // pass 1: column means over the valid rows
  const int g = tid / 16;
#pragma unroll
  for (int y = 0; y < TC; ++y) {
    float s = 0.f;
#pragma unroll
    for (int x = 0; x < TR; ++x)
      if (r0 + x < count) s += acc[x][y];
    red[g * D + c0 + y] = s;
  }
  __syncthreads();
  if (tid < D) {
    float s = 0.f;
    for (int q = 0; q < 16; ++q) s += red[q * D + tid];
    var[tid] = s / static_cast<float>(count);  // mean for now
  }
  __syncthreads();
  // pass 2: squared deviations
#pragma unroll
  for (int y = 0; y < TC; ++y) {
    const float m = var[c0 + y];
    float s = 0.f;
#pragma unroll
    for (int x = 0; x < TR; ++x)
      if (r0 + x < count) {
        const float dv = acc[x][y] - m;
        s = fmaf(dv, dv, s);
      }
    red[g * D + c0 + y] = s;
  }
  __syncthreads();
  if (tid < D) {
    float s = 0.f;
    for (int q = 0; q < 16; ++q) s += red[q * D + tid];
    var[tid] = fmaxf(s / static_cast<float>(count), 0.f);
  }
  __syncthreads();
  if (tid < D) {
    float v = var[tid];
    const int rank = a.rank;
    if (rank > 0 && rank < D && tid >= rank) {
      float s = 0.f;
      for (int c = rank; c < D; ++c) s += var[c];
      v = s / static_cast<float>(D - rank);
    }
    a.variance[(static_cast<size_t>(bank) * a.nB + blk) * D + tid] = v;
    if (a.variance_bf16)
      a.variance_bf16[(static_cast<size_t>(bank) * a.nB_pad + blk) * D + tid] = __float2bfloat16_rn(v);
  }
}

__global__ void basis_prep_kernel(const BasisPrepArgs a) {
  const int bank = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= a.D * a.D) return;
  const int n = e / a.D, k = e % a.D;
  a.basis_t[static_cast<size_t>(bank) * a.D * a.D + e] =
      __float2bfloat16_rn(a.basis[static_cast<size_t>(bank) * a.D * a.D + k * a.D + n]);
}

int n_chunks(int nB) { return (nB + kChunkBlocks - 1) / kChunkBlocks; }

}  // namespace

int64_t closure_workspace_floats(int banks, int D, int nB) {
  return 2LL * banks * n_chunks(nB) * D * D;
}

int launch_closure_moments(const ClosureArgs& a, cudaStream_t s) {
  if (a.scatter == nullptr && a.cvk == nullptr) return kOk;
  const int nch = n_chunks(a.nB);
  float* ws_s = a.scatter ? a.workspace : nullptr;
  float* ws_c = a.cvk ? a.workspace + static_cast<int64_t>(a.banks) * nch * a.D * a.D : nullptr;
  dim3 grid(nch, a.banks);
  if (a.D == 128)
    moments_kernel<128><<<grid, 256, 0, s>>>(a, ws_s, ws_c, nch);
  else if (a.D == 64)
    moments_kernel<64><<<grid, 256, 0, s>>>(a, ws_s, ws_c, nch);
  else
    return kErrShape;
  if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
  const float inv_n = 1.f / static_cast<float>(a.n_video);
  dim3 rgrid((a.D * a.D + 255) / 256, a.banks);
  if (ws_s) moments_reduce_kernel<<<rgrid, 256, 0, s>>>(ws_s, nch, a.D, inv_n, a.scatter, nullptr);
  if (ws_c) moments_reduce_kernel<<<rgrid, 256, 0, s>>>(ws_c, nch, a.D, inv_n, a.cvk, a.cvk_bf16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_closure_variance(const ClosureArgs& a, cudaStream_t s) {
  dim3 grid(a.nB, a.banks);
  if (a.D == 128) {
    const int smem = (128 * 129 + 128 * 128 + 16 * 128 + 128) * 4;
    cudaFuncSetAttribute(variance_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    variance_kernel<128><<<grid, 256, smem, s>>>(a);
  } else if (a.D == 64) {
    const int smem = (128 * 65 + 64 * 64 + 16 * 64 + 64) * 4;
    cudaFuncSetAttribute(variance_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    variance_kernel<64><<<grid, 256, smem, s>>>(a);
  } else {
    return kErrShape;
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_moments_reduce(const float* ws, int banks, int nchunks, int D, float inv_n, float* out,
                          __nv_bfloat16* out_bf16, cudaStream_t s) {
  dim3 rgrid((D * D + 255) / 256, banks);
  moments_reduce_kernel<<<rgrid, 256, 0, s>>>(ws, nchunks, D, inv_n, out, out_bf16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_basis_prep(const BasisPrepArgs& a, cudaStream_t s) {
  dim3 grid((a.D * a.D + 255) / 256, a.banks);
  basis_prep_kernel<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
