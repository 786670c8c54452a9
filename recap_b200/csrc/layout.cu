// Layout gather fused with block pooling.
//
// One pass over the native-order Q, K and V of a layer call:
//  * reorders the tokens into [Hilbert-ordered video | text] (Layout.reorder,
//    recap/sparse/layout.py:86-90), writing Q and K as [banks, S_pad, D] and V
//    transposed as [banks, D, S_pad] (the K-major operand layout of P V);
//  * sums each 128-token block over its video tokens in fp32 and divides by the
//    block's token count (pool_blocks, recap/sparse/pooling.py:10-34), writing
//    the fp32 means and the bf16 copies the coarse tail reads.
// Rows past S (up to S_pad) are written as zeros.  HBM-bound: every input byte
// is read once and every output byte written once.
#include "kernels.h"

namespace recap {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void add8(float (&acc)[8], const uint4& w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(h[e]);
    acc[2 * e] += f.x;
    acc[2 * e + 1] += f.y;
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads) gather_kernel(const GatherArgs a) {
  constexpr int CPR = D / 8;              // 16-byte chunks per row
  constexpr int RPP = kThreads / CPR;     // rows per pass
  constexpr int PASSES = 128 / RPP;
  constexpr int VSTRIDE = D + 8;          // padded row of the staged V tile
  __shared__ __align__(16) __nv_bfloat16 vtile[128 * VSTRIDE];
  __shared__ float red[RPP * D];

  const int blk = blockIdx.x;
  const int bank = blockIdx.y;
  const int bi = bank / a.heads;
  const int hi = bank - bi * a.heads;
  const int tid = threadIdx.x;
  const int ch = tid % CPR;
  const int rsub = tid / CPR;
  const int row0 = blk * 128;
  const int video_rows = min(128, a.n_video - row0);  // <= 0 for text-only blocks

  for (int t = 0; t < 3; ++t) {
    const __nv_bfloat16* src = a.src[t];
    if (src == nullptr) continue;
    const __nv_bfloat16* base = src + bi * a.stride_b[t] + hi * a.stride_h[t];
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 4
    for (int p = 0; p < PASSES; ++p) {
      const int rl = p * RPP + rsub;
      const int r = row0 + rl;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (r < a.S) {
        const int64_t native = a.src_row[r];
        if (native >= 0 && native < a.S)  // a corrupt index reads nothing out of bounds
          val = *reinterpret_cast<const uint4*>(base + native * a.stride_s[t] + ch * 8);
      }
      if (t == 0 && a.qr) {
        *reinterpret_cast<uint4*>(a.qr + (static_cast<size_t>(bank) * a.S_pad + r) * D + ch * 8) = val;
      } else if (t == 1 && a.kr) {
        *reinterpret_cast<uint4*>(a.kr + (static_cast<size_t>(bank) * a.S_pad + r) * D + ch * 8) = val;
      } else if (t == 2) {
        *reinterpret_cast<uint4*>(vtile + rl * VSTRIDE + ch * 8) = val;
      }
      if (rl < video_rows) add8(acc, val);
    }
    if (a.mean[t] != nullptr && blk < a.nB) {
#pragma unroll
      for (int e = 0; e < 8; ++e) red[rsub * D + ch * 8 + e] = acc[e];
      __syncthreads();
      if (tid < D) {
        float s = 0.f;
#pragma unroll 4
        for (int g = 0; g < RPP; ++g) s += red[g * D + tid];
        const float m = s / static_cast<float>(video_rows);
        a.mean[t][(static_cast<size_t>(bank) * a.nB + blk) * D + tid] = m;
        if (t == 1 && a.kmean_bf16)
          a.kmean_bf16[(static_cast<size_t>(bank) * a.nB_pad + blk) * D + tid] = __float2bfloat16_rn(m);
        if (t == 2 && a.vmean_t_bf16)
          a.vmean_t_bf16[(static_cast<size_t>(bank) * D + tid) * a.nB_pad + blk] = __float2bfloat16_rn(m);
      }
      __syncthreads();
    }
  }
  if (a.vt != nullptr && a.src[2] != nullptr) {
    __syncthreads();
    // transposed write: lanes run over d so that the staged reads are conflict-free
    for (int idx = tid; idx < D * 16; idx += kThreads) {
      const int d = idx % D;
      const int kc = idx / D;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 lo = vtile[(kc * 8 + 2 * e) * VSTRIDE + d];
        const __nv_bfloat16 hi = vtile[(kc * 8 + 2 * e + 1) * VSTRIDE + d];
        w[e] = static_cast<uint32_t>(__bfloat16_as_ushort(lo)) |
               (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
      }
      *reinterpret_cast<uint4*>(a.vt + (static_cast<size_t>(bank) * D + d) * a.S_pad + row0 + kc * 8) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

}  // namespace

int launch_gather(const GatherArgs& a, cudaStream_t s) {
  if (a.S_pad % 128 || a.S > a.S_pad || a.n_video > a.S || a.n_video <= 0) return kErrShape;
  dim3 grid(a.S_pad / 128, a.batch * a.heads);
  if (a.D == 128)
    gather_kernel<128><<<grid, kThreads, 0, s>>>(a);
  else if (a.D == 64)
    gather_kernel<64><<<grid, kThreads, 0, s>>>(a);
  else
    return kErrShape;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
