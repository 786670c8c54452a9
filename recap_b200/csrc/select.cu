// Block selection and the small mask kernels around it.
//
// select_kernel   block_proxy_mask + head_partition (recap/sparse/router.py:10-23,
//                 recap/sparse/attention.py:74-94): score = (qbar . kbar) * s in fp32,
//                 top-`keep` key blocks per query block, then a trailing partial video
//                 block is selected in full as a row and as a column.  The k-th largest
//                 score is found by an exact radix select on the order-preserving integer
//                 image of the fp32 scores; among scores equal to it, lower block indices
//                 win (torch.topk leaves that order unspecified).
// overlap_kernel  |new & old| and |new| of two partitions (recap/operator.py:288-291, 425-428).
// mask_kernel     build_kernel_block_mask (recap/kernels/block_sparse.py:52-75).
// center_kernel   _drift_center (recap/operator.py:148-150) from per-query-block partial sums.
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

constexpr int kRows = 16;        // query blocks per CTA (one warp each in the top-k phase)
constexpr int kSelThreads = 512;
constexpr int kDc = 8;           // dimensions of every key mean staged per step
constexpr int kPitch = kDc + 1;  // odd row pitch: lane l reads word 9 l + dd, no bank conflicts

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Scores: each thread holds KPT key blocks x the CTA's 16 query blocks in registers.  The key
// means go through shared memory 8 dimensions at a time (32-byte row segments, whole sectors;
// a lane per key row reading its own 512-byte row had touched 32 lines per load), by
// asynchronous copies into two buffers, so one chunk is in flight while the other is used.
// Every score is still one fmaf chain over d = 0 .. D-1: the order of the fp32 sums is that
// of the plain dot product.
template <int D, int KPT>
__global__ void __launch_bounds__(kSelThreads, KPT <= 2 ? 2 : 1) select_kernel(const SelectArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nB = a.nB;
  float* qt = reinterpret_cast<float*>(smem);                    // [D][kRows]: q means, transposed
  uint32_t* hist = reinterpret_cast<uint32_t*>(qt + D * kRows);  // [kRows warps][256]
  float* kc = reinterpret_cast<float*>(hist + kRows * 256);      // 2 x [nB][kPitch] while scoring
  uint32_t* keys = reinterpret_cast<uint32_t*>(kc);              // [kRows][nB] afterwards
  const int bank = blockIdx.y;
  const int i0 = blockIdx.x * kRows;
  const int tid = threadIdx.x;
  for (int idx = tid; idx < kRows * D; idx += kSelThreads) {
    const int r = idx / D;
    const int d = idx - r * D;
    const int i = i0 + r;
    qt[d * kRows + r] = i < nB ? a.qmean[(static_cast<size_t>(bank) * nB + i) * D + d] : 0.f;
  }
  float acc[KPT][kRows];
#pragma unroll
  for (int m = 0; m < KPT; ++m)
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[m][r] = 0.f;
  const float* kbase = a.kmean + static_cast<size_t>(bank) * nB * D;
  const uint32_t kc_u32 = static_cast<uint32_t>(__cvta_generic_to_shared(kc));
  const int buf_words = nB * kPitch;
  auto stage = [&](int chunk) {  // dimensions 8 chunk .. 8 chunk + 7 of every key mean
    const uint32_t dst0 = kc_u32 + static_cast<uint32_t>((chunk & 1) * buf_words) * 4u;
    for (int idx = tid; idx < nB * kDc; idx += kSelThreads) {
      const int j = idx / kDc;
      const int e = idx - j * kDc;
      cp_async4(dst0 + static_cast<uint32_t>(j * kPitch + e) * 4u, kbase + static_cast<size_t>(j) * D + chunk * kDc + e);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  constexpr int kChunks = D / kDc;
  stage(0);
  for (int c = 0; c < kChunks; ++c) {
    if (c + 1 < kChunks) {
      stage(c + 1);  // its buffer was last read in step c - 1, which ended at a barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // chunk c has landed for every thread (and, the first time, qt is written)
    const float* kb = kc + (c & 1) * buf_words;
#pragma unroll 1
    for (int dd = 0; dd < kDc; ++dd) {
      float kv[KPT];
#pragma unroll
      for (int m = 0; m < KPT; ++m) {
        const int j = tid + m * kSelThreads;
        kv[m] = j < nB ? kb[j * kPitch + dd] : 0.f;
      }
      const float4* q4 = reinterpret_cast<const float4*>(qt + (c * kDc + dd) * kRows);
#pragma unroll
      for (int r4 = 0; r4 < kRows / 4; ++r4) {
        const float4 q = q4[r4];
#pragma unroll
        for (int m = 0; m < KPT; ++m) {  // two rows per packed fma (each lane an fp32 fma, same bits)
          fma2(acc[m][4 * r4 + 0], acc[m][4 * r4 + 1], q.x, q.y, kv[m], kv[m], acc[m][4 * r4 + 0],
               acc[m][4 * r4 + 1]);
          fma2(acc[m][4 * r4 + 2], acc[m][4 * r4 + 3], q.z, q.w, kv[m], kv[m], acc[m][4 * r4 + 2],
               acc[m][4 * r4 + 3]);
        }
      }
    }
    __syncthreads();  // every thread is done with buffer c & 1 before step c + 1 refills it
  }
  __syncthreads();  // the last chunk is consumed: its space takes the order keys
#pragma unroll
  for (int m = 0; m < KPT; ++m) {
    const int j = tid + m * kSelThreads;
    if (j < nB) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) keys[r * nB + j] = order_key(acc[m][r] * a.scale);
    }
  }
  __syncthreads();

  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int i = i0 + warp;
  if (i >= nB) return;
  const uint32_t* k = keys + warp * nB;
  uint32_t* h = hist + warp * 256;
  const int want = max(1, min(a.keep, nB));
  uint32_t prefix = 0;
  int need = want;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) h[b] = 0;
    __syncwarp();
    const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
    // Scores of one row lie close together, so most keys of a pass share a digit: the lanes
    // with equal digits add their count once (one shared-memory atomic per distinct digit
    // of the warp instead of up to 32 serialised ones on the same bin).
    for (int base = 0; base < nB; base += 32) {
      const int j = base + lane;
      const uint32_t key = j < nB ? k[j] : 0u;
      const bool hit = j < nB && (key & hi_mask) == prefix;
      const uint32_t bin = (key >> shift) & 0xFFu;
      const unsigned peers = __match_any_sync(0xffffffffu, hit ? bin : 0x100u);
      if (hit && lane == __ffs(peers) - 1) atomicAdd(&h[bin], static_cast<uint32_t>(__popc(peers)));
    }
    __syncwarp();
    // lane l owns bins 255-8l .. 248-8l (descending)
    int cnt[8];
    int lane_sum = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      cnt[e] = static_cast<int>(h[255 - 8 * lane - e]);
      lane_sum += cnt[e];
    }
    int incl = lane_sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = incl - lane_sum;
    const unsigned hit = __ballot_sync(0xffffffffu, incl >= need && excl < need);
    const int src = __ffs(hit) - 1;
    int digit = 0, above = 0;
    if (lane == src) {
      int run = excl;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (run + cnt[e] >= need) {
          digit = 255 - 8 * lane - e;
          above = run;
          break;
        }
        run += cnt[e];
      }
    }
    digit = __shfl_sync(0xffffffffu, digit, src);
    above = __shfl_sync(0xffffffffu, above, src);
    need -= above;
    prefix |= static_cast<uint32_t>(digit) << shift;
    __syncwarp();
  }
  // prefix is the key of the want-th largest score; `need` of the scores equal to it
  // are taken, in increasing block order.
  const bool forced = (a.n_video % a.block_size) != 0;
  uint8_t* out = a.partition + (static_cast<size_t>(bank) * nB + i) * nB;
  int taken_eq = 0;
  for (int base = 0; base < nB; base += 32) {
    const int j = base + lane;
    const uint32_t key = j < nB ? k[j] : 0u;
    const bool eq = j < nB && key == prefix;
    const unsigned m = __ballot_sync(0xffffffffu, eq);
    const int rank = taken_eq + __popc(m & ((1u << lane) - 1u));
    taken_eq += __popc(m);
    bool sel = j < nB && (key > prefix || (eq && rank < need));
    if (forced && (i == nB - 1 || j == nB - 1)) sel = true;
    if (j < nB) out[j] = sel ? 1 : 0;
  }
}

__global__ void overlap_kernel(const OverlapArgs a) {
  long long both = 0, total = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; base < a.n;
       base += stride) {
    if (base + 4 <= a.n && ((reinterpret_cast<uintptr_t>(a.a + base) | reinterpret_cast<uintptr_t>(a.b + base)) & 3) == 0) {
      const uint32_t x = *reinterpret_cast<const uint32_t*>(a.a + base);
      const uint32_t y = *reinterpret_cast<const uint32_t*>(a.b + base);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t xb = (x >> (8 * e)) & 0xFFu, yb = (y >> (8 * e)) & 0xFFu;
        total += xb != 0;
        both += (xb != 0) && (yb != 0);
      }
    } else {
      for (int64_t e = base; e < base + 4 && e < a.n; ++e) {
        total += a.a[e] != 0;
        both += (a.a[e] != 0) && (a.b[e] != 0);
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    both += __shfl_down_sync(0xffffffffu, both, o);
    total += __shfl_down_sync(0xffffffffu, total, o);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(a.out), static_cast<unsigned long long>(both));
    atomicAdd(reinterpret_cast<unsigned long long*>(a.out + 1), static_cast<unsigned long long>(total));
  }
}

__global__ void mask_kernel(const KernelMaskArgs a) {
  const int bank = blockIdx.y;
  const int i = blockIdx.x;
  uint8_t* out = a.mask + (static_cast<size_t>(bank) * a.NB + i) * a.NB;
  const uint8_t* p = a.partition + (static_cast<size_t>(bank) * a.nB + i) * a.nB;
  for (int j = threadIdx.x; j < a.NB; j += blockDim.x) {
    bool v;
    if (i >= a.dense_start || j >= a.dense_start)
      v = true;
    else
      v = p[j] != 0;
    out[j] = v ? 1 : 0;
  }
}

__global__ void center_kernel(const CenterArgs a) {
  const int bank = blockIdx.x;
  const int lane = threadIdx.x;
  float s = 0.f;
  for (int i = lane; i < a.nqb; i += 32) s += a.partial[static_cast<size_t>(bank) * a.nqb + i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) a.center[bank] = s / static_cast<float>(a.rows);
}

}  // namespace

template <int D, int KPT>
int launch_select_t(const SelectArgs& a, size_t smem, cudaStream_t s) {
  cudaFuncSetAttribute(select_kernel<D, KPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  dim3 grid((a.nB + kRows - 1) / kRows, a.banks);
  select_kernel<D, KPT><<<grid, kSelThreads, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

template <int D>
int launch_select_d(const SelectArgs& a, size_t smem, cudaStream_t s) {
  if (a.nB <= kSelThreads) return launch_select_t<D, 1>(a, smem, s);
  if (a.nB <= 2 * kSelThreads) return launch_select_t<D, 2>(a, smem, s);
  return launch_select_t<D, 4>(a, smem, s);
}

int launch_select(const SelectArgs& a, cudaStream_t s) {
  if (a.nB <= 0 || a.banks <= 0 || a.nB > 4 * kSelThreads) return kErrShape;
  // q means + histograms + max(two key-mean chunks, order keys)
  const size_t chunk = 2 * static_cast<size_t>(a.nB) * kPitch * 4;
  const size_t keys = static_cast<size_t>(kRows) * a.nB * 4;
  const size_t smem = static_cast<size_t>(a.D) * kRows * 4 + kRows * 256 * 4 + (chunk > keys ? chunk : keys);
  if (smem > 220 * 1024) return kErrShape;
  if (a.D == 128) return launch_select_d<128>(a, smem, s);
  if (a.D == 64) return launch_select_d<64>(a, smem, s);
  return kErrShape;
}

int launch_overlap(const OverlapArgs& a, cudaStream_t s) {
  if (cudaMemsetAsync(a.out, 0, 2 * sizeof(long long), s) != cudaSuccess) return kErrLaunch;
  if (a.n <= 0) return kOk;
  int blocks = static_cast<int>((a.n / 4 + 255) / 256);
  if (blocks > 1184) blocks = 1184;
  if (blocks < 1) blocks = 1;
  overlap_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_kernel_mask(const KernelMaskArgs& a, cudaStream_t s) {
  if (a.NB <= 0 || a.banks <= 0) return kOk;
  dim3 grid(a.NB, a.banks);
  mask_kernel<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_center(const CenterArgs& a, cudaStream_t s) {
  if (a.banks <= 0) return kOk;
  center_kernel<<<a.banks, 32, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
