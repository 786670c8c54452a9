// Refinement write at a dense refresh (_refresh_detail_kernel and refresh_detail,
// recap/kernels/detail_cache.py:26-186, 304-379).
//
// For every cached video row r (< rows), with native row n = video_offset + perm[r]:
//   ratio = min(exp(min(lh - lf_n, 0)), 1 - 1e-6),  den = 1 - ratio
//   det   = clamp((of_n - ratio oh) / den - go, +-6e4), zero where ratio > 1 - 1e-3  (fp16)
//   dl    = clamp(lf_n + ln den - gl, +-30)
// When validating, the sparse output the old refinement would have produced (the merge of
// recap/kernels/detail_cache.py:267-292, with the drift weight when a reference coarse LSE is
// given) is compared with the dense output first: sum (old - of)^2 and sum of^2.  The reference
// adds those with fp32 atomics; here every CTA writes its two partial sums and one more kernel
// adds them in a fixed order, so the result is deterministic.
#include <mutex>

#include "kernels.h"

namespace recap {
namespace {

constexpr int kRowsPerCta = 32;

template <int D>
__global__ void __launch_bounds__(256) refresh_kernel(const RefreshArgs a) {
  constexpr int CPR = D / 8;           // 8-column chunks per row
  constexpr int RPP = 256 / CPR;       // rows per pass
  __shared__ float red[2][8];
  const int bank = blockIdx.y;
  const int tid = threadIdx.x;
  const int ch = tid % CPR;
  const int rsub = tid / CPR;
  float err2 = 0.f, ref2 = 0.f;
  for (int p = 0; p < kRowsPerCta / RPP; ++p) {
    const int r = blockIdx.x * kRowsPerCta + p * RPP + rsub;
    if (r >= a.rows) continue;
    const int n = a.video_offset + a.perm[r];
    if (n < 0 || n >= a.S) continue;  // a corrupt permutation reads nothing out of bounds
    const size_t srow = static_cast<size_t>(bank) * a.S;
    const size_t vrow = static_cast<size_t>(bank) * a.rows + r;
    const float lf = a.full_lse[srow + n];
    const float lh = a.head_lse[srow + r];
    float ratio = expf(fminf(lh - lf, 0.f));
    ratio = fminf(ratio, 1.f - 1.0e-6f);
    const float den = 1.f - ratio;
    const float gl = a.gl[vrow];
    float of[8], oh[8], go[8];
    {
      const uint4 w0 = *reinterpret_cast<const uint4*>(a.full_o + (srow + n) * D + ch * 8);
      const uint4 w1 = *reinterpret_cast<const uint4*>(a.head_o + (srow + r) * D + ch * 8);
      const uint4 w2 = *reinterpret_cast<const uint4*>(a.go + vrow * D + ch * 8);
      const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&w0);
      const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&w1);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w2);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f0 = __bfloat1622float2(h0[e]);
        const float2 f1 = __bfloat1622float2(h1[e]);
        const float2 f2 = __bfloat1622float2(h2[e]);
        of[2 * e] = f0.x; of[2 * e + 1] = f0.y;
        oh[2 * e] = f1.x; oh[2 * e + 1] = f1.y;
        go[2 * e] = f2.x; go[2 * e + 1] = f2.y;
      }
    }
    __half* det_ptr = a.det + vrow * D + ch * 8;
    if (a.validate) {
      float od[8];
      const uint4 wd = *reinterpret_cast<const uint4*>(det_ptr);
      const __half2* hd = reinterpret_cast<const __half2*>(&wd);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(hd[e]);
        od[2 * e] = f.x;
        od[2 * e + 1] = f.y;
      }
      const float old_dl = a.dl[vrow];
      float tail_o_ms = 0.f, tail_o_mc = 1.f, inv_td = 1.f, old_tail_l;
      if (a.ogl != nullptr) {
        const float admit = expf(-fabsf(gl - a.ogl[vrow] - a.center[bank]));
        const float cl = gl + old_dl;
        const float tc = fmaxf(gl, cl);
        tail_o_ms = (1.f - admit) * expf(gl - tc);
        tail_o_mc = admit * expf(cl - tc);
        const float td = fmaxf(tail_o_ms + tail_o_mc, 1.0e-30f);
        inv_td = 1.f / td;
        old_tail_l = tc + logf(td);
      } else {
        old_tail_l = gl + old_dl;
      }
      const float common = fmaxf(lh, old_tail_l);
      const float wh = expf(lh - common);
      const float wt = expf(old_tail_l - common);
      const float inv_den = 1.f / fmaxf(wh + wt, 1.0e-30f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float tail_o;
        if (a.ogl != nullptr)
          tail_o = (go[e] * tail_o_ms + (go[e] + od[e]) * tail_o_mc) * inv_td;
        else
          tail_o = go[e] + od[e];
        const float old_sparse = (oh[e] * wh + tail_o * wt) * inv_den;
        const float dv = old_sparse - of[e];
        err2 = fmaf(dv, dv, err2);
        ref2 = fmaf(of[e], of[e], ref2);
      }
    }
    const bool zero = ratio > 1.f - 1.0e-3f;
    const float inv = 1.f / den;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float c0 = (of[2 * e] - ratio * oh[2 * e]) * inv - go[2 * e];
      float c1 = (of[2 * e + 1] - ratio * oh[2 * e + 1]) * inv - go[2 * e + 1];
      c0 = fmaxf(fminf(c0, 6.0e4f), -6.0e4f);
      c1 = fmaxf(fminf(c1, 6.0e4f), -6.0e4f);
      if (zero) c0 = c1 = 0.f;
      __half2 hv = __floats2half2_rn(c0, c1);
      w[e] = *reinterpret_cast<uint32_t*>(&hv);
    }
    *reinterpret_cast<uint4*>(det_ptr) = make_uint4(w[0], w[1], w[2], w[3]);
    if (ch == 0) {
      float dl = lf + logf(den) - gl;
      a.dl[vrow] = fmaxf(fminf(dl, 30.f), -30.f);
    }
  }
  if (a.validate) {
    for (int o = 16; o > 0; o >>= 1) {
      err2 += __shfl_xor_sync(0xffffffffu, err2, o);
      ref2 += __shfl_xor_sync(0xffffffffu, ref2, o);
    }
    if ((tid & 31) == 0) {
      red[0][tid >> 5] = err2;
      red[1][tid >> 5] = ref2;
    }
    __syncthreads();
    if (tid == 0) {
      float e = 0.f, f = 0.f;
      for (int q = 0; q < 8; ++q) {
        e += red[0][q];
        f += red[1][q];
      }
      const size_t cta = static_cast<size_t>(bank) * gridDim.x + blockIdx.x;
      a.partials[2 * cta] = e;
      a.partials[2 * cta + 1] = f;
    }
  }
}

__global__ void stats_kernel(const float* partials, int n, float* stats) {
  __shared__ float red[2][32];
  const int tid = threadIdx.x;
  float e = 0.f, f = 0.f;
  for (int i = tid; i < n; i += 1024) {
    e += partials[2 * i];
    f += partials[2 * i + 1];
  }
  for (int o = 16; o > 0; o >>= 1) {
    e += __shfl_xor_sync(0xffffffffu, e, o);
    f += __shfl_xor_sync(0xffffffffu, f, o);
  }
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = e;
    red[1][tid >> 5] = f;
  }
  __syncthreads();
  if (tid < 32) {
    e = red[0][tid];
    f = red[1][tid];
    for (int o = 16; o > 0; o >>= 1) {
      e += __shfl_xor_sync(0xffffffffu, e, o);
      f += __shfl_xor_sync(0xffffffffu, f, o);
    }
    if (tid == 0) {
      stats[0] = e;
      stats[1] = f;
    }
  }
}

}  // namespace

int refresh_partials_count(int banks, int rows) {
  return banks * ((rows + kRowsPerCta - 1) / kRowsPerCta);
}

int launch_refresh(const RefreshArgs& a, cudaStream_t s) {
  if (a.rows <= 0) {
    if (a.validate && a.stats) return cudaMemsetAsync(a.stats, 0, 2 * sizeof(float), s) == cudaSuccess ? kOk : kErrLaunch;
    return kOk;
  }
  dim3 grid((a.rows + kRowsPerCta - 1) / kRowsPerCta, a.banks);
  if (a.D == 128)
    refresh_kernel<128><<<grid, 256, 0, s>>>(a);
  else if (a.D == 64)
    refresh_kernel<64><<<grid, 256, 0, s>>>(a);
  else
    return kErrShape;
  if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
  if (a.validate) {
    stats_kernel<<<1, 1024, 0, s>>>(a.partials, refresh_partials_count(a.banks, a.rows), a.stats);
    if (cudaGetLastError() != cudaSuccess) return kErrLaunch;
  }
  return kOk;
}


// ---------------------------------------------------------------------------------------
// Variant for callers that may not allocate device memory.
//
// Some hosts hand a plugin only the buffers they planned themselves and forbid it any
// device allocation of its own (serving runtimes with a fixed memory plan, custom-op
// interfaces that pass in every buffer), and cudaMalloc also synchronises the device,
// which a step loop cannot afford.  recap_refresh_detail needs one scratch buffer, the
// per-CTA validation partial sums; this variant keeps them in the file-scope device
// array below instead of a caller buffer.  Its size is fixed: at most
// kNoAllocMaxPairs (bank, 32-row) chunks, i.e. banks * ceil(rows / 32) <= 131072, which
// covers a 24-head HunyuanVideo-720p layer (89088 chunks).  Every GPU that loads the
// library holds the array (1 MiB) until the process exits.
constexpr int kNoAllocMaxPairs = 131072;
static __device__ __align__(256) float g_refresh_scratch[2 * kNoAllocMaxPairs];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
float* g_scratch_ptr[kMaxDevices] = {};
}  // namespace

// Device address of the scratch array on the current device, looked up once per device
// (the host-side symbol is not a device address).  Returns nullptr on failure.
static float* refresh_scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_refresh_scratch) != cudaSuccess) return nullptr;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

int launch_refresh_noalloc(RefreshArgs a, cudaStream_t s) {
  if (a.validate) {
    if (refresh_partials_count(a.banks, a.rows) > kNoAllocMaxPairs) return kErrScratchLimit;
    float* scratch = refresh_scratch_for_current_device();
    if (scratch == nullptr) return kErrLaunch;
    // every CTA writes its own pair before the sum reads it: nothing needs clearing
    a.partials = scratch;
  }
  return launch_refresh(a, s);
}

}  // namespace recap
