// The sequence-to-head exchange of a sequence-parallel (Ulysses) layer as one kernel of
// peer stores: rank p's projections of its tokens, [s, 3, H, D] bf16, go to the receive
// buffer of the rank that owns each head group, [S, 3, H/P, D] at rows p s .. p s + s - 1.
// Over NVLink a store is a posted write, so the kernel streams at the link's write rate
// where remote loads (the gather reading other ranks' shards) wait on every round trip.
// The caller orders the ranks around it: the receive buffers are free (their owners' layout
// passes of the previous layer are done) before, and every rank's stores are complete
// (a collective on the stream) before any owner reads.
#include "kernels.h"

namespace recap {
namespace {

__global__ void __launch_bounds__(256) push_kernel(const PushArgs a) {
  // one thread per 16-byte chunk of the local [s, 3, H D] rows, in row order: consecutive
  // threads read consecutive chunks and write consecutive chunks of one destination row
  const int64_t chunks_per_row = static_cast<int64_t>(a.heads) * a.D / 8;  // per (token, tensor)
  const int64_t total = static_cast<int64_t>(a.tokens) * 3 * chunks_per_row;
  const int64_t group_chunks = static_cast<int64_t>(a.heads_per_rank) * a.D / 8;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = c / chunks_per_row;  // token * 3 + tensor
    const int64_t col = c - row * chunks_per_row;
    const int q = static_cast<int>(col / group_chunks);
    const int64_t in_group = col - static_cast<int64_t>(q) * group_chunks;
    const int64_t token = row / 3;
    const int64_t t = row - token * 3;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.src) + c);
    __nv_bfloat16* base = a.dst[0];  // selected without indexing the parameter array (no local copy)
#pragma unroll
    for (int r = 1; r < kMaxRanks; ++r)
      if (q == r) base = a.dst[r];
    uint4* dst = reinterpret_cast<uint4*>(base) + ((a.token0 + token) * 3 + t) * group_chunks + in_group;
    *dst = v;
  }
  __threadfence_system();  // the stores are visible beyond this GPU before the kernel ends
}

// Rows of a locally computed [banks, S, D] output into the token shards of the ranks that
// own them (bank b, token n -> dst[q] + b bank_stride + (n - q tokens_per_rank) row_stride).
__global__ void __launch_bounds__(256) scatter_kernel(const ScatterArgs a) {
  const int64_t cpr = a.D / 8;  // 16-byte chunks per row
  const int64_t total = static_cast<int64_t>(a.banks) * a.S * cpr;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = c / cpr;  // bank * S + token
    const int64_t j = c - row * cpr;
    const int64_t bank = row / a.S;
    const int64_t n = row - bank * a.S;
    const int q = static_cast<int>(n / a.tokens_per_rank);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.src) + c);
    __nv_bfloat16* base = a.dst[0];
#pragma unroll
    for (int r = 1; r < kMaxRanks; ++r)
      if (q == r) base = a.dst[r];
    *reinterpret_cast<uint4*>(base + bank * a.bank_stride + (n - static_cast<int64_t>(q) * a.tokens_per_rank) * a.row_stride +
                              j * 8) = v;
  }
  __threadfence_system();
}

}  // namespace

int launch_scatter(const ScatterArgs& a, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(a.banks) * a.S * (a.D / 8);
  if (total <= 0) return kOk;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256;
  const int grid = static_cast<int>(want < 8LL * sms ? want : 8LL * sms);
  scatter_kernel<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_push(const PushArgs& a, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(a.tokens) * 3 * a.heads * a.D / 8;
  if (total <= 0) return kOk;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256;
  const int grid = static_cast<int>(want < 8LL * sms ? want : 8LL * sms);
  push_kernel<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
