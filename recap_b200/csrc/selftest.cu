// Device self-checks reachable through the C ABI:
//  * exp2_check_kernel evaluates the FP32-pipe exponential (exp2_poly2) the softmax
//    kernels may use, for comparison with CUDA's exp2 on the same inputs;
//  * wait_selftest_kernel exercises the bounded mbarrier wait every kernel of this
//    library relies on: one thread waits on a barrier that nothing arrives on until its
//    limit runs out, records the timeout in the status word and raises the CTA abort
//    flag; a second waiter, with a longer limit, must leave through the abort flag.
//    Nothing faults, traps or hangs: both waits end by themselves.
#include "common.cuh"
#include "kernels.h"

namespace recap {
namespace {

__global__ void exp2_check_kernel(const float* in, float* out, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float y0 = in[i];
  const float y1 = i + 1 < n ? in[i + 1] : 0.f;
  float p0, p1;
  exp2_poly2(p0, p1, y0, y1);
  out[i] = p0;
  if (i + 1 < n) out[i + 1] = p1;
}

// result[0], result[1]: 1 if the first / second waiter saw its phase complete (never);
// result[2]: ns the second waiter spent before leaving.
__global__ void wait_selftest_kernel(int* status, uint64_t limit_ns, long long* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival completes the phase; none comes
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    result[0] = mbar_wait_ns(&bar, 0, &abort_flag, status, kStatusTimeoutSelftest, limit_ns) ? 1 : 0;
  } else if (threadIdx.x == 32) {
    const uint64_t t0 = global_ns();
    result[1] = mbar_wait_ns(&bar, 0, &abort_flag, status, kStatusTimeoutSelftest + 1, 4 * limit_ns) ? 1 : 0;
    result[2] = static_cast<long long>(global_ns() - t0);
  }
  __syncthreads();
}

}  // namespace

int launch_exp2_check(const float* in, float* out, int n, cudaStream_t stream) {
  if (n <= 0) return n == 0 ? kOk : kErrShape;
  if (in == nullptr || out == nullptr) return kErrShape;
  const int pairs = (n + 1) / 2;
  exp2_check_kernel<<<(pairs + 255) / 256, 256, 0, stream>>>(in, out, n);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

int launch_wait_selftest(int* status, long long limit_ns, long long* result, cudaStream_t stream) {
  if (status == nullptr || result == nullptr || limit_ns <= 0 || limit_ns > 1000000000ll) return kErrShape;
  wait_selftest_kernel<<<1, 64, 0, stream>>>(status, static_cast<uint64_t>(limit_ns), result);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace recap
