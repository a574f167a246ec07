// Health check of the failure-detection path: every wait of the pipelined
// kernels is bounded, and an expired wait records a code in the device status
// word, raises the CTA's abort flag so every other role unwinds, and returns.
// This entry point drives exactly that path on purpose, without TMA, MMA or
// any other asynchronous work in flight: one thread waits on an mbarrier that
// nothing ever completes (with a short limit) and a second warp waits on
// another such barrier with the production limit, so it can only leave
// through the abort flag.  The kernel then returns normally and the context
// stays usable.
#include "../../include/w4a8moe.h"
#include "common.cuh"
#include "w4a8_internal.h"

namespace w4a8 {
void set_last_error(const char* msg);

namespace {
__global__ void wait_timeout_kernel(int* status, long long limit, int* report) {
  __shared__ uint64_t bars[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* ab = &abort_flag;
  if (threadIdx.x == 0) {
    // phase 0 of bars[0] never completes: the wait must run out
    const bool ok = mbar_wait_limit(&bars[0], 0, status, kDevTimeoutSelfTest, ab, limit);
    report[0] = ok ? 1 : 0;
  } else if (threadIdx.x == 32) {
    // a second role: its own limit is the production one (about a second);
    // it returns through the abort flag raised by the first
    const long long t0 = clock64();
    const bool ok = mbar_wait(&bars[1], 0, status, kDevTimeoutLoadFull, ab);
    report[1] = ok ? 1 : 0;
    report[2] = static_cast<int>((clock64() - t0) >> 10);   // kilocycles spent waiting
  }
  __syncthreads();
}
}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" int w4a8_selftest_wait_timeout(int64_t limit_cycles, int32_t* report, void* stream) {
  if (cudaError_t be = bind_stream_device(stream); be != cudaSuccess) {
    set_last_error(cudaGetErrorString(be));
    return W4A8_ERR_CUDA;
  }
  if (limit_cycles <= 0 || limit_cycles > W4A8_WAIT_LIMIT_CYCLES || report == nullptr) {
    set_last_error("w4a8_selftest_wait_timeout: limit_cycles must be in (0, production limit] and report non-null");
    return W4A8_ERR_INVALID;
  }
  int* st = device_status_ptr();
  if (st == nullptr) {
    set_last_error("cannot resolve the device status word");
    return W4A8_ERR_CUDA;
  }
  wait_timeout_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(st, limit_cycles, report);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return W4A8_ERR_CUDA;
  }
  return W4A8_OK;
}
