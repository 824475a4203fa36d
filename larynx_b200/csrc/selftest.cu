// lx_flow_selftest_wait: makes the library's bounded device wait run out on
// purpose, so the host-observable failure path (error word -> LX_ERR_TIMEOUT,
// CTA abort flag, tensor memory freed, context still usable) can be tested
// without faulting, trapping or hanging a GPU.
//
// One CTA of four warps, laid out like the library's pipelines:
//   warp 0  producer: arrives on `full` only when asked to
//   warp 1  allocates 32 tensor-memory columns up front and frees them at the
//           end, whatever happened in between
//   warp 2  consumer: mbar_wait_for(`full`) with the caller's limit; when it
//           completes, arrives on `done`
//   warp 3  second waiter, on `done`: it leaves through the abort flag the
//           consumer raises when its own wait runs out
// The waits are the same mbar_wait_for every kernel of the library uses (the
// kernels pass LX_WAIT_TIMEOUT_NS, 2 s; this entry point passes a shorter
// limit so a test finishes in milliseconds).
#include "../../include/larynx_flow.h"
#include "common.cuh"

using namespace lx;

namespace {

__global__ void __launch_bounds__(128, 1) k_wait_selftest(int producer_arrives, uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t full, done;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    mbar_init(&done, 1);
    abort_word = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0) {
    if (lane == 0 && producer_arrives) mbar_arrive(&full);
  } else if (warp == 2) {
    if (lane == 0 && mbar_wait_for(&full, 0, err, abort_flag, DEV_TIMEOUT_EPILOGUE, limit_ns)) mbar_arrive(&done);
  } else if (warp == 3) {
    if (lane == 0) mbar_wait_for(&done, 0, err, abort_flag, DEV_TIMEOUT_SOFTMAX, 4 * limit_ns);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

}  // namespace

extern "C" int lx_flow_selftest_wait(int producer_arrives, double limit_ms, int* device_code, void* stream) {
  if (!(limit_ms > 0.0 && limit_ms <= 2000.0)) return LX_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* d_err = nullptr;
  if (cudaMalloc(&d_err, sizeof(int)) != cudaSuccess) return LX_ERR_OOM;
  int rc = LX_OK;
  int e = 0;
  if (cudaMemsetAsync(d_err, 0, sizeof(int), s) != cudaSuccess) {
    rc = LX_ERR_CUDA;
  } else {
    k_wait_selftest<<<1, 128, 0, s>>>(producer_arrives, static_cast<uint64_t>(limit_ms * 1e6), d_err);
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpyAsync(&e, d_err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      rc = LX_ERR_CUDA;
    else if (e)
      rc = LX_ERR_TIMEOUT;
  }
  cudaFree(d_err);
  if (device_code) *device_code = e;
  return rc;
}
