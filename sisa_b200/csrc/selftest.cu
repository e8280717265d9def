// selftest.cu - a diagnostic entry point that runs the library's bounded-wait and unwind pattern on a
// handshake whose producer can be told not to arrive, so a test can show on a real GPU that a wait
// which runs out records SISA_ST_TIMEOUT, frees its tensor memory and returns with the context intact.
//
// The kernel has the shape of the library's warp-specialised kernels: warp 0 initialises an mbarrier
// and is the producer, warp 1 owns a tensor-memory allocation, warps 2 and 3 are consumers that wait on
// the barrier with the library's wait (mbar_wait_for, here with the caller's limit instead of
// SISA_WAIT_NS). Every warp then meets at the final block barrier and warp 1 frees the tensor memory,
// as every kernel here does after a timed-out wait.
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100.cuh"
#include "capi_util.h"

namespace sisa {
namespace selftest {

__global__ void __launch_bounds__(128, 1)
    wait_kernel(int producer_arrives, uint64_t limit_ns, int32_t* status, int32_t* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int timed_out;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_barrier_init();
    timed_out = 0;
  }
  if (warp == 1) { tmem_alloc(smem_u32(&tmem_slot), 32); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_slot;
  if (warp == 0) {
    if (lane == 0 && producer_arrives) mbar_arrive(b);
  } else if (warp >= 2) {
    const bool ok = __all_sync(0xffffffffu, mbar_wait_for(b, 0, status, limit_ns));
    if (ok) {
      // the handshake completed: use the tensor memory the way a consumer would
      float v = (float)lane;
      tmem_st1(tbase + ((uint32_t)((warp & 3) * 32) << 16), v);
      tmem_wait_st();
    } else if (lane == 0) {
      atomicAdd(&timed_out, 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 32);
  }
  if (threadIdx.x == 0) result[0] = timed_out;
}

}  // namespace selftest
}  // namespace sisa

extern "C" int sisa_selftest_wait(int producer_arrives, int64_t limit_ns, int32_t* status, int32_t* result,
                                  void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000)
    return sisa::capi_fail(SISA_ERR_VALUE, "sisa_selftest_wait: limit_ns must lie in [1e3, 1e9]");
  if (!result) return sisa::capi_fail(SISA_ERR_VALUE, "sisa_selftest_wait: null result");
  sisa::selftest::wait_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      producer_arrives, (uint64_t)limit_ns, status, result);
  return cudaGetLastError() == cudaSuccess ? SISA_OK
                                           : sisa::capi_fail(SISA_ERR_CUDA, "sisa_selftest_wait launch failed");
}
