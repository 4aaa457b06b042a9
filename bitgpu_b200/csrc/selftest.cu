// bg_selftest_wait_expiry: proves on the device that a bounded mbarrier wait gives up cleanly.
//
// One CTA initialises an mbarrier that expects one arrival, never arrives on it, and waits with the
// same bounded wait (mbar_wait_limit) every kernel of this library uses, here with a caller-chosen
// poll limit.  On expiry the wait records BG_ETIMEOUT in this translation unit's device flag and the
// kernel returns: no trap, no fault, the context stays usable.  bg_device_status reads the flag.
#include "tma.cuh"

namespace bg {
namespace {

__global__ void wait_expiry_kernel(uint32_t polls, int *result) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait_limit(&bar, 0, polls);  // nothing arrives: must expire
    *result = ok ? 1 : 0;
  }
}

}  // namespace

int poll_device_error_selftest() {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return BG_ELAUNCH;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
  return v;
}

}  // namespace bg

static __device__ int g_selftest_result;

extern "C" int bg_selftest_wait_expiry(uint32_t polls, bg_stream_t stream) {
  if (polls == 0 || polls > bg::kSpinLimit) return BG_EINVAL;
  int *res = nullptr;
  if (cudaGetSymbolAddress((void **)&res, g_selftest_result) != cudaSuccess) return BG_ELAUNCH;
  bg::wait_expiry_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(polls, res);
  return cudaGetLastError() == cudaSuccess ? BG_OK : BG_ELAUNCH;
}
