// selftest.cu -- ltxattn_selftest_wait_timeout: makes the library's bounded
// wait run out on the GPU, so the failure-detection path can be tested
// without a fault.
//
// One CTA of 128 threads, laid out like the attention kernels' set-up: warp 0
// allocates TMEM, one thread initialises an mbarrier that expects a single
// arrival, and every warp then waits on that barrier's first phase with the
// same whole-warp bounded wait (warp_wait -> mbar_wait) the attention kernels
// use.  Nothing ever arrives.  The first wait to pass the caller's limit
// records (site << 8) | timeout in the device error word and raises the CTA's
// abort flag; the other warps see the flag and stop waiting.  The CTA then
// frees its TMEM and exits normally: no trap, no fault, and the context stays
// usable.  The host reads the word with ltxattn_device_status.
#include "../../include/ltxattn.h"
#include "sm100.cuh"

namespace ltx {

int* device_error_word();
int set_error_message(int status, const char* msg);

namespace {

constexpr int kSelftestSite = 99;

__global__ void __launch_bounds__(128, 1) selftest_wait_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // the wait that cannot complete (phase 0 of a barrier nobody arrives on)
  const bool ok = warp_wait(&bar, 0, &abort_flag, err, kSelftestSite, limit_ns);
  (void)ok;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

}  // namespace
}  // namespace ltx

extern "C" {

int ltxattn_selftest_wait_timeout(uint32_t limit_us, void* stream) {
  if (limit_us < 1 || limit_us > 1000000)
    return ltx::set_error_message(LTXATTN_ERR_ARG, "ltxattn_selftest_wait_timeout: limit_us must be in [1, 1000000]");
  int* err = ltx::device_error_word();
  if (err == nullptr) return ltx::set_error_message(LTXATTN_ERR_CUDA, "no device error word");
  ltx::selftest_wait_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(err, uint64_t(limit_us) * 1000ull);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ltx::set_error_message(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
  return LTXATTN_OK;
}

}  // extern "C"
