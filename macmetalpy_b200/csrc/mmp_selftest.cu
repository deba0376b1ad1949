// mmp_selftest_bounded_wait: demonstrates, on the device, the failure
// behaviour every waiting kernel of the library follows (the scan's
// look-back, the GEMM's mbarrier waits): a wait is bounded; when it runs out
// the kernel records an error code in the device error word and returns, the
// context stays usable, and mmp_check_device_error reports the code.
//
// One block waits on a flag in device memory that nothing sets, polling with
// __nanosleep until `timeout_us` of %globaltimer have passed, then sets
// error code 6.  No memory outside the library's own allocations is touched
// and nothing faults.  No counterpart in the reference (its Metal kernels do
// not wait on one another).
#include <cuda_runtime.h>
#include <stdint.h>

#include "mmp_internal.h"

namespace {

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void bounded_wait_kernel(const volatile unsigned *flag, unsigned long long timeout_ns, int *err,
                                    unsigned *polls) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = gtimer();
  unsigned n = 0;
  while (*flag == 0u) {
    ++n;
    if (gtimer() - t0 > timeout_ns || n > 10000000u) {  // device time, and a poll cap as a second bound
      atomicExch(err, 6);  // the wait ran out: report and return
      break;
    }
    __nanosleep(1000);
  }
  *polls = n;
}

}  // namespace

extern "C" int mmp_selftest_bounded_wait(int timeout_us, unsigned *polls) {
  if (timeout_us <= 0 || timeout_us > 5000000) return mmp::set_error(MMP_E_ARG, "timeout_us must be in (0, 5e6]");
  cudaStream_t st = mmp::stream();
  if (!st) return mmp::set_error(MMP_E_CUDA, "no stream");
  void *buf = nullptr;
  MMP_CUDA_TRY(cudaMallocAsync(&buf, 16, st));
  MMP_CUDA_TRY(cudaMemsetAsync(buf, 0, 16, st));
  unsigned *flag = (unsigned *)buf, *dpolls = flag + 1;
  bounded_wait_kernel<<<1, 32, 0, st>>>(flag, (unsigned long long)timeout_us * 1000ull, mmp::device_error_word(),
                                        dpolls);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && polls) e = cudaMemcpyAsync(polls, dpolls, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
  cudaFreeAsync(buf, st);
  if (e != cudaSuccess) return mmp::cuda_error(e, "bounded_wait_kernel");
  MMP_CUDA_TRY(cudaStreamSynchronize(st));
  return MMP_OK;
}
