// Diagnostic entry point: proves on a GPU that the library's bounded waits
// end with a recorded error instead of a hang.  One CTA waits, with a short
// limit, on an mbarrier phase that nothing will ever complete -- the same
// wait every pipeline role uses -- then records kDevSelfTest in the device
// error word and returns.  Nothing faults, traps or spins without a limit.
#include "internal.h"
#include "ptx.cuh"

namespace cmpx {
namespace {

__global__ void bounded_wait_kernel(int* err, unsigned long long timeout_ns, int* waited_ok) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none will come
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait_limit(&bar, 0, &abort_flag, timeout_ns);
    *waited_ok = ok ? 1 : 0;
    if (!ok) atomicCAS(err, 0, kDevSelfTest);
  }
}

}  // namespace
}  // namespace cmpx

extern "C" CMPX_API int cmpx_selftest_bounded_wait(unsigned long long timeout_ns, cmpx_stream_t stream) {
  using namespace cmpx;
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return CMPX_ERR_INVALID_ARG;
  int* err = device_error_word();
  if (err == nullptr) return CMPX_ERR_CUDA;
  int* flag = nullptr;  // the kernel's "wait succeeded" flag (a tiny stream-ordered allocation)
  if (cudaMallocAsync(reinterpret_cast<void**>(&flag), sizeof(int), stream) != cudaSuccess) return CMPX_ERR_NO_MEMORY;
  bounded_wait_kernel<<<1, 32, 0, stream>>>(err, timeout_ns, flag);
  cudaError_t e = cudaGetLastError();
  int waited_ok = 1;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&waited_ok, flag, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFreeAsync(flag, stream);
  if (e != cudaSuccess) return CMPX_ERR_CUDA;
  return waited_ok ? CMPX_ERR_CUDA : CMPX_ERR_DEVICE;  // the wait must have expired
}
