// Self-test of the kernels' bounded waits: a wait on an mbarrier that nothing
// ever arms must give up after its limit, record its code in the library's
// device error word and let the kernel return, leaving the context usable.
// It runs the same wait functions the GEMM roles use (mbar_wait_bounded for
// the TMA producer and MMA issuer, mbar_wait_bounded_sleep for the epilogue),
// with a short limit in place of their 5 s default.
#include "common.cuh"
#include "ptx.cuh"

namespace po {
namespace {

__global__ void wait_timeout_kernel(unsigned long long limit_ns, int sleeping, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Phase 0 of a fresh barrier with one expected arrival and none made.
    if (sleeping) mbar_wait_bounded_sleep(&bar, 0, &abort_flag, err, kErrTimeoutSelfTest, limit_ns);
    else mbar_wait_bounded(&bar, 0, &abort_flag, err, kErrTimeoutSelfTest, limit_ns);
  }
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" int po_selftest_wait_timeout(unsigned long long limit_ns, int sleeping, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return set_error(PO_ERR_ARG, "selftest_wait_timeout: limit must be in (0, 10 s]");
  int* err = device_error_word();
  if (err == nullptr) return set_error(PO_ERR_CUDA, "device error word unavailable");
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, sleeping, err);
  return check_cuda(cudaGetLastError(), "selftest launch");
}
