// Launcher template for the tcgen05 GEMM kernel. Each (operand kind, tile
// width, accumulation mode) combination is instantiated in its own
// translation unit (gemm_inst_*.cu) so the kernels compile in parallel.
#pragma once

#include "gemm_host.cuh"

namespace po {

constexpr int kMaxLaunchDevices = 64;

template <int KIND, int BN, bool A_MN, bool B_MN, bool CHUNKED>
int launch_inst(const GemmParams& P, cudaStream_t stream) {
  using C = GemmCfg<KIND, BN>;
  auto kern = tc_gemm_kernel<KIND, BN, A_MN, B_MN, CHUNKED>;
  static bool configured[kMaxLaunchDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxLaunchDevices && !configured[dev]) {
    int r = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES),
                       "cudaFuncSetAttribute");
    if (r) return r;
    configured[dev] = true;
  }
  const int grid = P.total_tiles < sm_count() ? P.total_tiles : sm_count();
  kern<<<grid, kGemmThreads, C::SMEM_BYTES, stream>>>(P);
  return check_cuda(cudaGetLastError(), "tc_gemm launch");
}

template <int KIND, int BN, bool CHUNKED>
int dispatch_major(const GemmParams& P, bool a_mn, bool b_mn, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_inst<KIND, BN, false, false, CHUNKED>(P, s);
  if (!a_mn && b_mn) return launch_inst<KIND, BN, false, true, CHUNKED>(P, s);
  if (a_mn && !b_mn) return launch_inst<KIND, BN, true, false, CHUNKED>(P, s);
  return launch_inst<KIND, BN, true, true, CHUNKED>(P, s);
}


#define PO_DECLARE_GEMM_INST(KIND, BN, CHUNKED) \
  extern template int dispatch_major<KIND, BN, CHUNKED>(const GemmParams&, bool, bool, cudaStream_t);
#define PO_DEFINE_GEMM_INST(KIND, BN, CHUNKED) \
  template int dispatch_major<KIND, BN, CHUNKED>(const GemmParams&, bool, bool, cudaStream_t);

PO_DECLARE_GEMM_INST(KIND_BF16, 128, false)
PO_DECLARE_GEMM_INST(KIND_BF16, 256, false)
PO_DECLARE_GEMM_INST(KIND_TF32, 128, false)
PO_DECLARE_GEMM_INST(KIND_TF32, 256, false)
PO_DECLARE_GEMM_INST(KIND_BF16, 128, true)
PO_DECLARE_GEMM_INST(KIND_TF32, 128, true)

}  // namespace po
