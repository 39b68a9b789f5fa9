// Launcher for the two-SM tcgen05 GEMM (clusters of two CTAs). Instantiated
// per operand kind in gemm_inst_pair_*.cu.
#pragma once

#include "gemm_host.cuh"
#include "gemm_pair.cuh"

namespace po {

// Persistent launch: one cluster per co-resident CTA pair, capped by what the
// occupancy query allows on this device (clusters are placed inside one GPC,
// so this can be below SMs / 2).
template <int KIND, bool A_MN, bool B_MN, int ATOMS>
int launch_pair_inst(const GemmParams& P, cudaStream_t stream) {
  using C = PairCfg<KIND, ATOMS>;
  auto kern = tc_gemm_pair_kernel<KIND, A_MN, B_MN, ATOMS>;
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(PO_ERR_CUDA, "device ordinal out of range");
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_pairs[dev] == 0) {
    int r = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES),
                       "cudaFuncSetAttribute");
    if (r) return r;
    cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
    int n = 0;
    r = check_cuda(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "cudaOccupancyMaxActiveClusters");
    if (r) return r;
    if (n <= 0) return set_error(PO_ERR_CUDA, "two-SM GEMM: no cluster of two CTAs fits on this device");
    max_pairs[dev] = n;
  }
  const int pairs = P.total_tiles < max_pairs[dev] ? P.total_tiles : max_pairs[dev];
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, P), "tc_gemm_pair launch");
}

// Three 64 KB stages of two 128-byte K atoms each (PairCfg's default). Six
// 32 KB stages of one atom were measured slower on the Llama step (487 ms
// against 463 ms on one box, at a higher clock: the tensor pipes idled more).
template <int KIND>
int dispatch_pair(const GemmParams& P, bool a_mn, bool b_mn, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_pair_inst<KIND, false, false, 2>(P, s);
  if (!a_mn && b_mn) return launch_pair_inst<KIND, false, true, 2>(P, s);
  if (a_mn && !b_mn) return launch_pair_inst<KIND, true, false, 2>(P, s);
  return launch_pair_inst<KIND, true, true, 2>(P, s);
}

extern template int dispatch_pair<KIND_BF16>(const GemmParams&, bool, bool, cudaStream_t);
extern template int dispatch_pair<KIND_TF32>(const GemmParams&, bool, bool, cudaStream_t);

}  // namespace po
