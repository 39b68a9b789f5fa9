// Instantiation of the two-SM tcgen05 GEMM: bf16 operands.
#include "gemm_pair_launch.cuh"

namespace po {
template int dispatch_pair<KIND_BF16>(const GemmParams&, bool, bool, cudaStream_t);
}  // namespace po
