// Instantiation of the two-SM tcgen05 GEMM: tf32 operands.
#include "gemm_pair_launch.cuh"

namespace po {
template int dispatch_pair<KIND_TF32>(const GemmParams&, bool, bool, cudaStream_t);
}  // namespace po
