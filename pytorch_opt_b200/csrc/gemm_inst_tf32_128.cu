// Instantiation of the tcgen05 GEMM: tf32 operands, BN = 128.
#include "gemm_launch.cuh"

namespace po {
PO_DEFINE_GEMM_INST(KIND_TF32, 128, false)
}  // namespace po
