// Instantiation of the tcgen05 GEMM: tf32 operands, BN = 256.
#include "gemm_launch.cuh"

namespace po {
PO_DEFINE_GEMM_INST(KIND_TF32, 256, false)
}  // namespace po
