// Instantiation of the tcgen05 GEMM: bf16 operands, BN = 256.
#include "gemm_launch.cuh"

namespace po {
PO_DEFINE_GEMM_INST(KIND_BF16, 256, false)
}  // namespace po
