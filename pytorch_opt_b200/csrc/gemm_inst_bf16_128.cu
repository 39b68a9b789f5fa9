// Instantiation of the tcgen05 GEMM: bf16 operands, BN = 128.
#include "gemm_launch.cuh"

namespace po {
PO_DEFINE_GEMM_INST(KIND_BF16, 128, false)
}  // namespace po
