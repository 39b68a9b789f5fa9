// Instantiation of the tcgen05 GEMM: bf16 operands, BN = 128, chunked accumulation.
#include "gemm_launch.cuh"

namespace po {
PO_DEFINE_GEMM_INST(KIND_BF16, 128, true)
}  // namespace po
