// Host-side description of one batched tensor-core product and its launcher.
#pragma once

#include "common.cuh"
#include "gemm.cuh"

namespace po {

// A batched row-major matrix in device memory: [batch][rows][cols], row pitch
// ld, batch pitch bstride (elements). dtype: PO_BF16 or PO_F32.
struct MatView {
  const void* ptr = nullptr;
  int dtype = PO_BF16;
  long long rows = 0, cols = 0, ld = 0, bstride = 0;
};

// D = epilogue(opA * opB) with opA: M x K, opB: K x N.
//   a_kmajor: A stored as [M][K] (K contiguous); otherwise stored as [K][M].
//   b_kmajor: B stored as [N][K] (i.e. B^T row-major); otherwise [K][N].
struct GemmDesc {
  int kind = KIND_BF16;  // operand format on the tensor cores
  int M = 0, N = 0, K = 0, batch = 1;
  MatView a[2];  // [0] plain / hi, [1] lo (npass == 3)
  MatView b[2];
  bool a_kmajor = true;
  bool b_kmajor = true;
  int npass = 1;
  bool tri = false;
  bool chunked = false;  // sum 256-wide K chunks in the epilogue (fp32, round to nearest); BN = 128
  const int* active = nullptr;
  const int* passes = nullptr;
  int bn = 0;  // 0 = choose
  int pair = -1;  // two-SM 256 x 256 tiles: 1 = yes, 0 = no, -1 = choose (never with chunked)
  bool no_mn4d = false;
  // Tile queue of the two-SM kernel: 8 bytes of the caller's workspace, zero
  // before the first launch that uses them (each launch leaves them zero for
  // the next one on the same stream). Null: static round-robin schedule.
  unsigned int* sched = nullptr;  // load MN-major operands block by block (3-D maps) instead of one 4-D copy
  Epilogue epi{};
};

// Helpers to fill epilogue slots.
EpiIn epi_in(const void* ptr, int in_kind, long long ld, long long bstride, float beta);
EpiOut epi_out(void* ptr, int out_kind, long long ld, long long bstride, bool trans = false);

int launch_gemm(const GemmDesc& d, cudaStream_t stream);
// Whether launch_gemm runs this product on the two-SM kernel (256 x 256 tiles).
bool gemm_uses_pair(const GemmDesc& d);

// Tile-queue words for GemmDesc::sched, carved from an op's workspace.
inline unsigned int* take_sched(Arena& ar) { return static_cast<unsigned int*>(ar.take(8)); }
inline int zero_sched(unsigned int* q, cudaStream_t s) {
  return q == nullptr ? PO_OK : check_cuda(cudaMemsetAsync(q, 0, 8, s), "memset");
}

}  // namespace po
