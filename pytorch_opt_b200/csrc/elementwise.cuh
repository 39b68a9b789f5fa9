// Bandwidth-bound helper kernels around the tensor-core products: norms,
// packing (cast / transpose / split into bf16 hi-lo), identity-shifted
// initialisation and typed copies.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace po {

// A strided batched matrix of any supported element type.
struct AnyMat {
  const void* ptr;
  int dtype;  // PO_F32 / PO_BF16 / PO_F16 / PO_F64
  long long rows, cols, ld, bstride;
};

// sums[b] += sum of squares of M[b] (fp64 accumulation). sums must be zeroed.
int launch_sumsq(const AnyMat& M, int batch, double* sums, cudaStream_t s);

// Pack a matrix batch into the Newton–Schulz working buffers:
//   X[b] = src[b] (transposed when `trans`) / (sqrt(sums[b]) + eps)
// written as fp32 master (xf, pitch ldx) and as the first product operand
// (xop: bf16 when op_kind == OUT_BF16, tf32-rounded fp32 when OUT_TF32;
// with OUT_BF16 and a non-null xlo, also the low bf16 half of a split pair).
// The packed matrix is rows_out x cols_out.
int launch_ns_pack(const AnyMat& src, int batch, bool trans, const double* sums, float eps, float* xf,
                   void* xop, void* xlo, int op_kind, long long ldx, long long rows_out, long long cols_out,
                   cudaStream_t s);

// out[b] = cast(src[b]) (transposed when `trans`); src fp32 [rows][cols].
int launch_copy_out(const float* src, long long ld_src, long long bs_src, int batch, long long rows, long long cols,
                    bool trans, void* out, int out_dtype, long long ld_out, long long bs_out, cudaStream_t s);

// dst[b] = src[b] converted to dst_dtype (PO_F32 or PO_BF16) with pitch ld_dst.
int launch_convert(const AnyMat& src, int batch, void* dst, int dst_dtype, long long ld_dst, long long bs_dst,
                   cudaStream_t s);

// Split a matrix batch into bf16 hi/lo parts (hi = bf16(x), lo = bf16(x - hi))
// with padded pitch ld_dst; lo may be null (hi only).
int launch_split_bf16(const AnyMat& src, int batch, __nv_bfloat16* hi, __nv_bfloat16* lo, long long ld_dst,
                      long long bs_dst, cudaStream_t s);

// Split a matrix batch into a tf32 pair (hi = tf32(x), lo = tf32(x - hi),
// both stored as fp32, round to nearest): hi + lo carries ~22 significant
// bits, and hi*hi + hi*lo + lo*hi on the tf32 tensor cores gives products
// accurate to ~2^-21 (fp32-grade; the bf16 pair gives ~2^-16).
int launch_split_tf32(const AnyMat& src, int batch, float* hi, float* lo, long long ld_dst, long long bs_dst,
                      cudaStream_t s);

// Muon momentum (pytorch_opt/optim/muon.py:82-83) of a [batch][per] group of
// dtype PO_BF16 / PO_F32: buf <- buf*mu + g, u <- nesterov ? g + mu*buf :
// buf, and sums[b] += sum(u^2) of matrix b (sums must be zeroed).
int launch_momentum_sumsq(const void* g, void* buf, void* u, int dtype, long long batch, long long per, float mu,
                          int nesterov, double* sums, cudaStream_t s);

}  // namespace po
