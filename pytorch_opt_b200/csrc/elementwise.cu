// Bandwidth-bound helper kernels (see elementwise.cuh).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "elementwise.cuh"
#include "gemm.cuh"

namespace po {

template <int DT>
struct Elem;
template <>
struct Elem<PO_F32> {
  using T = float;
  __device__ static double ld(const void* p, long long i) { return static_cast<const float*>(p)[i]; }
};
template <>
struct Elem<PO_BF16> {
  using T = __nv_bfloat16;
  __device__ static double ld(const void* p, long long i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
};
template <>
struct Elem<PO_F16> {
  using T = __half;
  __device__ static double ld(const void* p, long long i) { return __half2float(static_cast<const __half*>(p)[i]); }
};
template <>
struct Elem<PO_F64> {
  using T = double;
  __device__ static double ld(const void* p, long long i) { return static_cast<const double*>(p)[i]; }
};

__device__ __forceinline__ double block_sum(double v) {
  __shared__ double part[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) part[w] = v;
  __syncthreads();
  double t = 0.0;
  if (w == 0) {
    t = (l < static_cast<int>(blockDim.x >> 5)) ? part[l] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

// ------------------------------------------------------------------ sumsq
template <int DT>
__global__ void sumsq_kernel(AnyMat M, double* sums) {
  const int b = blockIdx.y;
  double acc = 0.0;
  for (long long r = blockIdx.x; r < M.rows; r += gridDim.x) {
    const long long base = b * M.bstride + r * M.ld;
    for (long long c = threadIdx.x; c < M.cols; c += blockDim.x) {
      const double v = Elem<DT>::ld(M.ptr, base + c);
      acc += v * v;
    }
  }
  acc = block_sum(acc);
  if (threadIdx.x == 0) atomicAdd(sums + b, acc);
}

int launch_sumsq(const AnyMat& M, int batch, double* sums, cudaStream_t s) {
  if (M.rows <= 0 || M.cols <= 0 || batch <= 0) return PO_OK;
  const int per = static_cast<int>(M.rows < 4LL * sm_count() ? M.rows : 4LL * sm_count());
  const int blocks = batch >= 16 ? (per + 7) / 8 : per;
  dim3 grid(blocks > 0 ? blocks : 1, batch);
  switch (M.dtype) {
    case PO_F32: sumsq_kernel<PO_F32><<<grid, 256, 0, s>>>(M, sums); break;
    case PO_BF16: sumsq_kernel<PO_BF16><<<grid, 256, 0, s>>>(M, sums); break;
    case PO_F16: sumsq_kernel<PO_F16><<<grid, 256, 0, s>>>(M, sums); break;
    case PO_F64: sumsq_kernel<PO_F64><<<grid, 256, 0, s>>>(M, sums); break;
    default: return set_error(PO_ERR_ARG, "sumsq: unsupported dtype");
  }
  return check_cuda(cudaGetLastError(), "sumsq launch");
}

// --------------------------------------------------------------- ns_pack
// One 32 x 128 output tile per block (256 threads): each thread writes four
// consecutive columns of a row with 16-byte (fp32) / 8-byte (bf16) stores.
constexpr int kPackRows = 32, kPackCols = 128;

__device__ __forceinline__ void pack_store4(float* xf, void* xop, void* xlo, int op_kind, long long o, int nvalid,
                                            bool vec, const float (&v)[4]) {
  if (vec && nvalid == 4) {
    *reinterpret_cast<float4*>(xf + o) = make_float4(v[0], v[1], v[2], v[3]);
    if (op_kind == OUT_BF16) {
      __nv_bfloat162 h[2] = {__floats2bfloat162_rn(v[0], v[1]), __floats2bfloat162_rn(v[2], v[3])};
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(xop) + o) = *reinterpret_cast<const uint2*>(h);
      if (xlo != nullptr) {
        const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
        __nv_bfloat162 l[2] = {__floats2bfloat162_rn(v[0] - f0.x, v[1] - f0.y),
                               __floats2bfloat162_rn(v[2] - f1.x, v[3] - f1.y)};
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(xlo) + o) = *reinterpret_cast<const uint2*>(l);
      }
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(xop) + o) =
          make_float4(round_tf32(v[0]), round_tf32(v[1]), round_tf32(v[2]), round_tf32(v[3]));
    }
    return;
  }
  for (int j = 0; j < nvalid; ++j) {
    xf[o + j] = v[j];
    if (op_kind == OUT_BF16) {
      const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
      static_cast<__nv_bfloat16*>(xop)[o + j] = h;
      if (xlo != nullptr) static_cast<__nv_bfloat16*>(xlo)[o + j] = __float2bfloat16_rn(v[j] - __bfloat162float(h));
    } else {
      static_cast<float*>(xop)[o + j] = round_tf32(v[j]);
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(256) ns_pack_kernel(AnyMat src, const double* sums, float eps, float* xf, void* xop,
                                                      void* xlo, int op_kind, long long ldx, long long rows_out,
                                                      long long cols_out, int vec) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int b = blockIdx.z;
  const long long r0 = static_cast<long long>(blockIdx.y) * kPackRows, c0 = static_cast<long long>(blockIdx.x) * kPackCols;
  const float den = static_cast<float>(sqrt(sums[b])) + eps;
  const long long sbase = b * src.bstride;
  const long long xbase = b * rows_out * ldx;
  const long long c = c0 + 4 * tx;
  const int nvalid = c >= cols_out ? 0 : static_cast<int>(cols_out - c < 4 ? cols_out - c : 4);
  for (int i = ty; i < kPackRows; i += 8) {
    const long long r = r0 + i;
    if (r >= rows_out || nvalid == 0) continue;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      v[j] = __fdiv_rn(j < nvalid ? static_cast<float>(Elem<DT>::ld(src.ptr, sbase + r * src.ld + c + j)) : 0.0f, den);
    pack_store4(xf, xop, xlo, op_kind, xbase + r * ldx + c, nvalid, vec != 0, v);
  }
}

// Transposing pack: output element (r, c) = src(c, r) / den. 64 x 64 tiles
// through shared memory; both the src rows read (64 elements) and the output
// rows written (64 elements, two per lane) are contiguous across a warp.
constexpr int kPackT = 64;

template <int DT>
__global__ void __launch_bounds__(256) ns_pack_t_kernel(AnyMat src, const double* sums, float eps, float* xf,
                                                        void* xop, void* xlo, int op_kind, long long ldx,
                                                        long long rows_out, long long cols_out, int vec) {
  __shared__ float tile[kPackT][kPackT + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int b = blockIdx.z;
  const long long r0 = static_cast<long long>(blockIdx.y) * kPackT, c0 = static_cast<long long>(blockIdx.x) * kPackT;
  const float den = static_cast<float>(sqrt(sums[b])) + eps;
  const long long sbase = b * src.bstride;
  // src rows c0.. (output columns), src columns r0.. (output rows).
  for (int i = ty; i < kPackT; i += 8) {
    const long long sr = c0 + i;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const long long sc = r0 + 2 * tx + j;
      float v = 0.0f;
      if (sr < cols_out && sc < rows_out) v = static_cast<float>(Elem<DT>::ld(src.ptr, sbase + sr * src.ld + sc));
      tile[i][2 * tx + j] = v;
    }
  }
  __syncthreads();
  const long long xbase = b * rows_out * ldx;
  const long long c = c0 + 2 * tx;
  const int nvalid = c >= cols_out ? 0 : static_cast<int>(cols_out - c < 2 ? cols_out - c : 2);
  for (int i = ty; i < kPackT; i += 8) {
    const long long r = r0 + i;
    if (r >= rows_out || nvalid == 0) continue;
    const float v0 = __fdiv_rn(tile[2 * tx][i], den), v1 = __fdiv_rn(tile[2 * tx + 1][i], den);
    const long long o = xbase + r * ldx + c;
    if (vec && nvalid == 2) {
      *reinterpret_cast<float2*>(xf + o) = make_float2(v0, v1);
      if (op_kind == OUT_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
        *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(xop) + o) = h;
        if (xlo != nullptr) {
          const float2 f = __bfloat1622float2(h);
          *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(xlo) + o) =
              __floats2bfloat162_rn(v0 - f.x, v1 - f.y);
        }
      } else {
        *reinterpret_cast<float2*>(static_cast<float*>(xop) + o) = make_float2(round_tf32(v0), round_tf32(v1));
      }
    } else {
      const float vv[4] = {v0, v1, 0.0f, 0.0f};
      pack_store4(xf, xop, xlo, op_kind, o, nvalid, false, vv);
    }
  }
}

template <int DT>
static void ns_pack_dt(const AnyMat& src, int batch, bool trans, const double* sums, float eps, float* xf, void* xop,
                       void* xlo, int op_kind, long long ldx, long long rows_out, long long cols_out, cudaStream_t s) {
  // Vector stores need 16-byte aligned rows of every destination.
  const uintptr_t bases = reinterpret_cast<uintptr_t>(xf) | reinterpret_cast<uintptr_t>(xop) |
                          reinterpret_cast<uintptr_t>(xlo);
  const int vec = (bases & 15) == 0 && ldx % 4 == 0;
  if (trans) {
    dim3 grid(cdiv(cols_out, kPackT), cdiv(rows_out, kPackT), batch);
    ns_pack_t_kernel<DT><<<grid, 256, 0, s>>>(src, sums, eps, xf, xop, xlo, op_kind, ldx, rows_out, cols_out, vec);
  } else {
    dim3 grid(cdiv(cols_out, kPackCols), cdiv(rows_out, kPackRows), batch);
    ns_pack_kernel<DT><<<grid, 256, 0, s>>>(src, sums, eps, xf, xop, xlo, op_kind, ldx, rows_out, cols_out, vec);
  }
}

int launch_ns_pack(const AnyMat& src, int batch, bool trans, const double* sums, float eps, float* xf, void* xop,
                   void* xlo, int op_kind, long long ldx, long long rows_out, long long cols_out, cudaStream_t s) {
  if (rows_out <= 0 || cols_out <= 0 || batch <= 0) return PO_OK;
  switch (src.dtype) {
    case PO_F32: ns_pack_dt<PO_F32>(src, batch, trans, sums, eps, xf, xop, xlo, op_kind, ldx, rows_out, cols_out, s); break;
    case PO_BF16: ns_pack_dt<PO_BF16>(src, batch, trans, sums, eps, xf, xop, xlo, op_kind, ldx, rows_out, cols_out, s); break;
    case PO_F16: ns_pack_dt<PO_F16>(src, batch, trans, sums, eps, xf, xop, xlo, op_kind, ldx, rows_out, cols_out, s); break;
    case PO_F64: ns_pack_dt<PO_F64>(src, batch, trans, sums, eps, xf, xop, xlo, op_kind, ldx, rows_out, cols_out, s); break;
    default: return set_error(PO_ERR_ARG, "ns_pack: unsupported dtype");
  }
  return check_cuda(cudaGetLastError(), "ns_pack launch");
}

// --------------------------------------------------------------- copy_out
__device__ __forceinline__ void store_any(void* p, int dt, long long i, float v) {
  switch (dt) {
    case PO_F32: static_cast<float*>(p)[i] = v; break;
    case PO_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case PO_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
    default: static_cast<double*>(p)[i] = static_cast<double>(v); break;
  }
}

// out (rows x cols, or cols x rows when TRANS) from src rows x cols.
template <bool TRANS>
__global__ void copy_out_kernel(const float* src, long long ld_src, long long bs_src, long long rows, long long cols,
                                void* out, int out_dtype, long long ld_out, long long bs_out) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const long long r0 = static_cast<long long>(blockIdx.y) * 32, c0 = static_cast<long long>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = r0 + i, c = c0 + threadIdx.x;
    float v = 0.0f;
    if (r < rows && c < cols) v = src[b * bs_src + r * ld_src + c];
    if (!TRANS) {
      if (r < rows && c < cols) store_any(out, out_dtype, b * bs_out + r * ld_out + c, v);
    } else {
      tile[i][threadIdx.x] = v;
    }
  }
  if (TRANS) {
    __syncthreads();
    // out(c, r) = src(r, c): write rows c0.. of out, coalesced along r.
    for (int i = threadIdx.y; i < 32; i += 8) {
      const long long oc = c0 + i, orr = r0 + threadIdx.x;
      if (oc < cols && orr < rows) store_any(out, out_dtype, b * bs_out + oc * ld_out + orr, tile[threadIdx.x][i]);
    }
  }
}

int launch_copy_out(const float* src, long long ld_src, long long bs_src, int batch, long long rows, long long cols,
                    bool trans, void* out, int out_dtype, long long ld_out, long long bs_out, cudaStream_t s) {
  if (rows <= 0 || cols <= 0 || batch <= 0) return PO_OK;
  dim3 grid(cdiv(cols, 32), cdiv(rows, 32), batch), block(32, 8);
  if (trans) copy_out_kernel<true><<<grid, block, 0, s>>>(src, ld_src, bs_src, rows, cols, out, out_dtype, ld_out, bs_out);
  else copy_out_kernel<false><<<grid, block, 0, s>>>(src, ld_src, bs_src, rows, cols, out, out_dtype, ld_out, bs_out);
  return check_cuda(cudaGetLastError(), "copy_out launch");
}

// ---------------------------------------------------------------- convert
template <int DT>
__global__ void convert_kernel(AnyMat src, void* dst, int dst_dtype, long long ld_dst, long long bs_dst) {
  const int b = blockIdx.y;
  for (long long r = blockIdx.x; r < src.rows; r += gridDim.x) {
    const long long sb = b * src.bstride + r * src.ld, db = b * bs_dst + r * ld_dst;
    for (long long c = threadIdx.x; c < src.cols; c += blockDim.x) {
      const float v = static_cast<float>(Elem<DT>::ld(src.ptr, sb + c));
      if (dst_dtype == PO_F32) static_cast<float*>(dst)[db + c] = v;
      else static_cast<__nv_bfloat16*>(dst)[db + c] = __float2bfloat16_rn(v);
    }
  }
}

int launch_convert(const AnyMat& src, int batch, void* dst, int dst_dtype, long long ld_dst, long long bs_dst,
                   cudaStream_t s) {
  if (src.rows <= 0 || src.cols <= 0 || batch <= 0) return PO_OK;
  if (dst_dtype != PO_F32 && dst_dtype != PO_BF16) return set_error(PO_ERR_ARG, "convert: bad destination dtype");
  const int per = static_cast<int>(src.rows < 8LL * sm_count() ? src.rows : 8LL * sm_count());
  dim3 grid(per, batch);
  switch (src.dtype) {
    case PO_F32: convert_kernel<PO_F32><<<grid, 256, 0, s>>>(src, dst, dst_dtype, ld_dst, bs_dst); break;
    case PO_BF16: convert_kernel<PO_BF16><<<grid, 256, 0, s>>>(src, dst, dst_dtype, ld_dst, bs_dst); break;
    case PO_F16: convert_kernel<PO_F16><<<grid, 256, 0, s>>>(src, dst, dst_dtype, ld_dst, bs_dst); break;
    case PO_F64: convert_kernel<PO_F64><<<grid, 256, 0, s>>>(src, dst, dst_dtype, ld_dst, bs_dst); break;
    default: return set_error(PO_ERR_ARG, "convert: unsupported dtype");
  }
  return check_cuda(cudaGetLastError(), "convert launch");
}

// ------------------------------------------------------------- split bf16
template <int DT>
__global__ void split_kernel(AnyMat src, __nv_bfloat16* hi, __nv_bfloat16* lo, long long ld_dst, long long bs_dst) {
  const int b = blockIdx.y;
  for (long long r = blockIdx.x; r < src.rows; r += gridDim.x) {
    const long long sb = b * src.bstride + r * src.ld, db = b * bs_dst + r * ld_dst;
    for (long long c = threadIdx.x; c < src.cols; c += blockDim.x) {
      const float v = static_cast<float>(Elem<DT>::ld(src.ptr, sb + c));
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      hi[db + c] = h;
      if (lo != nullptr) lo[db + c] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
  }
}

int launch_split_bf16(const AnyMat& src, int batch, __nv_bfloat16* hi, __nv_bfloat16* lo, long long ld_dst,
                      long long bs_dst, cudaStream_t s) {
  if (src.rows <= 0 || src.cols <= 0 || batch <= 0) return PO_OK;
  const int per = static_cast<int>(src.rows < 8LL * sm_count() ? src.rows : 8LL * sm_count());
  dim3 grid(per, batch);
  switch (src.dtype) {
    case PO_F32: split_kernel<PO_F32><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    case PO_BF16: split_kernel<PO_BF16><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    case PO_F16: split_kernel<PO_F16><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    case PO_F64: split_kernel<PO_F64><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    default: return set_error(PO_ERR_ARG, "split: unsupported dtype");
  }
  return check_cuda(cudaGetLastError(), "split launch");
}

// ------------------------------------------------------------- split tf32
template <int DT>
__global__ void split_tf32_kernel(AnyMat src, float* hi, float* lo, long long ld_dst, long long bs_dst) {
  const int b = blockIdx.y;
  for (long long r = blockIdx.x; r < src.rows; r += gridDim.x) {
    const long long sb = b * src.bstride + r * src.ld, db = b * bs_dst + r * ld_dst;
    for (long long c = threadIdx.x; c < src.cols; c += blockDim.x) {
      const float v = static_cast<float>(Elem<DT>::ld(src.ptr, sb + c));
      const float h = round_tf32(v);
      hi[db + c] = h;
      lo[db + c] = round_tf32(v - h);
    }
  }
}

int launch_split_tf32(const AnyMat& src, int batch, float* hi, float* lo, long long ld_dst, long long bs_dst,
                      cudaStream_t s) {
  if (src.rows <= 0 || src.cols <= 0 || batch <= 0) return PO_OK;
  const int per = static_cast<int>(src.rows < 8LL * sm_count() ? src.rows : 8LL * sm_count());
  dim3 grid(per, batch);
  switch (src.dtype) {
    case PO_F32: split_tf32_kernel<PO_F32><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    case PO_BF16: split_tf32_kernel<PO_BF16><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    case PO_F16: split_tf32_kernel<PO_F16><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    case PO_F64: split_tf32_kernel<PO_F64><<<grid, 256, 0, s>>>(src, hi, lo, ld_dst, bs_dst); break;
    default: return set_error(PO_ERR_ARG, "split: unsupported dtype");
  }
  return check_cuda(cudaGetLastError(), "split launch");
}

}  // namespace po
