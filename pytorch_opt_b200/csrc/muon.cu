// Bandwidth-bound halves of the Muon step (pytorch_opt/optim/muon.py:79-93):
//   momentum:  buf <- buf * mu + g ;  u <- g + mu * buf   (Nesterov) or u <- buf
//   apply:     p <- p * (1 - lr * wd) ;  p <- p - eff * O  ;  sq += sum(O^2)
// The roundings follow the reference's sequence of in-place tensor ops on
// the parameter dtype: every in-place op rounds to that dtype.
#include <cuda_bf16.h>

#include "common.cuh"

namespace po {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p, long long i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, long long i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, long long i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ T cvt(float v);
template <>
__device__ __forceinline__ float cvt<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  const T t = cvt<T>(v);
  return ld<T>(&t, 0);
}

template <typename T>
__global__ void momentum_kernel(const T* __restrict__ g, T* __restrict__ buf, T* __restrict__ u, long long n,
                                float mu, int nesterov) {
  // torch's add(..., alpha) on a bf16 tensor rounds alpha to bf16 first; mul_ by a scalar does not.
  const float mu_alpha = round_to<T>(mu);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float gi = ld(g, i);
    const float b1 = round_to<T>(ld(buf, i) * mu);  // buf.mul_(mu)
    const float b2 = round_to<T>(b1 + gi);          // buf.add_(g)
    buf[i] = cvt<T>(b2);
    u[i] = nesterov ? cvt<T>(gi + mu_alpha * b2) : cvt<T>(b2);  // g.add(buf, alpha=mu)
  }
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void apply_kernel(T* __restrict__ p, const T* __restrict__ o, long long n, float neg_eff, float decay,
                             int use_decay, double* sq) {
  double acc = 0.0;
  const float alpha = round_to<T>(neg_eff);  // add_(o, alpha=-eff) rounds alpha to the tensor dtype
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float pi = ld(p, i);
    if (use_decay) pi = round_to<T>(pi * decay);  // p.mul_(1 - lr * wd)
    const float oi = ld(o, i);
    p[i] = cvt<T>(fmaf(alpha, oi, pi));  // p.add_(upd, alpha=-eff)
    acc += static_cast<double>(oi) * oi;
  }
  if (sq != nullptr) {
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) atomicAdd(sq, acc);
  }
}

int grid_for(long long n) {
  const long long per = 4LL * sm_count();
  const long long need = (n + 255) / 256;
  return static_cast<int>(need < per ? (need > 0 ? need : 1) : per);
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" int po_muon_momentum(const void* g, void* buf, void* u, int dtype, long long n, float momentum,
                                int nesterov, void* stream) {
  if (n < 0) return set_error(PO_ERR_ARG, "muon_momentum: negative size");
  if (n == 0) return PO_OK;
  if (!g || !buf || !u) return set_error(PO_ERR_ARG, "muon_momentum: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PO_BF16)
    momentum_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(g),
                                                               static_cast<__nv_bfloat16*>(buf),
                                                               static_cast<__nv_bfloat16*>(u), n, momentum, nesterov);
  else if (dtype == PO_F32)
    momentum_kernel<float><<<grid_for(n), 256, 0, s>>>(static_cast<const float*>(g), static_cast<float*>(buf),
                                                       static_cast<float*>(u), n, momentum, nesterov);
  else
    return set_error(PO_ERR_ARG, "muon_momentum: dtype must be fp32 or bf16");
  return check_cuda(cudaGetLastError(), "muon_momentum launch");
}

extern "C" int po_muon_apply(void* p, const void* o, int dtype, long long n, float lr_eff, float decay,
                             double* sq_sum, void* stream) {
  if (n < 0) return set_error(PO_ERR_ARG, "muon_apply: negative size");
  if (n == 0) return PO_OK;
  if (!p || !o) return set_error(PO_ERR_ARG, "muon_apply: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int use_decay = decay != 1.0f;
  if (dtype == PO_BF16)
    apply_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, s>>>(static_cast<__nv_bfloat16*>(p),
                                                            static_cast<const __nv_bfloat16*>(o), n, -lr_eff, decay,
                                                            use_decay, sq_sum);
  else if (dtype == PO_F32)
    apply_kernel<float><<<grid_for(n), 256, 0, s>>>(static_cast<float*>(p), static_cast<const float*>(o), n, -lr_eff,
                                                    decay, use_decay, sq_sum);
  else
    return set_error(PO_ERR_ARG, "muon_apply: dtype must be fp32 or bf16");
  return check_cuda(cudaGetLastError(), "muon_apply launch");
}
