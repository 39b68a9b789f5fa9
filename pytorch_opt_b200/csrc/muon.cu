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

// 16-byte vectors of T, widened to fp32 in registers.
template <typename T>
struct Vec;
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&f)[N]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __bfloat1622float2(h[e]);
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&f)[N]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const float* p, float (&f)[N]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&f)[N]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

template <typename T>
struct MomentumOp {
  float mu, mu_alpha;
  int nesterov;
  __device__ __forceinline__ void operator()(float gi, float& b, float& out) const {
    const float b1 = round_to<T>(b * mu);  // buf.mul_(mu)
    b = round_to<T>(b1 + gi);              // buf.add_(g)
    out = nesterov ? gi + mu_alpha * b : b;  // g.add(buf, alpha=mu)
  }
};

// vec: every pointer is 16-byte aligned, so whole 16-byte vectors are used
// up to the last full one; the tail (and unaligned arrays) go element-wise.
template <typename T>
__global__ void momentum_kernel(const T* __restrict__ g, T* __restrict__ buf, T* __restrict__ u, long long n,
                                float mu, int nesterov, int vec) {
  // torch's add(..., alpha) on a bf16 tensor rounds alpha to bf16 first; mul_ by a scalar does not.
  const MomentumOp<T> op{mu, round_to<T>(mu), nesterov};
  constexpr int N = Vec<T>::N;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long nvec = vec ? n / N : 0;
  for (long long v = tid; v < nvec; v += stride) {
    float gf[N], bf[N], of[N];
    Vec<T>::load(g + v * N, gf);
    Vec<T>::load(buf + v * N, bf);
#pragma unroll
    for (int e = 0; e < N; ++e) op(gf[e], bf[e], of[e]);
    Vec<T>::store(buf + v * N, bf);
    Vec<T>::store(u + v * N, of);
  }
  for (long long i = nvec * N + tid; i < n; i += stride) {
    float b = ld(buf, i), o;
    op(ld(g, i), b, o);
    buf[i] = cvt<T>(b);
    u[i] = cvt<T>(o);
  }
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void apply_kernel(T* __restrict__ p, const T* __restrict__ o, long long n, float neg_eff, float decay,
                             int use_decay, double* sq, int vec) {
  double acc = 0.0;
  const float alpha = round_to<T>(neg_eff);  // add_(o, alpha=-eff) rounds alpha to the tensor dtype
  auto upd = [&](float pi, float oi) {
    if (use_decay) pi = round_to<T>(pi * decay);  // p.mul_(1 - lr * wd)
    return fmaf(alpha, oi, pi);                    // p.add_(upd, alpha=-eff)
  };
  constexpr int N = Vec<T>::N;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long nvec = vec ? n / N : 0;
  for (long long v = tid; v < nvec; v += stride) {
    float pf[N], of[N];
    Vec<T>::load(p + v * N, pf);
    Vec<T>::load(o + v * N, of);
#pragma unroll
    for (int e = 0; e < N; ++e) {
      pf[e] = upd(pf[e], of[e]);
      acc += static_cast<double>(of[e]) * of[e];
    }
    Vec<T>::store(p + v * N, pf);
  }
  for (long long i = nvec * N + tid; i < n; i += stride) {
    const float oi = ld(o, i);
    p[i] = cvt<T>(upd(ld(p, i), oi));
    acc += static_cast<double>(oi) * oi;
  }
  if (sq != nullptr) {
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) atomicAdd(sq, acc);
  }
}

// Momentum of a [batch][per] group (blockIdx.y = matrix) with the squared
// Frobenius norm of each matrix's u summed on the way: sums[b] += sum(u^2)
// over the values as stored (rounded to T). This is the norm of the
// Newton-Schulz pre-normalisation, so no separate pass over u is needed.
template <typename T>
__global__ void momentum_sumsq_kernel(const T* __restrict__ g, T* __restrict__ buf, T* __restrict__ u, long long per,
                                      float mu, int nesterov, int vec, double* __restrict__ sums) {
  const MomentumOp<T> op{mu, round_to<T>(mu), nesterov};
  const long long off = static_cast<long long>(blockIdx.y) * per;
  g += off;
  buf += off;
  u += off;
  constexpr int N = Vec<T>::N;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long nvec = vec ? per / N : 0;
  double acc = 0.0;
  for (long long v = tid; v < nvec; v += stride) {
    float gf[N], bf[N], of[N];
    Vec<T>::load(g + v * N, gf);
    Vec<T>::load(buf + v * N, bf);
    float part = 0.0f;
#pragma unroll
    for (int e = 0; e < N; ++e) {
      op(gf[e], bf[e], of[e]);
      const float r = round_to<T>(of[e]);
      part = fmaf(r, r, part);
    }
    acc += part;
    Vec<T>::store(buf + v * N, bf);
    Vec<T>::store(u + v * N, of);
  }
  for (long long i = nvec * N + tid; i < per; i += stride) {
    float b = ld(buf, i), o;
    op(ld(g, i), b, o);
    buf[i] = cvt<T>(b);
    u[i] = cvt<T>(o);
    const float r = round_to<T>(o);
    acc += static_cast<double>(r) * r;
  }
  __shared__ double part[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
    atomicAdd(sums + blockIdx.y, t);
  }
}

bool aligned16(const void* a, const void* b, const void* c = nullptr) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15) == 0;
}

int grid_for(long long n) {
  const long long per = 8LL * sm_count();
  const long long need = (n / 8 + 255) / 256 + 1;
  return static_cast<int>(need < per ? (need > 0 ? need : 1) : per);
}

}  // namespace

int launch_momentum_sumsq(const void* g, void* buf, void* u, int dtype, long long batch, long long per, float mu,
                          int nesterov, double* sums, cudaStream_t s) {
  if (batch <= 0 || per <= 0) return PO_OK;
  if (batch > 65535) return set_error(PO_ERR_ARG, "muon momentum: batch too large");
  const int es = dtype == PO_BF16 ? 2 : 4;
  const long long per_block = 256LL * (16 / es) * 4;  // four 16-byte vectors per thread
  long long bx = (per + per_block - 1) / per_block;
  const long long cap = (8LL * sm_count() + batch - 1) / batch;
  if (bx > cap) bx = cap;
  if (bx < 1) bx = 1;
  dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(batch));
  const int vec = aligned16(g, buf, u) && (per * es) % 16 == 0;
  if (dtype == PO_BF16)
    momentum_sumsq_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(g), static_cast<__nv_bfloat16*>(buf), static_cast<__nv_bfloat16*>(u), per,
        mu, nesterov, vec, sums);
  else if (dtype == PO_F32)
    momentum_sumsq_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(g), static_cast<float*>(buf),
                                                      static_cast<float*>(u), per, mu, nesterov, vec, sums);
  else
    return set_error(PO_ERR_ARG, "muon momentum: dtype must be fp32 or bf16");
  return check_cuda(cudaGetLastError(), "muon momentum launch");
}

}  // namespace po

using namespace po;

extern "C" int po_muon_momentum(const void* g, void* buf, void* u, int dtype, long long n, float momentum,
                                int nesterov, void* stream) {
  if (n < 0) return set_error(PO_ERR_ARG, "muon_momentum: negative size");
  if (n == 0) return PO_OK;
  if (!g || !buf || !u) return set_error(PO_ERR_ARG, "muon_momentum: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PO_BF16)
    momentum_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(g), static_cast<__nv_bfloat16*>(buf), static_cast<__nv_bfloat16*>(u), n,
        momentum, nesterov, aligned16(g, buf, u));
  else if (dtype == PO_F32)
    momentum_kernel<float><<<grid_for(n), 256, 0, s>>>(static_cast<const float*>(g), static_cast<float*>(buf),
                                                       static_cast<float*>(u), n, momentum, nesterov,
                                                       aligned16(g, buf, u));
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
                                                            use_decay, sq_sum, aligned16(p, o));
  else if (dtype == PO_F32)
    apply_kernel<float><<<grid_for(n), 256, 0, s>>>(static_cast<float*>(p), static_cast<const float*>(o), n, -lr_eff,
                                                    decay, use_decay, sq_sum, aligned16(p, o));
  else
    return set_error(PO_ERR_ARG, "muon_apply: dtype must be fp32 or bf16");
  return check_cuda(cudaGetLastError(), "muon_apply launch");
}
