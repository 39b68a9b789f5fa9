// SOAP's second-moment transport on a basis refresh
// (pytorch_opt/optim/soap.py:98-110): with C_L = Q_L_old^T Q_L_new and
// C_R = Q_R_old^T Q_R_new,
//   V <- (C_L o C_L)^T V (C_R o C_R)          (o: elementwise product)
// as two basis-change products, one squaring pass, and the two-sided apply
// with the transposed left operand read in place. fp32 state runs every
// product as split-tf32 (fp32-grade); bf16 state runs bf16 products with the
// squares rounded to bf16, as the reference's bf16 matmuls round C.
#include <cuda_bf16.h>

#include "common.cuh"

extern "C" size_t po_matmul_workspace_bytes(long long batch, long long M, long long N, long long K, int dtype,
                                            int precision);
extern "C" int po_matmul(const void* A, long long lda, long long sa, int trans_a, const void* B, long long ldb,
                         long long sb, int trans_b, float* C, long long ldc, long long sc, int dtype, int precision,
                         long long batch, long long M, long long N, long long K, float alpha, float beta,
                         void* workspace, size_t workspace_bytes, void* stream);
extern "C" size_t po_precond_workspace_bytes(long long m, long long n, int dtype);
extern "C" int po_precond_apply_ex(const void* L, long long l_ld, int trans_l, const void* G, long long g_ld,
                                   const void* R, long long r_ld, int trans_r, void* out, long long out_ld, int dtype,
                                   long long m, long long n, double* sq_sum, void* workspace, size_t workspace_bytes,
                                   void* stream);

namespace po {
namespace {

// out[i] = c[i]^2 over `count` contiguous elements (out may alias c for fp32).
template <typename T>
__global__ void square_kernel(const float* __restrict__ c, T* __restrict__ out, long long count) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    const float v = c[i];
    if constexpr (sizeof(T) == 4) out[i] = v * v;
    else out[i] = __float2bfloat16_rn(v * v);
  }
}

int launch_square(const float* c, void* out, int dtype, long long count, cudaStream_t s) {
  if (count <= 0) return PO_OK;
  const int threads = 256;
  const long long want = (count + threads - 1) / threads;
  const int blocks = static_cast<int>(want < 8LL * sm_count() ? want : 8LL * sm_count());
  if (dtype == PO_F32) square_kernel<float><<<blocks, threads, 0, s>>>(c, static_cast<float*>(out), count);
  else square_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(c, static_cast<__nv_bfloat16*>(out), count);
  return check_cuda(cudaGetLastError(), "soap_transport square");
}

struct TransportBufs {
  float *cl, *cr;       // basis changes (fp32 product outputs, squared in place for fp32 state)
  void *sl, *sr;        // squares in the state dtype (bf16 state only; else = cl, cr)
  void* rest;           // scratch of the products, reused stage after stage
  size_t rest_bytes;
};

size_t transport_rest(long long m, long long n, int dtype) {
  const int prec = dtype == PO_F32 ? 2 : 0;
  size_t r = po_matmul_workspace_bytes(1, m, m, m, dtype, prec);
  const size_t rr = po_matmul_workspace_bytes(1, n, n, n, dtype, prec);
  if (rr > r) r = rr;
  const size_t ra = po_precond_workspace_bytes(m, n, dtype);
  return ra > r ? ra : r;
}

void transport_layout(Arena& ar, long long m, long long n, int dtype, TransportBufs& B) {
  B.cl = static_cast<float*>(ar.take(static_cast<size_t>(m * m) * 4));
  B.cr = static_cast<float*>(ar.take(static_cast<size_t>(n * n) * 4));
  if (dtype == PO_BF16) {
    B.sl = ar.take(static_cast<size_t>(m * m) * 2);
    B.sr = ar.take(static_cast<size_t>(n * n) * 2);
  } else {
    B.sl = B.cl;
    B.sr = B.cr;
  }
  B.rest_bytes = transport_rest(m, n, dtype);
  B.rest = ar.take(B.rest_bytes);
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" size_t po_soap_transport_workspace_bytes(long long m, long long n, int dtype) {
  if (m <= 0 || n <= 0 || (dtype != PO_F32 && dtype != PO_BF16)) return 0;
  Arena ar(nullptr, 0);
  TransportBufs B;
  transport_layout(ar, m, n, dtype, B);
  return ar.used + 256;
}

extern "C" int po_soap_transport(const void* ql_old, const void* ql_new, long long ql_ld, const void* qr_old,
                                 const void* qr_new, long long qr_ld, void* v, long long v_ld, int dtype, long long m,
                                 long long n, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != PO_F32 && dtype != PO_BF16) return set_error(PO_ERR_ARG, "soap_transport: dtype must be fp32 or bf16");
  if (m < 0 || n < 0) return set_error(PO_ERR_ARG, "soap_transport: negative size");
  if (m == 0 || n == 0) return PO_OK;
  if (!ql_old || !ql_new || !qr_old || !qr_new || !v) return set_error(PO_ERR_ARG, "soap_transport: null pointer");
  if (ql_ld < m || qr_ld < n || v_ld < n) return set_error(PO_ERR_ARG, "soap_transport: pitch too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Arena ar(workspace, workspace_bytes);
  TransportBufs B;
  transport_layout(ar, m, n, dtype, B);
  if (workspace == nullptr || ar.overflow()) return set_error(PO_ERR_WORKSPACE, "soap_transport: workspace too small");
  const int prec = dtype == PO_F32 ? 2 : 0;
  int r;
  // C_L = Q_L_old^T Q_L_new, C_R = Q_R_old^T Q_R_new (fp32 outputs).
  if ((r = po_matmul(ql_old, ql_ld, 0, 1, ql_new, ql_ld, 0, 0, B.cl, m, 0, dtype, prec, 1, m, m, m, 1.0f, 0.0f,
                     B.rest, B.rest_bytes, stream)))
    return r;
  if ((r = po_matmul(qr_old, qr_ld, 0, 1, qr_new, qr_ld, 0, 0, B.cr, n, 0, dtype, prec, 1, n, n, n, 1.0f, 0.0f,
                     B.rest, B.rest_bytes, stream)))
    return r;
  if ((r = launch_square(B.cl, B.sl, dtype, m * m, s))) return r;
  if ((r = launch_square(B.cr, B.sr, dtype, n * n, s))) return r;
  // V <- (C_L o C_L)^T V (C_R o C_R); the apply stages V before its first product, so out may be V.
  return po_precond_apply_ex(B.sl, m, 1, v, v_ld, B.sr, n, 0, v, v_ld, dtype, m, n, nullptr, B.rest, B.rest_bytes,
                             stream);
}
