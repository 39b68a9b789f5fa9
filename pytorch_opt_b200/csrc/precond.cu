// Two-sided preconditioner application out = L G R
// (pytorch_opt/ops/reference.py:117-121; ATen version
// pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:96-99) as two chained tensor-core
// products. The first product's epilogue writes L G directly as the operand
// of the second. fp32 inputs run as split-tf32 pairs (hi = tf32(x),
// lo = tf32(x - hi); hi*hi + hi*lo + lo*hi, ~2^-21 relative, fp32-grade:
// Shampoo's eigh-route roots of rank-deficient factors carry entries of
// order damping^(-1/4) whose products with G must stay accurate); bf16
// inputs run as bf16 products.
#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {
namespace {

// Operand buffers: fp32 (hi, lo) pairs for fp32 inputs, bf16 (hi only) for bf16 inputs.
struct PrecondBufs {
  void *lh, *ll, *gh, *gl, *rh, *rl, *ph, *pl;
  long long ldl, ldg, ldr;
  unsigned int* sched;  // tile queue of the two products
};

void precond_layout(Arena& ar, long long m, long long n, bool split, PrecondBufs& B) {
  B.ldl = round_up(m, 64);
  B.ldg = round_up(n, 64);
  B.ldr = round_up(n, 64);
  const size_t es = split ? 4 : 2;
  auto take = [&](long long elems) { return ar.take(static_cast<size_t>(elems) * es); };
  B.lh = take(m * B.ldl);
  B.gh = take(m * B.ldg);
  B.rh = take(n * B.ldr);
  B.ph = take(m * B.ldg);
  B.ll = split ? take(m * B.ldl) : nullptr;
  B.gl = split ? take(m * B.ldg) : nullptr;
  B.rl = split ? take(n * B.ldr) : nullptr;
  B.pl = split ? take(m * B.ldg) : nullptr;
  B.sched = take_sched(ar);
}

MatView oview(const void* p, bool split, long long rows, long long cols, long long ld) {
  MatView v;
  v.ptr = p;
  v.dtype = split ? PO_F32 : PO_BF16;
  v.rows = rows;
  v.cols = cols;
  v.ld = ld;
  v.bstride = rows * ld;
  return v;
}

int stage(const AnyMat& src, bool split, void* hi, void* lo, long long ld, cudaStream_t s) {
  if (split) return launch_split_tf32(src, 1, static_cast<float*>(hi), static_cast<float*>(lo), ld, src.rows * ld, s);
  return launch_split_bf16(src, 1, static_cast<__nv_bfloat16*>(hi), nullptr, ld, src.rows * ld, s);
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" size_t po_precond_workspace_bytes(long long m, long long n, int dtype) {
  if (m <= 0 || n <= 0) return 0;
  Arena ar(nullptr, 0);
  PrecondBufs B;
  precond_layout(ar, m, n, dtype == PO_F32, B);
  return ar.used + 256;
}

extern "C" int po_precond_apply_ex(const void* L, long long l_ld, int trans_l, const void* G, long long g_ld,
                                   const void* R, long long r_ld, int trans_r, void* out, long long out_ld, int dtype,
                                   long long m, long long n, double* sq_sum, void* workspace, size_t workspace_bytes,
                                   void* stream);

extern "C" int po_precond_apply(const void* L, long long l_ld, const void* G, long long g_ld, const void* R,
                                long long r_ld, void* out, long long out_ld, int dtype, long long m, long long n,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return po_precond_apply_ex(L, l_ld, 0, G, g_ld, R, r_ld, 0, out, out_ld, dtype, m, n, nullptr, workspace,
                             workspace_bytes, stream);
}

// As po_precond_apply; with sq_sum (device fp64) also ||out||_F^2 summed by
// the second product's epilogue over the values it stores (grafting norm).
extern "C" int po_precond_apply_norm(const void* L, long long l_ld, const void* G, long long g_ld, const void* R,
                                     long long r_ld, void* out, long long out_ld, int dtype, long long m,
                                     long long n, double* sq_sum, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  return po_precond_apply_ex(L, l_ld, 0, G, g_ld, R, r_ld, 0, out, out_ld, dtype, m, n, sq_sum, workspace,
                             workspace_bytes, stream);
}

// out = op(L) G op(R) with op = transpose when trans_l / trans_r: the staged
// operand is read MN-major instead of K-major, so no transposed copy is made.
extern "C" int po_precond_apply_ex(const void* L, long long l_ld, int trans_l, const void* G, long long g_ld,
                                   const void* R, long long r_ld, int trans_r, void* out, long long out_ld, int dtype,
                                   long long m, long long n, double* sq_sum, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (dtype != PO_F32 && dtype != PO_BF16) return set_error(PO_ERR_ARG, "precond_apply: dtype must be fp32 or bf16");
  if (m < 0 || n < 0) return set_error(PO_ERR_ARG, "precond_apply: negative size");
  if (sq_sum != nullptr) {
    const int rz = check_cuda(cudaMemsetAsync(sq_sum, 0, sizeof(double), static_cast<cudaStream_t>(stream)),
                              "memset");
    if (rz) return rz;
  }
  if (m == 0 || n == 0) return PO_OK;
  if (!L || !G || !R || !out) return set_error(PO_ERR_ARG, "precond_apply: null pointer");
  if (l_ld < m || g_ld < n || r_ld < n || out_ld < n) return set_error(PO_ERR_ARG, "precond_apply: pitch too small");
  if (m > 0x3fffffff || n > 0x3fffffff) return set_error(PO_ERR_ARG, "precond_apply: size too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool split = dtype == PO_F32;
  Arena ar(workspace, workspace_bytes);
  PrecondBufs B;
  precond_layout(ar, m, n, split, B);
  if (workspace == nullptr || ar.overflow()) return set_error(PO_ERR_WORKSPACE, "precond_apply: workspace too small");

  int r;
  if ((r = zero_sched(B.sched, s))) return r;
  AnyMat lm{L, dtype, m, m, l_ld, m * l_ld}, gm{G, dtype, m, n, g_ld, m * g_ld}, rm{R, dtype, n, n, r_ld, n * r_ld};
  if ((r = stage(lm, split, B.lh, B.ll, B.ldl, s))) return r;
  if ((r = stage(gm, split, B.gh, B.gl, B.ldg, s))) return r;
  if ((r = stage(rm, split, B.rh, B.rl, B.ldr, s))) return r;
  const int kind = split ? KIND_TF32 : KIND_BF16;

  // P = L G : A = L [m][m] (K-major), B = G stored [K = m][N = n] (MN-major).
  GemmDesc g1;
  g1.kind = kind;
  g1.M = static_cast<int>(m);
  g1.N = static_cast<int>(n);
  g1.K = static_cast<int>(m);
  g1.a[0] = oview(B.lh, split, m, m, B.ldl);
  g1.b[0] = oview(B.gh, split, m, n, B.ldg);
  if (split) {
    g1.a[1] = oview(B.ll, split, m, m, B.ldl);
    g1.b[1] = oview(B.gl, split, m, n, B.ldg);
    g1.npass = 3;
  }
  g1.a_kmajor = !trans_l;  // L [m][m] read K-major is L, MN-major is L^T
  g1.b_kmajor = false;
  g1.sched = B.sched;
  g1.chunked = split && 3 * m > 1024;
  g1.epi.alpha = 1.0f;
  g1.epi.nout = split ? 2 : 1;
  g1.epi.out[0] = epi_out(B.ph, split ? OUT_TF32 : OUT_BF16, B.ldg, m * B.ldg);
  if (split) g1.epi.out[1] = epi_out(B.pl, OUT_TF32_LO, B.ldg, m * B.ldg);
  if ((r = launch_gemm(g1, s))) return r;

  // out = P R : A = P [m][n] (K-major), B = R stored [K = n][N = n] (MN-major).
  GemmDesc g2;
  g2.kind = kind;
  g2.M = static_cast<int>(m);
  g2.N = static_cast<int>(n);
  g2.K = static_cast<int>(n);
  g2.a[0] = oview(B.ph, split, m, n, B.ldg);
  g2.b[0] = oview(B.rh, split, n, n, B.ldr);
  if (split) {
    g2.a[1] = oview(B.pl, split, m, n, B.ldg);
    g2.b[1] = oview(B.rl, split, n, n, B.ldr);
    g2.npass = 3;
  }
  g2.b_kmajor = trans_r != 0;  // R [n][n] read as [K][N] is R, as [N][K] is R^T
  g2.sched = B.sched;
  g2.chunked = split && 3 * n > 1024;
  g2.epi.alpha = 1.0f;
  g2.epi.nout = 1;
  g2.epi.out[0] = epi_out(out, dtype == PO_F32 ? OUT_F32 : OUT_BF16, out_ld, m * out_ld);
  g2.epi.red_sumsq = sq_sum;  // sums the fp32 values before the store's rounding
  return launch_gemm(g2, s);
}
