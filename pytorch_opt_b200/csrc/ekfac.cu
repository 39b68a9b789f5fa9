// EKFAC preconditioning of one layer's gradient
// (pytorch_opt/optim/ekfac.py:44-58):
//   Vt  = QG^T V QA
//   S   = first ? Vt^2 : decay * S + (1 - decay) * Vt^2        (in place)
//   out = QG (Vt / (S + lam)) QA^T
// as four chained tensor-core products on split-tf32 operands (hi*hi + hi*lo
// + lo*hi on the tf32 tensor cores, ~2^-21 relative: fp32-grade, like the
// two-sided apply; the division by S + lam amplifies operand rounding where
// Vt is small, so bf16 pairs are not accurate enough). The second product's epilogue
// updates S and writes Vt / (S + lam) straight into the operand pair of the
// third, so Vt itself is never stored.
#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {
namespace {

struct EkfacBufs {  // tf32 (hi, lo) pairs stored as fp32
  float *gh, *gl;  // QG  [m][m]
  float *ah, *al;  // QA  [n][n]
  float *vh, *vl;  // V   [m][n]
  float *th, *tl;  // QG^T V, then QG W  [m][n]
  float *wh, *wl;  // W = Vt / (S + lam)  [m][n]
  long long ldm, ldn;
  unsigned int* sched;
};

void ekfac_layout(Arena& ar, long long m, long long n, EkfacBufs& B) {
  B.ldm = round_up(m, 64);
  B.ldn = round_up(n, 64);
  auto take = [&](long long elems) { return static_cast<float*>(ar.take(static_cast<size_t>(elems) * 4)); };
  B.gh = take(m * B.ldm);
  B.gl = take(m * B.ldm);
  B.ah = take(n * B.ldn);
  B.al = take(n * B.ldn);
  B.vh = take(m * B.ldn);
  B.vl = take(m * B.ldn);
  B.th = take(m * B.ldn);
  B.tl = take(m * B.ldn);
  B.wh = take(m * B.ldn);
  B.wl = take(m * B.ldn);
  B.sched = take_sched(ar);
}

MatView fview(const float* p, long long rows, long long cols, long long ld) {
  MatView v;
  v.ptr = p;
  v.dtype = PO_F32;
  v.rows = rows;
  v.cols = cols;
  v.ld = ld;
  v.bstride = rows * ld;
  return v;
}

// C = op(A) op(B) on split-tf32 pairs; epilogue set by the caller.
GemmDesc split_product(const MatView (&a)[2], bool a_kmajor, const MatView (&b)[2], bool b_kmajor, long long M,
                       long long N, long long K, unsigned int* sched) {
  GemmDesc g;
  g.kind = KIND_TF32;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.a[0] = a[0];
  g.a[1] = a[1];
  g.b[0] = b[0];
  g.b[1] = b[1];
  g.a_kmajor = a_kmajor;
  g.b_kmajor = b_kmajor;
  g.npass = 3;
  g.chunked = 3 * K > 1024;
  g.sched = sched;
  g.epi.alpha = 1.0f;
  return g;
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" size_t po_ekfac_workspace_bytes(long long m, long long n) {
  if (m <= 0 || n <= 0) return 0;
  Arena ar(nullptr, 0);
  EkfacBufs B;
  ekfac_layout(ar, m, n, B);
  return ar.used + 256;
}

extern "C" int po_ekfac_precondition(const float* QG, long long qg_ld, const float* QA, long long qa_ld, const float* V,
                                     long long v_ld, float* S, long long s_ld, float* out, long long out_ld,
                                     long long m, long long n, int first, float decay, float lam, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (m < 0 || n < 0) return set_error(PO_ERR_ARG, "ekfac_precondition: negative size");
  if (m == 0 || n == 0) return PO_OK;
  if (!QG || !QA || !V || !S || !out) return set_error(PO_ERR_ARG, "ekfac_precondition: null pointer");
  if (qg_ld < m || qa_ld < n || v_ld < n || s_ld < n || out_ld < n)
    return set_error(PO_ERR_ARG, "ekfac_precondition: pitch too small");
  if (m > 0x3fffffff || n > 0x3fffffff) return set_error(PO_ERR_ARG, "ekfac_precondition: size too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Arena ar(workspace, workspace_bytes);
  EkfacBufs B;
  ekfac_layout(ar, m, n, B);
  if (workspace == nullptr || ar.overflow())
    return set_error(PO_ERR_WORKSPACE, "ekfac_precondition: workspace too small (query po_ekfac_workspace_bytes)");
  int r;
  if ((r = zero_sched(B.sched, s))) return r;
  AnyMat gm{QG, PO_F32, m, m, qg_ld, m * qg_ld}, am{QA, PO_F32, n, n, qa_ld, n * qa_ld},
      vm{V, PO_F32, m, n, v_ld, m * v_ld};
  if ((r = launch_split_tf32(gm, 1, B.gh, B.gl, B.ldm, m * B.ldm, s))) return r;
  if ((r = launch_split_tf32(am, 1, B.ah, B.al, B.ldn, n * B.ldn, s))) return r;
  if ((r = launch_split_tf32(vm, 1, B.vh, B.vl, B.ldn, m * B.ldn, s))) return r;
  const MatView QGv[2] = {fview(B.gh, m, m, B.ldm), fview(B.gl, m, m, B.ldm)};
  const MatView QAv[2] = {fview(B.ah, n, n, B.ldn), fview(B.al, n, n, B.ldn)};
  const MatView Vv[2] = {fview(B.vh, m, n, B.ldn), fview(B.vl, m, n, B.ldn)};
  const MatView Tv[2] = {fview(B.th, m, n, B.ldn), fview(B.tl, m, n, B.ldn)};
  const MatView Wv[2] = {fview(B.wh, m, n, B.ldn), fview(B.wl, m, n, B.ldn)};
  auto split_out = [&](GemmDesc& g, float* hi, float* lo) {
    g.epi.nout = 2;
    g.epi.out[0] = epi_out(hi, OUT_TF32, B.ldn, m * B.ldn);
    g.epi.out[1] = epi_out(lo, OUT_TF32_LO, B.ldn, m * B.ldn);
  };

  // T = QG^T V: A = QG stored [K = m][M = m] (MN-major), B = V [K = m][N = n] (MN-major).
  GemmDesc g1 = split_product(QGv, false, Vv, false, m, n, m, B.sched);
  split_out(g1, B.th, B.tl);
  if ((r = launch_gemm(g1, s))) return r;

  // Vt = T QA: A = T [M][K = n] (K-major), B = QA [K][N] (MN-major); the epilogue
  // updates S and writes W = Vt / (S + lam).
  GemmDesc g2 = split_product(Tv, true, QAv, false, m, n, n, B.sched);
  g2.epi.ek_s = S;
  g2.epi.ek_ld = s_ld;
  g2.epi.ek_bstride = m * s_ld;
  g2.epi.ek_decay = decay;
  g2.epi.ek_lam = lam;
  g2.epi.ek_first = first ? 1 : 0;
  split_out(g2, B.wh, B.wl);
  if ((r = launch_gemm(g2, s))) return r;

  // T = QG W: A = QG [M][K] (K-major), B = W [K = m][N = n] (MN-major).
  GemmDesc g3 = split_product(QGv, true, Wv, false, m, n, m, B.sched);
  split_out(g3, B.th, B.tl);
  if ((r = launch_gemm(g3, s))) return r;

  // out = T QA^T: A = T [M][K = n] (K-major), B = QA^T, stored QA [N][K] (K-major).
  GemmDesc g4 = split_product(Tv, true, QAv, true, m, n, n, B.sched);
  g4.epi.nout = 1;
  g4.epi.out[0] = epi_out(out, OUT_F32, out_ld, m * out_ld);
  return launch_gemm(g4, s);
}
