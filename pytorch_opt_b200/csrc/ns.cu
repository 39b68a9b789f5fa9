// Newton–Schulz orthogonalisation on the tensor cores.
//
// Mirrors pytorch_opt/ops/reference.py:71-97 (and the ATen version
// pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:65-81). Per matrix (m = min dim):
//   pack   : X0 = G (transposed when rows > cols) / (||G||_F + eps)
//   iterate: A = X X^T          (symmetric: lower tiles only, mirrored)
//            B = b A + c A A    (symmetric: lower tiles only, A A = A A^T)
//            X = a X + B X      (fp32 master copy of X updated in place)
//   the last update writes the caller's output directly (transposed back,
//   cast to the input dtype).
// Iterations before the last `tf32_tail` ones use bf16 operands, the tail
// uses tf32 operands rounded to nearest; all products accumulate in fp32.
#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {

namespace {

struct NsBuffers {
  float* xf;                // fp32 master X            [batch][m][ldx]
  __nv_bfloat16* xb[2];     // bf16 operand copies of X (ping-pong)
  float* xt[2];             // tf32-rounded operand copies of X (ping-pong)
  float* af;                // fp32 A = X X^T           [batch][m][ldm]
  void* aop;                // A as product operand (bf16 or tf32)
  void* bop;                // B as product operand (bf16 or tf32)
  double* sums;             // per-matrix sum of squares
  long long ldx, ldm;
};

void ns_layout(Arena& ar, long long batch, long long m, long long n, NsBuffers& B) {
  B.ldx = round_up(n, 64);
  B.ldm = round_up(m, 64);
  const size_t xs = static_cast<size_t>(batch * m * B.ldx);
  const size_t ms = static_cast<size_t>(batch * m * B.ldm);
  B.xf = static_cast<float*>(ar.take(xs * 4));
  for (int i = 0; i < 2; ++i) B.xb[i] = static_cast<__nv_bfloat16*>(ar.take(xs * 2));
  for (int i = 0; i < 2; ++i) B.xt[i] = static_cast<float*>(ar.take(xs * 4));
  B.af = static_cast<float*>(ar.take(ms * 4));
  B.aop = ar.take(ms * 4);
  B.bop = ar.take(ms * 4);
  B.sums = static_cast<double*>(ar.take(static_cast<size_t>(batch) * 8));
}

// Default precision schedule. bf16 products on all but the last two steps
// keep the result within 1e-2 (relative Frobenius) of the fp32 reference for
// m >= 512; smaller matrices, whose error is dominated by fewer singular
// values, run every step on tf32 (they are cheap).
int ns_auto_tf32_tail(long long m, int steps) { return m < 512 ? steps : (steps < 2 ? steps : 2); }

int out_kind_of(int dtype) {
  switch (dtype) {
    case PO_F32: return OUT_F32;
    case PO_BF16: return OUT_BF16;
    case PO_F16: return OUT_F16;
    default: return OUT_F64;
  }
}

MatView view(const void* p, int dtype, long long rows, long long cols, long long ld) {
  MatView v;
  v.ptr = p;
  v.dtype = dtype;
  v.rows = rows;
  v.cols = cols;
  v.ld = ld;
  v.bstride = rows * ld;
  return v;
}

}  // namespace

}  // namespace po

using namespace po;

extern "C" size_t po_ns_workspace_bytes(long long batch, long long rows, long long cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  const long long m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  Arena ar(nullptr, 0);
  NsBuffers B;
  ns_layout(ar, batch, m, n, B);
  return ar.used + 256;
}

extern "C" int po_newton_schulz(const void* G, int dtype, long long batch, long long rows, long long cols,
                                long long ld, long long bstride, void* out, long long out_ld, long long out_bstride,
                                int steps, float a, float b, float c, float eps, int tf32_tail, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (dtype != PO_F32 && dtype != PO_BF16 && dtype != PO_F16 && dtype != PO_F64)
    return set_error(PO_ERR_ARG, "newton_schulz: dtype must be fp32, bf16, fp16 or fp64");
  if (batch < 0 || rows < 0 || cols < 0 || steps < 0)
    return set_error(PO_ERR_ARG, "newton_schulz: negative size or step count");
  if (batch == 0 || rows == 0 || cols == 0) return PO_OK;
  if (G == nullptr || out == nullptr) return set_error(PO_ERR_ARG, "newton_schulz: null pointer");
  if (ld < cols || out_ld < cols) return set_error(PO_ERR_ARG, "newton_schulz: row pitch smaller than cols");
  if (batch > 65535) return set_error(PO_ERR_ARG, "newton_schulz: batch too large (max 65535)");
  if (tf32_tail < 0) tf32_tail = ns_auto_tf32_tail(rows < cols ? rows : cols, steps);
  if (tf32_tail > steps) tf32_tail = steps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const bool trans = rows > cols;
  const long long m = trans ? cols : rows, n = trans ? rows : cols;
  if (m > 0x7fffffffLL / 2 || n > 0x7fffffffLL / 2) return set_error(PO_ERR_ARG, "newton_schulz: matrix too large");
  Arena ar(workspace, workspace_bytes);
  NsBuffers B;
  ns_layout(ar, batch, m, n, B);
  if (workspace == nullptr || ar.overflow())
    return set_error(PO_ERR_WORKSPACE, "newton_schulz: workspace too small (query po_ns_workspace_bytes)");

  int r = check_cuda(cudaMemsetAsync(B.sums, 0, static_cast<size_t>(batch) * 8, s), "memset");
  if (r) return r;
  AnyMat src{G, dtype, rows, cols, ld, bstride};
  if ((r = launch_sumsq(src, static_cast<int>(batch), B.sums, s))) return r;
  const bool first_tf32 = steps - tf32_tail <= 0;
  if ((r = launch_ns_pack(src, static_cast<int>(batch), trans, B.sums, eps, B.xf,
                          first_tf32 ? static_cast<void*>(B.xt[0]) : static_cast<void*>(B.xb[0]),
                          first_tf32 ? OUT_TF32 : OUT_BF16, B.ldx, m, n, s)))
    return r;
  if (steps == 0)
    return launch_copy_out(B.xf, B.ldx, m * B.ldx, static_cast<int>(batch), m, n, trans, out, dtype, out_ld,
                           out_bstride, s);

  const long long xs = m * B.ldx, ms = m * B.ldm;
  int cur = 0;
  for (int it = 0; it < steps; ++it) {
    const bool tf = it >= steps - tf32_tail;
    const int kind = tf ? KIND_TF32 : KIND_BF16;
    const int op_dt = tf ? PO_F32 : PO_BF16;
    const int op_out = tf ? OUT_TF32 : OUT_BF16;
    const MatView X = tf ? view(B.xt[cur], PO_F32, m, n, B.ldx) : view(B.xb[cur], PO_BF16, m, n, B.ldx);
    const MatView Aop = view(B.aop, op_dt, m, m, B.ldm);
    const MatView Bop = view(B.bop, op_dt, m, m, B.ldm);

    // A = X X^T
    GemmDesc g;
    g.kind = kind;
    g.M = g.N = static_cast<int>(m);
    g.K = static_cast<int>(n);
    g.batch = static_cast<int>(batch);
    g.a[0] = X;
    g.b[0] = X;
    g.tri = true;
    g.epi.alpha = 1.0f;
    g.epi.nout = 2;
    g.epi.out[0] = epi_out(B.af, OUT_F32, B.ldm, ms);
    g.epi.out[1] = epi_out(B.aop, op_out, B.ldm, ms);
    if ((r = launch_gemm(g, s))) return r;

    // B = b A + c A A
    GemmDesc q;
    q.kind = kind;
    q.M = q.N = q.K = static_cast<int>(m);
    q.batch = static_cast<int>(batch);
    q.a[0] = Aop;
    q.b[0] = Aop;
    q.tri = true;
    q.epi.alpha = c;
    q.epi.nin = 1;
    q.epi.in[0] = epi_in(B.af, IN_F32, B.ldm, ms, b);
    q.epi.nout = 1;
    q.epi.out[0] = epi_out(B.bop, op_out, B.ldm, ms);
    if ((r = launch_gemm(q, s))) return r;

    // X = a X + B X ; B operand is X stored [K = m][N = n] (MN-major).
    GemmDesc u;
    u.kind = kind;
    u.M = static_cast<int>(m);
    u.N = static_cast<int>(n);
    u.K = static_cast<int>(m);
    u.batch = static_cast<int>(batch);
    u.a[0] = Bop;
    u.b[0] = X;
    u.b_kmajor = false;
    u.epi.alpha = 1.0f;
    u.epi.nin = 1;
    u.epi.in[0] = epi_in(B.xf, IN_F32, B.ldx, xs, a);
    if (it + 1 < steps) {
      const bool next_tf = it + 1 >= steps - tf32_tail;
      const int nxt = cur ^ 1;
      u.epi.nout = 2;
      u.epi.out[0] = epi_out(B.xf, OUT_F32, B.ldx, xs);
      u.epi.out[1] = next_tf ? epi_out(B.xt[nxt], OUT_TF32, B.ldx, xs) : epi_out(B.xb[nxt], OUT_BF16, B.ldx, xs);
    } else {
      u.epi.nout = 1;
      u.epi.out[0] = epi_out(out, out_kind_of(dtype), out_ld, out_bstride, trans);
    }
    if ((r = launch_gemm(u, s))) return r;
    cur ^= 1;
  }
  return PO_OK;
}
