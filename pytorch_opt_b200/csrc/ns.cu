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
//
// Precision. All products accumulate in fp32. By default (m >= 256) every
// step runs bf16 tensor-core products with the diagonal split: A and B have
// diagonals that dominate their rows (A ~ X X^T, B ~ b A + c A^2 near the
// identity's multiples), and rounding a dominant diagonal to bf16 puts a
// random diagonal perturbation of ~2^-9 |A_ii| into every singular
// direction, the small ones included. So the operand copies of A and B carry
// zeroed diagonals and the epilogues add the diagonal terms exactly in fp32:
//   A A = F F + D A + A D - D^2       (F: A off the diagonal, D = diag(A))
//   B X = F_B X + D_B X               (D_B X: a per-row scale of the fp32 X
//                                      addend, a X + D_B X = (a + B_ii) X_ij)
// The square writes diag(B) (fp32) for the update's epilogue. Measured in a
// CPU emulation against the fp32 reference: 2.3e-3 .. 6.3e-3 relative
// Frobenius error over shapes 64x100 .. 4096^2 (randn, 1/k spectra,
// low-rank + noise), against 1.0e-2 .. 2.5e-2 for plain bf16 steps.
// `tf32_tail` >= 0 runs that many final steps on tf32 products instead (also
// with the split). Matrices with m < 256 run every step on split-bf16 pairs
// (hi*hi + hi*lo + lo*hi) with chunked accumulation, which keeps even long
// or oscillating schedules close to the fp32 reference.
#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {

namespace {

enum Prec : int { P_BF16 = 0, P_TF32 = 1, P_SPLIT = 2 };

// m below which the automatic schedule uses split-bf16 on every step.
constexpr long long kSplitBelow = 256;

struct NsBuffers {
  float* xf;                // fp32 master X            [batch][m][ldx]
  __nv_bfloat16* xb[2];     // bf16 (hi) operand copies of X (ping-pong)
  __nv_bfloat16* xl[2];     // bf16 lo halves for split steps (allocated only when used)
  float* xt[2];             // tf32-rounded operand copies of X (ping-pong)
  float* af;                // fp32 A = X X^T           [batch][m][ldm]
  char* aop;                // A as product operand: fp32 (tf32) or bf16 hi | bf16 lo
  char* bop;                // B as product operand, same layout
  float* bdiag;             // diag(B) of the current step, fp32 [batch][m]
  double* sums;             // per-matrix sum of squares
  unsigned int* sched;      // tile queue of the products
  long long ldx, ldm, msz;  // msz: elements of one [batch][m][ldm] array
};

void ns_layout(Arena& ar, long long batch, long long m, long long n, bool split, NsBuffers& B) {
  B.ldx = round_up(n, 64);
  B.ldm = round_up(m, 64);
  const size_t xs = static_cast<size_t>(batch * m * B.ldx);
  B.msz = batch * m * B.ldm;
  const size_t ms = static_cast<size_t>(B.msz);
  B.xf = static_cast<float*>(ar.take(xs * 4));
  for (int i = 0; i < 2; ++i) B.xb[i] = static_cast<__nv_bfloat16*>(ar.take(xs * 2));
  for (int i = 0; i < 2; ++i) B.xl[i] = split ? static_cast<__nv_bfloat16*>(ar.take(xs * 2)) : nullptr;
  for (int i = 0; i < 2; ++i) B.xt[i] = static_cast<float*>(ar.take(xs * 4));
  B.af = static_cast<float*>(ar.take(ms * 4));
  B.aop = static_cast<char*>(ar.take(ms * 4));
  B.bop = static_cast<char*>(ar.take(ms * 4));
  B.bdiag = static_cast<float*>(ar.take(static_cast<size_t>(batch * m) * 4));
  B.sums = static_cast<double*>(ar.take(static_cast<size_t>(batch) * 8));
  B.sched = take_sched(ar);
}

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

// Operand views (hi, lo) of a product operand stored with precision `pr`.
struct OpView {
  MatView v[2];
};
OpView op_view(Prec pr, const void* hi, const void* lo, long long rows, long long cols, long long ld) {
  OpView o;
  if (pr == P_TF32) {
    o.v[0] = view(hi, PO_F32, rows, cols, ld);
    o.v[1] = o.v[0];
  } else {
    o.v[0] = view(hi, PO_BF16, rows, cols, ld);
    o.v[1] = pr == P_SPLIT ? view(lo, PO_BF16, rows, cols, ld) : o.v[0];
  }
  return o;
}

// Append the epilogue outputs that write an operand of precision `pr`
// (zero_diag: the diagonal is stored as 0, for the diagonal split).
void add_op_outputs(Epilogue& e, Prec pr, void* hi, void* lo, long long ld, long long bs, bool zero_diag = false) {
  const int first = e.nout;
  if (pr == P_TF32) {
    e.out[e.nout++] = epi_out(hi, OUT_TF32, ld, bs);
  } else {
    e.out[e.nout++] = epi_out(hi, OUT_BF16, ld, bs);
    if (pr == P_SPLIT) e.out[e.nout++] = epi_out(lo, OUT_BF16_LO, ld, bs);
  }
  for (int i = first; i < e.nout; ++i) e.out[i].zero_diag = zero_diag ? 1 : 0;
}

void set_kind(GemmDesc& g, Prec pr) {
  g.kind = pr == P_TF32 ? KIND_TF32 : KIND_BF16;
  g.npass = pr == P_SPLIT ? 3 : 1;
  g.chunked = pr == P_SPLIT;
}

}  // namespace

}  // namespace po

using namespace po;

extern "C" size_t po_ns_workspace_bytes(long long batch, long long rows, long long cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  const long long m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  Arena ar(nullptr, 0);
  NsBuffers B;
  ns_layout(ar, batch, m, n, m < kSplitBelow, B);
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const bool trans = rows > cols;
  const long long m = trans ? cols : rows, n = trans ? rows : cols;
  if (m > 0x7fffffffLL / 2 || n > 0x7fffffffLL / 2) return set_error(PO_ERR_ARG, "newton_schulz: matrix too large");
  // Precision schedule.
  const bool split = tf32_tail < 0 && m < kSplitBelow;
  if (tf32_tail < 0) tf32_tail = 0;
  if (tf32_tail > steps) tf32_tail = steps;
  auto prec_of = [&](int it) -> Prec {
    if (split) return P_SPLIT;
    return it >= steps - tf32_tail ? P_TF32 : P_BF16;
  };

  Arena ar(workspace, workspace_bytes);
  NsBuffers B;
  ns_layout(ar, batch, m, n, split, B);
  if (workspace == nullptr || ar.overflow())
    return set_error(PO_ERR_WORKSPACE, "newton_schulz: workspace too small (query po_ns_workspace_bytes)");

  int r = check_cuda(cudaMemsetAsync(B.sums, 0, static_cast<size_t>(batch) * 8, s), "memset");
  if (r) return r;
  if ((r = zero_sched(B.sched, s))) return r;
  AnyMat src{G, dtype, rows, cols, ld, bstride};
  if ((r = launch_sumsq(src, static_cast<int>(batch), B.sums, s))) return r;
  const Prec p0 = prec_of(0);
  if ((r = launch_ns_pack(src, static_cast<int>(batch), trans, B.sums, eps, B.xf,
                          p0 == P_TF32 ? static_cast<void*>(B.xt[0]) : static_cast<void*>(B.xb[0]),
                          p0 == P_SPLIT ? static_cast<void*>(B.xl[0]) : nullptr, p0 == P_TF32 ? OUT_TF32 : OUT_BF16,
                          B.ldx, m, n, s)))
    return r;
  if (steps == 0)
    return launch_copy_out(B.xf, B.ldx, m * B.ldx, static_cast<int>(batch), m, n, trans, out, dtype, out_ld,
                           out_bstride, s);

  const long long xs = m * B.ldx, ms = m * B.ldm;
  // Operand arrays of A and B: fp32 for tf32 steps, else bf16 hi then bf16 lo.
  char* a_hi = B.aop;
  char* a_lo = B.aop + B.msz * 2;
  char* b_hi = B.bop;
  char* b_lo = B.bop + B.msz * 2;
  int cur = 0;
  for (int it = 0; it < steps; ++it) {
    const Prec pr = prec_of(it);
    const OpView X = pr == P_TF32 ? op_view(pr, B.xt[cur], nullptr, m, n, B.ldx)
                                  : op_view(pr, B.xb[cur], B.xl[cur], m, n, B.ldx);
    const OpView Aop = op_view(pr, a_hi, a_lo, m, m, B.ldm);
    const OpView Bop = op_view(pr, b_hi, b_lo, m, m, B.ldm);

    // A = X X^T
    GemmDesc g;
    set_kind(g, pr);
    g.M = g.N = static_cast<int>(m);
    g.K = static_cast<int>(n);
    g.batch = static_cast<int>(batch);
    g.a[0] = X.v[0]; g.a[1] = X.v[1];
    g.b[0] = X.v[0]; g.b[1] = X.v[1];
    g.tri = true;
    g.sched = B.sched;
    g.epi.alpha = 1.0f;
    g.epi.mirror_same = 1;
    // The fp32 A is read only as the square's addend, on the square's own
    // (identically shaped) lower-triangle and diagonal tiles: no mirrored copy.
    g.pair = gemm_uses_pair(g) ? 1 : 0;
    g.epi.out[g.epi.nout] = epi_out(B.af, OUT_F32, B.ldm, ms);
    g.epi.out[g.epi.nout++].lower_only = 1;
    const bool ds = pr != P_SPLIT;  // diagonal split of the square and the update
    add_op_outputs(g.epi, pr, a_hi, a_lo, B.ldm, ms, ds);
    if ((r = launch_gemm(g, s))) return r;

    // B = b A + c A A
    GemmDesc q;
    set_kind(q, pr);
    q.M = q.N = q.K = static_cast<int>(m);
    q.batch = static_cast<int>(batch);
    q.a[0] = Aop.v[0]; q.a[1] = Aop.v[1];
    q.b[0] = Aop.v[0]; q.b[1] = Aop.v[1];
    q.tri = true;
    q.pair = g.pair;  // same tiling as the Gram, whose fp32 A holds only those tiles
    q.sched = B.sched;
    q.epi.alpha = c;
    q.epi.mirror_same = 1;  // A is stored exactly symmetric by the Gram's mirrored stores
    q.epi.nin = 1;
    q.epi.in[0] = epi_in(B.af, IN_F32, B.ldm, ms, b);
    if (ds) {
      // A A = F F + D A + A D - D^2 with F (the operands) zero on the diagonal.
      q.epi.diag_split = 1;
      q.epi.dU = epi_in(B.af, IN_F32, B.ldm, ms, 1.0f);
      q.epi.dV = q.epi.dU;
      q.epi.diag_out = B.bdiag;
      q.epi.diag_out_bs = m;
    }
    add_op_outputs(q.epi, pr, b_hi, b_lo, B.ldm, ms, ds);
    if ((r = launch_gemm(q, s))) return r;

    // X = a X + B X ; B operand is X stored [K = m][N = n] (MN-major).
    GemmDesc u;
    set_kind(u, pr);
    u.M = static_cast<int>(m);
    u.N = static_cast<int>(n);
    u.K = static_cast<int>(m);
    u.batch = static_cast<int>(batch);
    u.a[0] = Bop.v[0]; u.a[1] = Bop.v[1];
    u.b[0] = X.v[0]; u.b[1] = X.v[1];
    u.b_kmajor = false;
    u.sched = B.sched;
    u.epi.alpha = 1.0f;
    u.epi.nin = 1;
    u.epi.in[0] = epi_in(B.xf, IN_F32, B.ldx, xs, a);
    if (ds) {
      // B X = F_B X + diag(B) X: the fp32 addend X is scaled by a + B_ii.
      u.epi.in0_rowcoef = B.bdiag;
      u.epi.in0_rowcoef_bs = m;
    }
    if (it + 1 < steps) {
      const Prec pn = prec_of(it + 1);
      const int nxt = cur ^ 1;
      u.epi.out[u.epi.nout++] = epi_out(B.xf, OUT_F32, B.ldx, xs);
      if (pn == P_TF32) add_op_outputs(u.epi, pn, B.xt[nxt], nullptr, B.ldx, xs);
      else add_op_outputs(u.epi, pn, B.xb[nxt], B.xl[nxt], B.ldx, xs);
    } else {
      u.epi.out[u.epi.nout++] = epi_out(out, out_kind_of(dtype), out_ld, out_bstride, trans);
    }
    if ((r = launch_gemm(u, s))) return r;
    cur ^= 1;
  }
  return PO_OK;
}
