// Newton–Schulz orthogonalisation on the tensor cores.
//
// Mirrors pytorch_opt/ops/reference.py:71-97 (and the ATen version
// pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:65-81). Per matrix (m = min dim):
//   pack   : X0 = G / (||G||_F + eps), kept in G's orientation
//   iterate: A = X X^T          (symmetric: lower tiles only, mirrored)
//            B = b A + c A A    (symmetric: lower tiles only, A A = A A^T)
//            X = a X + B X      (fp32 master copy of X updated in place)
//   the last update writes the caller's output directly (cast to its dtype).
// Tall G (rows > cols): the reference transposes, iterates and transposes
// back; since B is symmetric that equals iterating X (n x m) from the
// right, A = X^T X, B = b A + c A A, X = a X + X B, which is what runs here:
// no matrix is ever transposed, every epilogue access is row-contiguous, and
// the update reads X K-major.
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
#include <cstdlib>

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
  float* adiag;             // diag(A) of the current step, fp32 [batch][m]
  float* scale;             // per matrix: 1 / (||G||_F + eps), then its square ([2][batch])
  double* sums;             // per-matrix sum of squares
  unsigned int* sched;      // tile queue of the products
  long long ldx, ldm, msz;  // msz: elements of one [batch][m][ldm] array
  // Grouped steps (grouped_shape): bf16 zero-diagonal operands of P^2 and of
  // the running product Q (ping-pong), and the second diagonals.
  __nv_bfloat16* fp2;
  __nv_bfloat16* fq[2];
  float* adiag2;            // diag of the other A operand (A ping-pongs between a_hi and a_lo)
  float* bdiag2;            // diag of the other B (P = a I + B ping-pongs between b_hi and b_lo)
  float* p2diag;
  float* qdiag[2];
};

// Shapes whose steps run in groups (see ns_core): far from square, so that
// one tall product per group and a few m x m products cost less than a tall
// Gram and update per step.
inline bool grouped_shape(long long rows, long long cols) {
  const long long m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  return m >= 256 && n >= 2 * m;
}

// X is kept in G's orientation: [rows][ldx], ldx = cols rounded up to 64.
void ns_layout(Arena& ar, long long batch, long long rows, long long cols, bool split, NsBuffers& B) {
  const long long m = rows < cols ? rows : cols;
  B.ldx = round_up(cols, 64);
  B.ldm = round_up(m, 64);
  const size_t xs = static_cast<size_t>(batch * rows * B.ldx);
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
  B.adiag = static_cast<float*>(ar.take(static_cast<size_t>(batch * m) * 4));
  B.scale = static_cast<float*>(ar.take(static_cast<size_t>(batch) * 8));
  B.sums = static_cast<double*>(ar.take(static_cast<size_t>(batch) * 8));
  B.sched = take_sched(ar);
  B.fp2 = B.fq[0] = B.fq[1] = nullptr;
  B.adiag2 = B.bdiag2 = B.p2diag = B.qdiag[0] = B.qdiag[1] = nullptr;
  if (grouped_shape(rows, cols)) {
    B.fp2 = static_cast<__nv_bfloat16*>(ar.take(ms * 2));
    for (int i = 0; i < 2; ++i) B.fq[i] = static_cast<__nv_bfloat16*>(ar.take(ms * 2));
    const size_t vs = static_cast<size_t>(batch * m) * 4;
    B.adiag2 = static_cast<float*>(ar.take(vs));
    B.bdiag2 = static_cast<float*>(ar.take(vs));
    B.p2diag = static_cast<float*>(ar.take(vs));
    for (int i = 0; i < 2; ++i) B.qdiag[i] = static_cast<float*>(ar.take(vs));
  }
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

// scale[b] = 1 / (sqrt(sums[b]) + eps), scale[batch + b] = scale[b]^2 (the
// reference's pre-normalisation, reference.py:90, as a device-side factor).
__global__ void ns_scale_kernel(const double* sums, float eps, float* scale, int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const float sc = 1.0f / (static_cast<float>(sqrt(sums[b])) + eps);
  scale[b] = sc;
  scale[batch + b] = sc * sc;
}

}  // namespace

// Muon's in-place parameter update applied by the last product's epilogue
// (see Epilogue::mu_p). p: [batch][rows][cols], pitch ld, batch pitch bs.
struct NsApply {
  void* p = nullptr;
  int dtype = PO_BF16;
  long long ld = 0, bs = 0;
  float decay = 1.0f;
  float lr_eff = 0.0f;
  double* sq = nullptr;
};

struct NsOptions {
  const double* sums = nullptr;  // per-matrix ||G||_F^2 already computed (nullable)
  const NsApply* apply = nullptr;
};

int ns_core(const void* G, int dtype, long long batch, long long rows, long long cols, long long ld,
            long long bstride, void* out, long long out_ld, long long out_bstride, int steps, float a, float b,
            float c, float eps, int tf32_tail, void* workspace, size_t workspace_bytes, cudaStream_t s,
            const NsOptions& opt);

}  // namespace po

using namespace po;

extern "C" size_t po_ns_workspace_bytes(long long batch, long long rows, long long cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  const long long m = rows < cols ? rows : cols;
  Arena ar(nullptr, 0);
  NsBuffers B;
  ns_layout(ar, batch, rows, cols, m < kSplitBelow, B);
  return ar.used + 256;
}

extern "C" int po_newton_schulz(const void* G, int dtype, long long batch, long long rows, long long cols,
                                long long ld, long long bstride, void* out, long long out_ld, long long out_bstride,
                                int steps, float a, float b, float c, float eps, int tf32_tail, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return po::ns_core(G, dtype, batch, rows, cols, ld, bstride, out, out_ld, out_bstride, steps, a, b, c, eps,
                     tf32_tail, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), po::NsOptions{});
}

namespace po {

// The Newton-Schulz driver. With opt.sums the per-matrix squared norms are
// given (the fused Muon step computes them with the momentum); with
// opt.apply the last product updates the parameters in place (out, if not
// null, still receives the orthogonalised matrix). When G is bf16 with
// 16-byte aligned pitches and the step runs bf16 products, step 0 reads G
// itself as its operands and addend (transposed views for tall matrices)
// and applies the normalisation as device-side per-matrix factors of the
// epilogues: no packed copy of G is made.
int ns_core(const void* G, int dtype, long long batch, long long rows, long long cols, long long ld,
            long long bstride, void* out, long long out_ld, long long out_bstride, int steps, float a, float b,
            float c, float eps, int tf32_tail, void* workspace, size_t workspace_bytes, cudaStream_t s,
            const NsOptions& opt) {
  if (dtype != PO_F32 && dtype != PO_BF16 && dtype != PO_F16 && dtype != PO_F64)
    return set_error(PO_ERR_ARG, "newton_schulz: dtype must be fp32, bf16, fp16 or fp64");
  if (batch < 0 || rows < 0 || cols < 0 || steps < 0)
    return set_error(PO_ERR_ARG, "newton_schulz: negative size or step count");
  if (batch == 0 || rows == 0 || cols == 0) return PO_OK;
  if (G == nullptr || (out == nullptr && opt.apply == nullptr)) return set_error(PO_ERR_ARG, "newton_schulz: null pointer");
  if (ld < cols || (out != nullptr && out_ld < cols))
    return set_error(PO_ERR_ARG, "newton_schulz: row pitch smaller than cols");
  if (batch > 65535) return set_error(PO_ERR_ARG, "newton_schulz: batch too large (max 65535)");

  const bool tall = rows > cols;
  const long long m = tall ? cols : rows, n = tall ? rows : cols;
  if (m > 0x7fffffffLL / 2 || n > 0x7fffffffLL / 2) return set_error(PO_ERR_ARG, "newton_schulz: matrix too large");
  // Precision schedule.
  const bool split = tf32_tail < 0 && m < kSplitBelow;
  if (tf32_tail < 0) tf32_tail = 0;
  if (tf32_tail > steps) tf32_tail = steps;
  auto prec_of = [&](int it) -> Prec {
    if (split) return P_SPLIT;
    return it >= steps - tf32_tail ? P_TF32 : P_BF16;
  };
  if (opt.apply != nullptr && steps == 0)
    return set_error(PO_ERR_UNSUPPORTED, "newton_schulz: a fused update needs at least one step");

  Arena ar(workspace, workspace_bytes);
  NsBuffers B;
  ns_layout(ar, batch, rows, cols, split, B);
  if (workspace == nullptr || ar.overflow())
    return set_error(PO_ERR_WORKSPACE, "newton_schulz: workspace too small (query po_ns_workspace_bytes)");

  int r;
  if ((r = zero_sched(B.sched, s))) return r;
  AnyMat src{G, dtype, rows, cols, ld, bstride};
  const double* sums = opt.sums;
  if (sums == nullptr) {
    if ((r = check_cuda(cudaMemsetAsync(B.sums, 0, static_cast<size_t>(batch) * 8, s), "memset"))) return r;
    if ((r = launch_sumsq(src, static_cast<int>(batch), B.sums, s))) return r;
    sums = B.sums;
  }
  const Prec p0 = prec_of(0);
  const bool direct = dtype == PO_BF16 && p0 == P_BF16 && steps > 0 && reinterpret_cast<uintptr_t>(G) % 16 == 0 &&
                      (ld * 2) % 16 == 0 && (batch == 1 || (bstride * 2) % 16 == 0);
  if (direct) {
    ns_scale_kernel<<<cdiv(batch, 128), 128, 0, s>>>(sums, eps, B.scale, static_cast<int>(batch));
    if ((r = check_cuda(cudaGetLastError(), "ns scale"))) return r;
  } else {
    if ((r = launch_ns_pack(src, static_cast<int>(batch), false, sums, eps, B.xf,
                            p0 == P_TF32 ? static_cast<void*>(B.xt[0]) : static_cast<void*>(B.xb[0]),
                            p0 == P_SPLIT ? static_cast<void*>(B.xl[0]) : nullptr, p0 == P_TF32 ? OUT_TF32 : OUT_BF16,
                            B.ldx, rows, cols, s)))
      return r;
    if (steps == 0)
      return launch_copy_out(B.xf, B.ldx, rows * B.ldx, static_cast<int>(batch), rows, cols, false, out, dtype, out_ld,
                             out_bstride, s);
  }

  const long long xs = rows * B.ldx, ms = m * B.ldm;
  // Operand arrays of A and B: fp32 for tf32 steps, else bf16 hi then bf16 lo.
  char* a_hi = B.aop;
  char* a_lo = B.aop + B.msz * 2;
  char* b_hi = B.bop;
  char* b_lo = B.bop + B.msz * 2;
  // G itself as the step-0 operand and addend (X0 = G / ||G||).
  MatView gv;
  gv.ptr = G;
  gv.dtype = PO_BF16;
  gv.rows = rows;
  gv.cols = cols;
  gv.ld = ld;
  gv.bstride = bstride;
  // Grouped steps. For a matrix far from square, the steps of a group share
  // one tall Gram and one tall update: with A_0 = X^T X (tall; X X^T wide) and
  // P_j = a I + b A_j + c A_j^2, the next Gram is A_{j+1} = A_j P_j^2 (P_j is a
  // polynomial in A_j) and the group's update is X <- X P_0 P_1 ... (P_j ...
  // X for wide matrices), so the steps inside a group cost m x m products
  // only. Groups of three steps, the last group what is left (5 = 3 + 2);
  // every m x m product keeps the diagonal split (operands with zeroed
  // diagonals, the split-product epilogue adds the diagonal terms in fp32).
  // Emulated in bf16 against the fp64 reference on 3584 x 1024 matrices
  // (randn and a k^-1/2 spectrum): 5.9e-3 and 7.4e-3, against 5.7e-3 and
  // 7.2e-3 for one Gram and update per step. PO_NS_GROUP=0 in the
  // environment runs one Gram and update per step (for measurement).
  const char* grp_env = getenv("PO_NS_GROUP");
  const bool grouping = !split && tf32_tail == 0 && B.fp2 != nullptr && !(grp_env != nullptr && grp_env[0] == '0');
  auto group_at = [&](int it) -> int {
    if (!grouping) return 1;
    const int left = steps - it;
    return left >= 3 ? 3 : left;
  };
  auto bview = [&](const void* ptr) { return view(ptr, PO_BF16, m, m, B.ldm); };
  int cur = 0;
  for (int it = 0; it < steps;) {
    const Prec pr = prec_of(it);
    const int gsz = group_at(it);
    const int it_next = it + gsz;
    const bool from_g = direct && it == 0;
    OpView X = pr == P_TF32 ? op_view(pr, B.xt[cur], nullptr, rows, cols, B.ldx)
                            : op_view(pr, B.xb[cur], B.xl[cur], rows, cols, B.ldx);
    if (from_g) X.v[0] = X.v[1] = gv;
    const OpView Aop = op_view(pr, a_hi, a_lo, m, m, B.ldm);
    const OpView Bop = op_view(pr, b_hi, b_lo, m, m, B.ldm);
    const bool ds = pr != P_SPLIT;  // diagonal split of the square and the update

    // A = X X^T (wide: X K-major), or X^T X (tall: X read MN-major).
    GemmDesc g;
    set_kind(g, pr);
    g.M = g.N = static_cast<int>(m);
    g.K = static_cast<int>(n);
    g.batch = static_cast<int>(batch);
    g.a[0] = X.v[0]; g.a[1] = X.v[1];
    g.b[0] = X.v[0]; g.b[1] = X.v[1];
    g.a_kmajor = g.b_kmajor = !tall;
    if (from_g) g.epi.alpha_scale = B.scale + batch;  // (G / ||G||) Gram = s^2 (G Gram)
    g.tri = true;
    g.sched = B.sched;
    g.epi.alpha = 1.0f;
    g.epi.mirror_same = 1;
    // The fp32 A is read only as the square's addend, on the square's own
    // (identically shaped) lower-triangle and diagonal tiles: no mirrored copy.
    g.pair = gemm_uses_pair(g) ? 1 : 0;
    g.epi.out[g.epi.nout] = epi_out(B.af, OUT_F32, B.ldm, ms);
    g.epi.out[g.epi.nout++].lower_only = 1;
    if (ds) {
      g.epi.diag_out = B.adiag;
      g.epi.diag_out_bs = m;
    }
    add_op_outputs(g.epi, pr, a_hi, a_lo, B.ldm, ms, ds);
    if ((r = launch_gemm(g, s))) return r;

    // The update's operand: B (one step) or the group's product Q.
    OpView Uop = Bop;
    const float* ucoef = B.bdiag;
    float ubeta = a;
    if (gsz == 1) {
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
        // A A = F F + D A + A D - D^2 with F (the operands) zero on the diagonal,
        // D = diag(A) as the Gram wrote it; one row read of A.
        q.epi.dsym = B.adiag;
        q.epi.dsym_bs = m;
        q.epi.diag_out = B.bdiag;
        q.epi.diag_out_bs = m;
      }
      add_op_outputs(q.epi, pr, b_hi, b_lo, B.ldm, ms, ds);
      if ((r = launch_gemm(q, s))) return r;
    } else {
      // A_j: (FA[ia], dA[ia]) with its fp32 master in af (lower tiles);
      // P_j = a I + B_j: (FP[ip], dP[ip]) with the constant a on the diagonal.
      __nv_bfloat16* FA[2] = {reinterpret_cast<__nv_bfloat16*>(a_hi), reinterpret_cast<__nv_bfloat16*>(a_lo)};
      float* dA[2] = {B.adiag, B.adiag2};
      __nv_bfloat16* FP[2] = {reinterpret_cast<__nv_bfloat16*>(b_hi), reinterpret_cast<__nv_bfloat16*>(b_lo)};
      float* dP[2] = {B.bdiag, B.bdiag2};
      // B_j = b A_j + c A_j A_j (as the one-step square).
      auto square = [&](const __nv_bfloat16* fa, const float* da, __nv_bfloat16* fb, float* db) -> int {
        GemmDesc h;
        set_kind(h, P_BF16);
        h.M = h.N = h.K = static_cast<int>(m);
        h.batch = static_cast<int>(batch);
        h.a[0] = h.a[1] = bview(fa);
        h.b[0] = h.b[1] = bview(fa);
        h.tri = true;
        h.pair = g.pair;
        h.sched = B.sched;
        h.epi.alpha = c;
        h.epi.mirror_same = 1;
        h.epi.nin = 1;
        h.epi.in[0] = epi_in(B.af, IN_F32, B.ldm, ms, b);
        h.epi.dsym = da;
        h.epi.dsym_bs = m;
        h.epi.diag_out = db;
        h.epi.diag_out_bs = m;
        add_op_outputs(h.epi, P_BF16, fb, nullptr, B.ldm, ms, true);
        return launch_gemm(h, s);
      };
      // S T for split symmetric S, T (polynomials in A_j): operands F_S, F_T.
      auto sprod = [&](const __nv_bfloat16* fs, const float* dsv, float ds_add, const __nv_bfloat16* ft,
                       const float* dtv, float dt_add, __nv_bfloat16* fo, float* dout, float* f32_out) -> int {
        GemmDesc h;
        set_kind(h, P_BF16);
        h.M = h.N = h.K = static_cast<int>(m);
        h.batch = static_cast<int>(batch);
        h.a[0] = h.a[1] = bview(fs);
        h.b[0] = h.b[1] = bview(ft);
        h.tri = true;
        h.pair = g.pair;  // af's lower tiles are read by the next square on the same tiling
        h.sched = B.sched;
        h.epi.alpha = 1.0f;
        h.epi.mirror_same = 1;
        h.epi.s2_fs = epi_in(fs, IN_BF16, B.ldm, ms, 0.0f);
        h.epi.s2_ft = epi_in(ft, IN_BF16, B.ldm, ms, 0.0f);
        h.epi.s2_ds = dsv;
        h.epi.s2_dt = dtv;
        h.epi.s2_d_bs = m;
        h.epi.s2_ds_add = ds_add;
        h.epi.s2_dt_add = dt_add;
        if (f32_out != nullptr) {
          h.epi.out[h.epi.nout] = epi_out(f32_out, OUT_F32, B.ldm, ms);
          h.epi.out[h.epi.nout++].lower_only = 1;
        }
        h.epi.diag_out = dout;
        h.epi.diag_out_bs = m;
        add_op_outputs(h.epi, P_BF16, fo, nullptr, B.ldm, ms, true);
        return launch_gemm(h, s);
      };
      int ia = 0, ip = 1, iq = -1;
      for (int j = 0; j < gsz; ++j) {
        const int ipn = ip ^ 1;
        if ((r = square(FA[ia], dA[ia], FP[ipn], dP[ipn]))) return r;
        if (j >= 1) {
          const int iqn = iq < 0 ? 0 : iq ^ 1;
          if (j == 1) r = sprod(FP[ip], dP[ip], a, FP[ipn], dP[ipn], a, B.fq[iqn], B.qdiag[iqn], nullptr);
          else r = sprod(B.fq[iq], B.qdiag[iq], 0.0f, FP[ipn], dP[ipn], a, B.fq[iqn], B.qdiag[iqn], nullptr);
          if (r) return r;
          iq = iqn;
        }
        if (j + 1 < gsz) {
          if ((r = sprod(FP[ipn], dP[ipn], a, FP[ipn], dP[ipn], a, B.fp2, B.p2diag, nullptr))) return r;
          if ((r = sprod(FA[ia], dA[ia], 0.0f, B.fp2, B.p2diag, 0.0f, FA[ia ^ 1], dA[ia ^ 1], B.af))) return r;
          ia ^= 1;
        }
        ip = ipn;
      }
      Uop.v[0] = Uop.v[1] = bview(B.fq[iq]);
      ucoef = B.qdiag[iq];
      ubeta = 0.0f;
    }

    // Wide: X = a X + B X (B operand X stored [K = m][N = n], MN-major).
    // Tall: X = a X + X B (A operand X [n][K = m], K-major; B symmetric).
    GemmDesc u;
    set_kind(u, pr);
    u.batch = static_cast<int>(batch);
    u.K = static_cast<int>(m);
    if (tall) {
      u.M = static_cast<int>(n);
      u.N = static_cast<int>(m);
      u.a[0] = X.v[0]; u.a[1] = X.v[1];
      u.b[0] = Uop.v[0]; u.b[1] = Uop.v[1];
      u.a_kmajor = true;
      u.b_kmajor = true;
    } else {
      u.M = static_cast<int>(m);
      u.N = static_cast<int>(n);
      u.a[0] = Uop.v[0]; u.a[1] = Uop.v[1];
      u.b[0] = X.v[0]; u.b[1] = X.v[1];
      u.b_kmajor = false;
    }
    u.sched = B.sched;
    u.epi.alpha = 1.0f;
    u.epi.nin = 1;
    if (from_g) {
      // s (B G or G B) + s (a + B_jj) G: both terms scaled by s = 1 / ||G||.
      u.epi.alpha_scale = B.scale;
      u.epi.in_scale = B.scale;
      u.epi.in[0] = epi_in(G, IN_BF16, ld, bstride, ubeta);
    } else {
      u.epi.in[0] = epi_in(B.xf, IN_F32, B.ldx, xs, ubeta);
    }
    if (ds) {
      // The dominant diagonal of B goes to the addend exactly: B X = F_B X +
      // diag(B) X (row scale a + B_ii) or X B = X F_B + X diag(B) (column scale).
      if (tall) {
        u.epi.in0_colcoef = ucoef;
        u.epi.in0_colcoef_bs = m;
      } else {
        u.epi.in0_rowcoef = ucoef;
        u.epi.in0_rowcoef_bs = m;
      }
    }
    if (it_next < steps) {
      const Prec pn = prec_of(it_next);
      const int nxt = cur ^ 1;
      u.epi.out[u.epi.nout++] = epi_out(B.xf, OUT_F32, B.ldx, xs);
      if (pn == P_TF32) add_op_outputs(u.epi, pn, B.xt[nxt], nullptr, B.ldx, xs);
      else add_op_outputs(u.epi, pn, B.xb[nxt], B.xl[nxt], B.ldx, xs);
    } else {
      if (out != nullptr) u.epi.out[u.epi.nout++] = epi_out(out, out_kind_of(dtype), out_ld, out_bstride);
      if (opt.apply != nullptr) {
        const NsApply& ap = *opt.apply;
        u.epi.mu_p = ap.p;
        u.epi.mu_ld = ap.ld;
        u.epi.mu_bs = ap.bs;
        u.epi.mu_bf16 = ap.dtype == PO_BF16 ? 1 : 0;
        const int es = ap.dtype == PO_BF16 ? 2 : 4;
        u.epi.mu_vec = reinterpret_cast<uintptr_t>(ap.p) % 16 == 0 && (ap.ld * es) % 16 == 0 && (ap.bs * es) % 16 == 0;
        u.epi.mu_use_decay = ap.decay != 1.0f;
        u.epi.mu_decay = ap.decay;
        // add_(O, alpha=-lr_eff) on a bf16 tensor rounds alpha to bf16 first.
        u.epi.mu_alpha = ap.dtype == PO_BF16 ? __bfloat162float(__float2bfloat16_rn(-ap.lr_eff)) : -ap.lr_eff;
        u.epi.red_sumsq = ap.sq;
        u.epi.red_sumsq_shared = 1;
      }
    }
    if ((r = launch_gemm(u, s))) return r;
    cur ^= 1;
    it = it_next;
  }
  return PO_OK;
}

}  // namespace po

using namespace po;

extern "C" size_t po_muon_step_workspace_bytes(long long batch, long long rows, long long cols, int dtype) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  const long long es = dtype == PO_BF16 ? 2 : 4;
  return static_cast<size_t>(round_up(batch * rows * cols * es, 256) + round_up(batch * 8, 256)) +
         po_ns_workspace_bytes(batch, rows, cols) + 256;
}

extern "C" int po_muon_step(const void* g, void* buf, void* p, int dtype, long long batch, long long rows,
                            long long cols, float momentum, int nesterov, int ns_steps, float a, float b, float c,
                            float eps, float lr_eff, float decay, double* sq_sum, void* o_out, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (dtype != PO_BF16 && dtype != PO_F32) return set_error(PO_ERR_ARG, "muon_step: dtype must be fp32 or bf16");
  if (batch < 0 || rows < 0 || cols < 0 || ns_steps < 0) return set_error(PO_ERR_ARG, "muon_step: negative size");
  if (batch == 0 || rows == 0 || cols == 0) return PO_OK;
  if (!g || !buf || !p) return set_error(PO_ERR_ARG, "muon_step: null pointer");
  if (batch > 65535) return set_error(PO_ERR_ARG, "muon_step: batch too large (max 65535)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long per = rows * cols, es = dtype == PO_BF16 ? 2 : 4;
  Arena ar(workspace, workspace_bytes);
  void* u = ar.take(static_cast<size_t>(batch * per * es));
  auto* sums = static_cast<double*>(ar.take(static_cast<size_t>(batch) * 8));
  const size_t ns_bytes = po_ns_workspace_bytes(batch, rows, cols);
  void* ns_ws = ar.take(ns_bytes);
  if (workspace == nullptr || ar.overflow())
    return set_error(PO_ERR_WORKSPACE, "muon_step: workspace too small (query po_muon_step_workspace_bytes)");
  int r = check_cuda(cudaMemsetAsync(sums, 0, static_cast<size_t>(batch) * 8, s), "memset");
  if (r) return r;
  if ((r = launch_momentum_sumsq(g, buf, u, dtype, batch, per, momentum, nesterov, sums, s))) return r;
  if (ns_steps == 0) {
    // O is the normalised u itself: write it over u, then the separate update pass.
    NsOptions opt;
    opt.sums = sums;
    if ((r = ns_core(u, dtype, batch, rows, cols, cols, per, u, cols, per, 0, a, b, c, eps, -1, ns_ws, ns_bytes, s,
                     opt)))
      return r;
    if (o_out != nullptr &&
        (r = check_cuda(cudaMemcpyAsync(o_out, u, static_cast<size_t>(batch * per * es), cudaMemcpyDeviceToDevice, s),
                        "copy")))
      return r;
    return po_muon_apply(p, u, dtype, batch * per, lr_eff, decay, sq_sum, stream);
  }
  NsApply ap;
  ap.p = p;
  ap.dtype = dtype;
  ap.ld = cols;
  ap.bs = per;
  ap.decay = decay;
  ap.lr_eff = lr_eff;
  ap.sq = sq_sum;
  NsOptions opt;
  opt.sums = sums;
  opt.apply = &ap;
  return ns_core(u, dtype, batch, rows, cols, cols, per, o_out, cols, per, ns_steps, a, b, c, eps, -1, ns_ws,
                 ns_bytes, s, opt);
}
