// Symmetric rank-k factor updates on the tensor cores:
//   * Kronecker factors of Shampoo/SOAP (pytorch_opt/ops/reference.py:100-114,
//     ATen version pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:83-94):
//       L <- beta2 L + (1 - beta2) G G^T,   R <- beta2 R + (1 - beta2) G^T G
//   * KFAC factor statistics with the EMA fused
//     (pytorch_opt/curvature/kron.py:95-113):
//       F <- first ? alpha X^T X : beta F + (1 - beta) alpha X^T X
// Only the lower triangle of 128x128 tiles is computed; the epilogue applies
// the update to both (i, j) and (j, i), each with its own old value, so the
// result equals the reference's elementwise update of a full square.
// bf16 inputs are used directly (their products are exact in fp32); fp32
// inputs are split into tf32 hi/lo pairs (hi*hi + hi*lo + lo*hi on the tf32
// tensor cores, ~2^-21 relative: fp32-grade factors, whose small eigenvalues
// the reference's eigh-based roots and bases depend on). Long K loops are
// summed in chunks outside the truncating accumulator.
#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {
namespace {

// K length above which the products are summed in chunks.
constexpr long long kChunkAboveK = 2048;

struct Operand {
  MatView v[2];
  int npass;
  int kind;  // KIND_BF16 (bf16 input) or KIND_TF32 (split fp32 input)
};

inline bool tma_aligned(const void* p, long long ld, int es) {
  return reinterpret_cast<uintptr_t>(p) % 16 == 0 && (ld * es) % 16 == 0;
}

// Bytes of staging needed for a rows x cols matrix of dtype `dt` (0 when it
// can be used in place).
size_t stage_bytes(const void* p, int dt, long long rows, long long cols, long long ld) {
  const long long pld = round_up(cols, 64);
  if (dt == PO_F32) return static_cast<size_t>(rows * pld) * 8;  // tf32 hi + lo
  if (p != nullptr && tma_aligned(p, ld, 2)) return 0;
  return static_cast<size_t>(rows * pld) * 2;
}

// Prepare a [rows][cols] matrix as tensor-core operand(s).
int prepare(const void* X, int dt, long long rows, long long cols, long long ld, Arena& ar, Operand& op,
            cudaStream_t s) {
  const long long pld = round_up(cols, 64);
  AnyMat am{X, dt, rows, cols, ld, rows * ld};
  auto set = [&](MatView& v, const void* ptr, long long l, int dtype) {
    v.ptr = ptr;
    v.dtype = dtype;
    v.rows = rows;
    v.cols = cols;
    v.ld = l;
    v.bstride = rows * l;
  };
  if (dt == PO_F32) {
    auto* hi = static_cast<float*>(ar.take(static_cast<size_t>(rows * pld) * 4));
    auto* lo = static_cast<float*>(ar.take(static_cast<size_t>(rows * pld) * 4));
    if (ar.overflow()) return set_error(PO_ERR_WORKSPACE, "factor update: workspace too small");
    int r = launch_split_tf32(am, 1, hi, lo, pld, rows * pld, s);
    if (r) return r;
    set(op.v[0], hi, pld, PO_F32);
    set(op.v[1], lo, pld, PO_F32);
    op.npass = 3;
    op.kind = KIND_TF32;
    return PO_OK;
  }
  op.kind = KIND_BF16;
  if (dt != PO_BF16) return set_error(PO_ERR_ARG, "factor update: input dtype must be fp32 or bf16");
  if (tma_aligned(X, ld, 2)) {
    set(op.v[0], X, ld, PO_BF16);
  } else {
    auto* c = static_cast<__nv_bfloat16*>(ar.take(static_cast<size_t>(rows * pld) * 2));
    if (ar.overflow()) return set_error(PO_ERR_WORKSPACE, "factor update: workspace too small");
    int r = launch_convert(am, 1, c, PO_BF16, pld, rows * pld, s);
    if (r) return r;
    set(op.v[0], c, pld, PO_BF16);
  }
  op.v[1] = op.v[0];
  op.npass = 1;
  return PO_OK;
}

// F (d x d fp32, pitch f_ld) <- alpha_acc * (X X^T or X^T X) + beta * F.
// `gram_of_rows`: product over the columns of X (X X^T, K-major operands);
// otherwise over its rows (X^T X, MN-major operands).
int syrk_update(float* F, long long f_ld, const Operand& op, bool gram_of_rows, long long d, long long K,
                float alpha_acc, float beta, unsigned int* sched, cudaStream_t s, double* trace = nullptr) {
  GemmDesc g;
  g.sched = sched;
  g.kind = op.kind;
  g.M = g.N = static_cast<int>(d);
  g.K = static_cast<int>(K);
  g.batch = 1;
  g.a[0] = op.v[0];
  g.a[1] = op.v[1];
  g.b[0] = op.v[0];
  g.b[1] = op.v[1];
  g.a_kmajor = g.b_kmajor = gram_of_rows;
  g.npass = op.npass;
  g.tri = true;
  g.chunked = K * op.npass > (op.kind == KIND_TF32 ? kChunkAboveK / 2 : kChunkAboveK);
  g.epi.alpha = alpha_acc;
  if (beta != 0.0f) {
    g.epi.nin = 1;
    g.epi.in[0] = epi_in(F, IN_F32, f_ld, d * f_ld, beta);
  }
  g.epi.nout = 1;
  g.epi.out[0] = epi_out(F, OUT_F32, f_ld, d * f_ld);
  g.epi.red_trace = trace;
  g.epi.sym_diag = op.npass > 1 ? 1 : 0;  // split passes: make diagonal tiles bit-symmetric
  return launch_gemm(g, s);
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" size_t po_kron_workspace_bytes(long long m, long long n, int g_dtype) {
  if (m <= 0 || n <= 0) return 0;
  return stage_bytes(nullptr, g_dtype, m, n, 0) + 512;
}

extern "C" int po_kron_factor_update(float* L, long long l_ld, float* R, long long r_ld, const void* G, int g_dtype,
                                     long long m, long long n, long long g_ld, double beta2, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (m < 0 || n < 0) return set_error(PO_ERR_ARG, "kron_factor_update: negative size");
  if (m == 0 || n == 0) return PO_OK;
  if (L == nullptr || R == nullptr || G == nullptr) return set_error(PO_ERR_ARG, "kron_factor_update: null pointer");
  if (l_ld < m || r_ld < n || g_ld < n) return set_error(PO_ERR_ARG, "kron_factor_update: pitch too small");
  if (m > 0x3fffffff || n > 0x3fffffff) return set_error(PO_ERR_ARG, "kron_factor_update: size too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (workspace == nullptr) return set_error(PO_ERR_WORKSPACE, "kron_factor_update: workspace required");
  Arena ar(workspace, workspace_bytes);
  unsigned int* sched = take_sched(ar);
  if (ar.overflow()) return set_error(PO_ERR_WORKSPACE, "workspace too small (query its *_workspace_bytes)");
  Operand op;
  int r = prepare(G, g_dtype, m, n, g_ld, ar, op, s);
  if (r) return r;
  if ((r = zero_sched(sched, s))) return r;
  // beta2 == 1: plain sums (reference adds G G^T without scaling).
  const float keep = beta2 == 1.0 ? 1.0f : static_cast<float>(beta2);
  const float add = beta2 == 1.0 ? 1.0f : static_cast<float>(1.0 - beta2);
  if ((r = syrk_update(L, l_ld, op, /*gram_of_rows=*/true, m, n, add, keep, sched, s))) return r;
  return syrk_update(R, r_ld, op, /*gram_of_rows=*/false, n, m, add, keep, sched, s);
}

extern "C" size_t po_syrk_workspace_bytes(long long rows, long long d, int x_dtype) {
  if (rows <= 0 || d <= 0) return 0;
  return stage_bytes(nullptr, x_dtype, rows, d, 0) + 512;
}

extern "C" int po_syrk_ema(float* F, long long d, long long f_ld, const void* X, int x_dtype, long long rows,
                           long long x_ld, double alpha, double beta, int first, double* trace, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (d < 0 || rows < 0) return set_error(PO_ERR_ARG, "syrk_ema: negative size");
  if (d == 0) return PO_OK;
  if (F == nullptr || (rows > 0 && X == nullptr)) return set_error(PO_ERR_ARG, "syrk_ema: null pointer");
  if (f_ld < d || x_ld < d) return set_error(PO_ERR_ARG, "syrk_ema: pitch too small");
  if (d > 0x3fffffff || rows > 0x3fffffff) return set_error(PO_ERR_ARG, "syrk_ema: size too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    // Empty batch: the statistic is the zero matrix.
    if (!first) return set_error(PO_ERR_UNSUPPORTED, "syrk_ema: EMA with an empty batch");
    if (trace != nullptr) {
      const int r = check_cuda(cudaMemsetAsync(trace, 0, sizeof(double), s), "memset");
      if (r) return r;
    }
    return check_cuda(cudaMemset2DAsync(F, f_ld * 4, 0, d * 4, d, s), "memset");
  }
  if (workspace == nullptr) return set_error(PO_ERR_WORKSPACE, "syrk_ema: workspace required");
  Arena ar(workspace, workspace_bytes);
  unsigned int* sched = take_sched(ar);
  if (ar.overflow()) return set_error(PO_ERR_WORKSPACE, "workspace too small (query its *_workspace_bytes)");
  Operand op;
  int r = prepare(X, x_dtype, rows, d, x_ld, ar, op, s);
  if (r) return r;
  if ((r = zero_sched(sched, s))) return r;
  if (trace != nullptr && (r = check_cuda(cudaMemsetAsync(trace, 0, sizeof(double), s), "memset"))) return r;
  const float a = first ? static_cast<float>(alpha) : static_cast<float>((1.0 - beta) * alpha);
  const float b = first ? 0.0f : static_cast<float>(beta);
  return syrk_update(F, f_ld, op, /*gram_of_rows=*/false, d, rows, a, b, sched, s, trace);
}
