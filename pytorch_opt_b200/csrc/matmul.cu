// General batched product C = alpha op(A) op(B) + beta C on the tcgen05 core
// (exported for tests and reused by the two-sided preconditioner).
#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {

// Storage shape of op(X) for a row-major operand: op(X) is r x c; stored
// transposed when `trans`.
struct Stored {
  long long rows, cols;
};
inline Stored stored(long long r, long long c, int trans) { return trans ? Stored{c, r} : Stored{r, c}; }

// Staging area for one operand: 4 bytes per padded element, used either as
// one fp32 / bf16 copy or as a bf16 (hi, lo) pair.
struct Staged {
  char* base;
  long long ld;
  long long elems;  // batch * rows * ld
};

inline Staged stage_layout(Arena& ar, long long batch, Stored st) {
  Staged s;
  s.ld = round_up(st.cols, 64);
  s.elems = batch * st.rows * s.ld;
  s.base = static_cast<char*>(ar.take(static_cast<size_t>(s.elems) * 4));
  return s;
}

inline bool tma_ok(const void* p, long long ld, long long bs, long long batch, int es) {
  return reinterpret_cast<uintptr_t>(p) % 16 == 0 && (ld * es) % 16 == 0 && (batch == 1 || (bs * es) % 16 == 0);
}

// Prepare operand views for the product (direct when aligned, else staged).
// split: fp32 source turned into a bf16 (hi, lo) pair.
inline int prepare_operand(const void* X, int dtype, long long ld, long long bs, Stored st, long long batch,
                           bool split, const Staged& stg, MatView out[2], cudaStream_t s) {
  AnyMat am{X, dtype, st.rows, st.cols, ld, bs};
  if (split) {
    __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(stg.base);
    __nv_bfloat16* lo = hi + stg.elems;
    int r = launch_split_bf16(am, static_cast<int>(batch), hi, lo, stg.ld, st.rows * stg.ld, s);
    if (r) return r;
    const void* ps[2] = {hi, lo};
    for (int i = 0; i < 2; ++i) {
      out[i].ptr = ps[i]; out[i].dtype = PO_BF16; out[i].rows = st.rows; out[i].cols = st.cols;
      out[i].ld = stg.ld; out[i].bstride = st.rows * stg.ld;
    }
    return PO_OK;
  }
  const int es = dtype_size(dtype);
  if (tma_ok(X, ld, bs, batch, es)) {
    out[0].ptr = X; out[0].dtype = dtype; out[0].rows = st.rows; out[0].cols = st.cols; out[0].ld = ld; out[0].bstride = bs;
  } else {
    int r = launch_convert(am, static_cast<int>(batch), stg.base, dtype, stg.ld, st.rows * stg.ld, s);
    if (r) return r;
    out[0].ptr = stg.base; out[0].dtype = dtype; out[0].rows = st.rows; out[0].cols = st.cols;
    out[0].ld = stg.ld; out[0].bstride = st.rows * stg.ld;
  }
  out[1] = out[0];
  return PO_OK;
}

}  // namespace po

using namespace po;

extern "C" size_t po_matmul_workspace_bytes(long long batch, long long M, long long N, long long K, int dtype,
                                            int precision) {
  (void)dtype;
  (void)precision;
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  size_t best = 0;
  for (int ta = 0; ta < 2; ++ta)
    for (int tb = 0; tb < 2; ++tb) {
      Arena ar(nullptr, 0);
      stage_layout(ar, batch, stored(M, K, ta));
      stage_layout(ar, batch, stored(K, N, tb));
      if (ar.used > best) best = ar.used;
    }
  return best + 256;
}

extern "C" int po_matmul(const void* A, long long lda, long long sa, int trans_a, const void* B, long long ldb,
                         long long sb, int trans_b, float* C, long long ldc, long long sc, int dtype, int precision,
                         long long batch, long long M, long long N, long long K, float alpha, float beta,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != PO_F32 && dtype != PO_BF16) return set_error(PO_ERR_ARG, "matmul: dtype must be fp32 or bf16");
  if (batch < 0 || M < 0 || N < 0 || K < 0) return set_error(PO_ERR_ARG, "matmul: negative size");
  if (batch == 0 || M == 0 || N == 0) return PO_OK;
  if (K == 0) return set_error(PO_ERR_UNSUPPORTED, "matmul: K == 0");
  if (batch > 65535 || M > 0x3fffffff || N > 0x3fffffff || K > 0x3fffffff)
    return set_error(PO_ERR_ARG, "matmul: size too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Stored sta = stored(M, K, trans_a), stb = stored(K, N, trans_b);
  Arena ar(workspace, workspace_bytes);
  unsigned int* sched = take_sched(ar);
  const Staged ga = stage_layout(ar, batch, sta);
  const Staged gb = stage_layout(ar, batch, stb);
  if (workspace == nullptr || ar.overflow()) return set_error(PO_ERR_WORKSPACE, "matmul: workspace too small");

  const bool split = dtype == PO_F32 && precision == 1;
  GemmDesc g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.batch = static_cast<int>(batch);
  g.a_kmajor = !trans_a;  // A stored [M][K] is K-major
  g.b_kmajor = trans_b;   // B stored [N][K] is K-major
  g.kind = (dtype == PO_BF16 || split) ? KIND_BF16 : KIND_TF32;
  g.npass = split ? 3 : 1;
  // The precise mode also sums K chunks outside the truncating accumulator
  // (for bf16 operands, precision 1 asks for that chunked accumulation alone).
  g.chunked = precision == 1;
  g.sched = sched;
  int r;
  if ((r = zero_sched(sched, s))) return r;
  if ((r = prepare_operand(A, dtype, lda, sa, sta, batch, split, ga, g.a, s))) return r;
  if ((r = prepare_operand(B, dtype, ldb, sb, stb, batch, split, gb, g.b, s))) return r;
  g.epi.alpha = alpha;
  if (beta != 0.0f) {
    g.epi.nin = 1;
    g.epi.in[0] = epi_in(C, IN_F32, ldc, sc, beta);
  }
  g.epi.nout = 1;
  g.epi.out[0] = epi_out(C, OUT_F32, ldc, sc);
  return launch_gemm(g, s);
}
