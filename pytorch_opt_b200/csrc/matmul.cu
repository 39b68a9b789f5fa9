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

// How an fp32 operand reaches the tensor cores.
enum Split : int { SPLIT_NONE = 0, SPLIT_BF16 = 1, SPLIT_TF32 = 2 };

// Staging area for one operand: 4 bytes per padded element (one fp32 / bf16
// copy, or a bf16 (hi, lo) pair), 8 for a tf32 (hi, lo) pair.
struct Staged {
  char* base;
  long long ld;
  long long elems;  // batch * rows * ld
};

inline Staged stage_layout(Arena& ar, long long batch, Stored st, int bytes_per_elem) {
  Staged s;
  s.ld = round_up(st.cols, 64);
  s.elems = batch * st.rows * s.ld;
  s.base = static_cast<char*>(ar.take(static_cast<size_t>(s.elems) * bytes_per_elem));
  return s;
}

inline bool tma_ok(const void* p, long long ld, long long bs, long long batch, int es) {
  return reinterpret_cast<uintptr_t>(p) % 16 == 0 && (ld * es) % 16 == 0 && (batch == 1 || (bs * es) % 16 == 0);
}

// Prepare operand views for the product (direct when aligned, else staged).
// split: fp32 source turned into a bf16 or tf32 (hi, lo) pair.
inline int prepare_operand(const void* X, int dtype, long long ld, long long bs, Stored st, long long batch,
                           int split, const Staged& stg, MatView out[2], cudaStream_t s) {
  AnyMat am{X, dtype, st.rows, st.cols, ld, bs};
  if (split != SPLIT_NONE) {
    const void* ps[2];
    int r;
    if (split == SPLIT_BF16) {
      __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(stg.base);
      __nv_bfloat16* lo = hi + stg.elems;
      r = launch_split_bf16(am, static_cast<int>(batch), hi, lo, stg.ld, st.rows * stg.ld, s);
      ps[0] = hi;
      ps[1] = lo;
    } else {
      float* hi = reinterpret_cast<float*>(stg.base);
      float* lo = hi + stg.elems;
      r = launch_split_tf32(am, static_cast<int>(batch), hi, lo, stg.ld, st.rows * stg.ld, s);
      ps[0] = hi;
      ps[1] = lo;
    }
    if (r) return r;
    for (int i = 0; i < 2; ++i) {
      out[i].ptr = ps[i]; out[i].dtype = split == SPLIT_BF16 ? PO_BF16 : PO_F32; out[i].rows = st.rows;
      out[i].cols = st.cols; out[i].ld = stg.ld; out[i].bstride = st.rows * stg.ld;
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
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  const int per = (dtype == PO_F32 && precision == 2) ? 8 : 4;
  size_t best = 0;
  for (int ta = 0; ta < 2; ++ta)
    for (int tb = 0; tb < 2; ++tb) {
      Arena ar(nullptr, 0);
      take_sched(ar);
      stage_layout(ar, batch, stored(M, K, ta), per);
      stage_layout(ar, batch, stored(K, N, tb), per);
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
  if (precision < 0 || precision > 2 || (precision == 2 && dtype != PO_F32))
    return set_error(PO_ERR_ARG, "matmul: precision must be 0, 1 or 2 (2: fp32 operands only)");
  const Stored sta = stored(M, K, trans_a), stb = stored(K, N, trans_b);
  const int split = dtype != PO_F32 ? SPLIT_NONE : (precision == 1 ? SPLIT_BF16 : (precision == 2 ? SPLIT_TF32
                                                                                                    : SPLIT_NONE));
  const int per = split == SPLIT_TF32 ? 8 : 4;
  Arena ar(workspace, workspace_bytes);
  unsigned int* sched = take_sched(ar);
  const Staged ga = stage_layout(ar, batch, sta, per);
  const Staged gb = stage_layout(ar, batch, stb, per);
  if (workspace == nullptr || ar.overflow()) return set_error(PO_ERR_WORKSPACE, "matmul: workspace too small");

  GemmDesc g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.batch = static_cast<int>(batch);
  g.a_kmajor = !trans_a;  // A stored [M][K] is K-major
  g.b_kmajor = trans_b;   // B stored [N][K] is K-major
  g.kind = (dtype == PO_BF16 || split == SPLIT_BF16) ? KIND_BF16 : KIND_TF32;
  g.npass = split != SPLIT_NONE ? 3 : 1;
  // The precise modes also sum K chunks outside the truncating accumulator
  // (for bf16 operands, precision 1 asks for that chunked accumulation alone).
  g.chunked = precision >= 1;
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
