/*
 * pytorch_opt_b200 — C ABI of the B200-native (sm_100a) numerics behind
 * pytorch_opt.ops.
 *
 * Every entry point takes plain device pointers, element counts and strides
 * (in elements), a caller-provided device workspace, and a cudaStream_t passed
 * as `void*` (NULL = legacy default stream). Nothing here allocates device
 * memory; query the workspace size first with the matching *_workspace_bytes
 * function and pass at least that many bytes.
 *
 * Return value: PO_OK (0) or a PO_ERR_* code; po_last_error() then holds a
 * message for the calling thread. Kernels never trap: a bounded wait that
 * gives up records a code in the device error word, read with
 * po_device_error().
 *
 * Layout convention: a "matrix batch" is [batch][rows][cols], row-major with
 * row pitch `ld` and batch pitch `bstride`; columns are contiguous.
 */
#ifndef PYTORCH_OPT_B200_H_
#define PYTORCH_OPT_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define PO_F32 0
#define PO_BF16 1
#define PO_F16 2
#define PO_F64 3

/* status codes */
#define PO_OK 0
#define PO_ERR_ARG 1         /* invalid argument (shape, dtype, stride, value) */
#define PO_ERR_CUDA 2        /* a CUDA runtime / driver call failed */
#define PO_ERR_WORKSPACE 3   /* workspace too small */
#define PO_ERR_DEVICE 4      /* a kernel recorded an error in the device error word */
#define PO_ERR_UNSUPPORTED 5 /* valid request this build does not implement */

/* Message describing the last failure on the calling thread ("" if none). */
const char* po_last_error(void);

/* Synchronises the current device, returns the device error word (0 = none)
 * and clears it when `reset` is nonzero. */
int po_device_error(int reset);

/* Measurement switch (no counterpart in the reference): while enabled, the
 * two-SM GEMM kernel adds, per role and summed over CTAs, the SM clock cycles
 * spent in its waits to 16 device counters (0: MMA issuer waiting for operand
 * stages, 1: MMA issuer waiting for a free accumulator, 2: MMA issuer total,
 * 3: TMA producer waiting for a free stage, 4: producer total, 5: first
 * epilogue warp waiting for an accumulator, 6: its draining and storing,
 * 7: its total, 8: tiles). With out != NULL, synchronises the device, copies
 * the first n counters to out and zeroes them; then sets the switch to
 * `enable`. Off by default; the counters cost a few clock reads per stage. */
int po_gemm_profile(int enable, unsigned long long* out, int n);

/* Library version string. */
const char* po_version(void);

/* Self-test of the kernels' bounded waits (no counterpart in the reference):
 * launches one block that waits on an mbarrier nothing arms, with the wait
 * functions the product kernels use (sleeping = 1: the epilogue's sleeping
 * wait) and a limit of limit_ns instead of their 5 s. The kernel gives up,
 * records code 5 in the device error word and returns; po_device_error()
 * then reports 5 and the context stays usable. */
int po_selftest_wait_timeout(unsigned long long limit_ns, int sleeping, void* stream);

/* ------------------------------------------------------------------------
 * Newton–Schulz orthogonalisation.
 * Replaces pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:65-81
 * (newton_schulz_orthogonalize(G, steps, a, b, c, eps), bound at :106) and
 * mirrors pytorch_opt/ops/reference.py:71-97: transpose when rows > cols,
 * divide by (||X||_F + eps), `steps` quintic iterations
 * A = X X^T, B = b A + c A^2, X = a X + B X, transpose back, cast to the
 * input dtype. G and out: [batch][rows][cols] of `dtype`
 * (PO_F32 / PO_BF16 / PO_F16 / PO_F64). Products accumulate in fp32.
 * tf32_tail < 0 selects the default schedule by m = min(rows, cols):
 * m >= 256: bf16 tensor-core products on every step, with the dominant
 * diagonals of A and B kept out of the bf16 operands and added exactly in
 * fp32 by the epilogues ("diagonal split"); m < 256: split-bf16 pairs
 * (hi*hi + hi*lo + lo*hi) on every step. tf32_tail >= 0 runs the last
 * `tf32_tail` steps on tf32 products and the others on bf16 (both with the
 * diagonal split). With bf16 products on every step (default schedule or
 * tf32_tail = 0), m >= 256 and max(rows, cols) >= 2m, the steps run in
 * groups of up to three: one Gram and one update of the full matrix per
 * group, the steps in between as m x m products (the next Gram is
 * A P^2 for P = a I + b A + c A^2, the update applies P_0 P_1 ...);
 * PO_NS_GROUP=0 in the environment runs one step at a time.
 * ---------------------------------------------------------------------- */
size_t po_ns_workspace_bytes(long long batch, long long rows, long long cols);
int po_newton_schulz(const void* G, int dtype, long long batch, long long rows, long long cols, long long ld,
                     long long bstride, void* out, long long out_ld, long long out_bstride, int steps, float a,
                     float b, float c, float eps, int tf32_tail, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ------------------------------------------------------------------------
 * Newton–Schulz without a caller workspace. No counterpart in the reference:
 * an addition for callers that cannot allocate device memory — code running
 * inside a framework that owns all device memory through its own pool (a
 * cudaMalloc would bypass it and synchronise the device mid-step), or a
 * plug-in handed device pointers but no allocator. Same arguments and result
 * as po_newton_schulz, minus the workspace: the library keeps a
 * PO_NS_STATIC_SCRATCH_BYTES scratch array in device memory on every GPU
 * that loads it (held until the process exits). Problems whose workspace
 * (po_ns_workspace_bytes) exceeds it are rejected with PO_ERR_ARG; one
 * 1024 x 1024 matrix fits. The first call on a device looks up the scratch
 * address (cudaGetSymbolAddress): make that first call before any stream
 * capture. Every call on a device uses the same scratch, so calls that
 * overlap on the GPU (different streams, or different host threads) race;
 * serialise them. Nothing is allocated or freed.
 * ---------------------------------------------------------------------- */
#define PO_NS_STATIC_SCRATCH_BYTES (32u << 20)
int po_newton_schulz_static(const void* G, int dtype, long long batch, long long rows, long long cols, long long ld,
                            long long bstride, void* out, long long out_ld, long long out_bstride, int steps,
                            float a, float b, float c, float eps, int tf32_tail, void* stream);

/* ------------------------------------------------------------------------
 * Inverse p-th root (A_sym + damping I)^(-1/p) by the coupled Newton
 * iteration. Replaces pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:15-39 and
 * :41-63 for method="newton" (bound at :104) and mirrors
 * pytorch_opt/ops/reference.py:17-40 and :43-68: symmetrise, add damping,
 * z = (1+p)/(2||M||_F), X0 = z^(1/p) I, M0 = z M, iterate
 * Mi = (1+1/p) I - Mk/p, X <- X Mi, Mk <- Mi^p Mk until max|Mk - I| < tol,
 * or it grows by more than 1.2x (then the previous X is kept), or max_iter;
 * finally symmetrise and cast back. Products run on the tensor cores as
 * split-bf16 (hi*hi + hi*lo + lo*hi, fp32 accumulate) while max|Mk - I| >
 * 1e-3 and as single bf16 afterwards; the iteration is carried in the
 * increment form E = Mk - I so that the stopping test sees the same values
 * as the fp64 reference. Convergence is tracked on the device; iterations are
 * enqueued in blocks of 4, after each of which the host reads one 4-byte
 * count of items still iterating from the workspace (a stream
 * synchronisation) and stops once it is zero. Under stream capture nothing
 * is read back and all max_iter iterations are enqueued (converged items are
 * skipped inside each launch).
 * A and out: [batch][d][d] of `dtype` (PO_F32 / PO_BF16 / PO_F64).
 * iters_out (nullable): device int[batch], iterations each item ran.
 * ---------------------------------------------------------------------- */
size_t po_root_workspace_bytes(long long batch, long long d, int p);
int po_inverse_root(const void* A, int dtype, long long batch, long long d, long long ld, long long bstride,
                    void* out, long long out_ld, long long out_bstride, int p, double damping, int max_iter,
                    double tol, int* iters_out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * In-place Kronecker factor update. Replaces
 * pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:83-94 (bound at :108) and mirrors
 * pytorch_opt/ops/reference.py:100-114:
 *   L <- beta2 L + (1 - beta2) G G^T,  R <- beta2 R + (1 - beta2) G^T G
 * (beta2 == 1: plain sums). G: m x n (row pitch g_ld) of g_dtype
 * (PO_F32 / PO_BF16); L (m x m, pitch l_ld) and R (n x n, pitch r_ld) are
 * fp32. Only the lower triangle of tiles is computed; the upper triangle is
 * written by mirroring. fp32 G uses split-tf32 products (hi*hi + hi*lo +
 * lo*hi on tf32 pairs, ~2^-21 relative: fp32-grade).
 * ---------------------------------------------------------------------- */
size_t po_kron_workspace_bytes(long long m, long long n, int g_dtype);
int po_kron_factor_update(float* L, long long l_ld, float* R, long long r_ld, const void* G, int g_dtype,
                          long long m, long long n, long long g_ld, double beta2, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * KFAC factor statistics with the exponential moving average fused:
 *   F <- first ? S : beta F + (1 - beta) S,   S = alpha * X^T X
 * X: rows x d (pitch x_ld) of x_dtype (PO_F32 / PO_BF16; fp32 X runs as
 * split-tf32 products, fp32-grade); F: d x d fp32.
 * Replaces pytorch_opt/curvature/kron.py:105-113 (_batch_factors, Linear:
 * A = a^T a / n with alpha = 1/n; G = ghat^T ghat / n with ghat = n g, i.e.
 * alpha = n) together with the EMA of kron.py:95-103 (first call clones).
 * trace (device fp64, nullable) receives tr(F) of the updated factor, summed
 * by the product's epilogue: the input of the pi-split damping of
 * pytorch_opt/curvature/damping.py:10-25 without a pass over F.
 * ---------------------------------------------------------------------- */
size_t po_syrk_workspace_bytes(long long rows, long long d, int x_dtype);
int po_syrk_ema(float* F, long long d, long long f_ld, const void* X, int x_dtype, long long rows, long long x_ld,
                double alpha, double beta, int first, double* trace, void* workspace, size_t workspace_bytes,
                void* stream);

/* ------------------------------------------------------------------------
 * Two-sided preconditioner application out = L @ G @ R. Replaces
 * pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:96-99 (bound at :110) and mirrors
 * pytorch_opt/ops/reference.py:117-121. All operands fp32 (or all bf16):
 * L m x m, G m x n, R n x n, out m x n, dense row-major with the given
 * pitches. fp32 operands use split-tf32 products (fp32-grade).
 * ---------------------------------------------------------------------- */
size_t po_precond_workspace_bytes(long long m, long long n, int dtype);
int po_precond_apply(const void* L, long long l_ld, const void* G, long long g_ld, const void* R, long long r_ld,
                     void* out, long long out_ld, int dtype, long long m, long long n, void* workspace,
                     size_t workspace_bytes, void* stream);
/* Same product, and *sq_sum (device fp64, set here) = ||out||_F^2 computed by
 * the second product's epilogue from the fp32 values it stores: the
 * denominator of Shampoo's grafting ratio target / (||P|| + 1e-30)
 * (pytorch_opt/optim/shampoo.py:128-137) without re-reading P or a separate
 * norm kernel. Same workspace as po_precond_apply. */
int po_precond_apply_norm(const void* L, long long l_ld, const void* G, long long g_ld, const void* R,
                          long long r_ld, void* out, long long out_ld, int dtype, long long m, long long n,
                          double* sq_sum, void* workspace, size_t workspace_bytes, void* stream);
/* out = op(L) @ G @ op(R), op = transpose when trans_l / trans_r (read in
 * place, no transposed copy): SOAP's rotations into and out of the factors'
 * eigenbases, Q_L^T X Q_R and Q_L X Q_R^T (pytorch_opt/optim/soap.py:118-121
 * with _soap_update :47-64). sq_sum nullable as above. Same workspace. */
int po_precond_apply_ex(const void* L, long long l_ld, int trans_l, const void* G, long long g_ld, const void* R,
                        long long r_ld, int trans_r, void* out, long long out_ld, int dtype, long long m, long long n,
                        double* sq_sum, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * SOAP second-moment transport on a basis refresh: replaces
 * pytorch_opt/optim/soap.py:101-108,
 *   C_L = Q_L_old^T Q_L_new;  C_R = Q_R_old^T Q_R_new;
 *   V <- (C_L o C_L)^T V (C_R o C_R)      (o: elementwise product),
 * in place on V (m x n, pitch v_ld). Q_L_* m x m (pitch ql_ld), Q_R_* n x n
 * (pitch qr_ld), all of `dtype` (PO_F32: split-tf32 products, fp32-grade;
 * PO_BF16: bf16 products, squares rounded to bf16), row-major.
 * ---------------------------------------------------------------------- */
size_t po_soap_transport_workspace_bytes(long long m, long long n, int dtype);
int po_soap_transport(const void* ql_old, const void* ql_new, long long ql_ld, const void* qr_old, const void* qr_new,
                      long long qr_ld, void* v, long long v_ld, int dtype, long long m, long long n, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * EKFAC preconditioning of one layer's gradient V (m x n, fp32): replaces
 * EKFAC._precondition, pytorch_opt/optim/ekfac.py:44-58:
 *   Vt = QG^T V QA; S <- first ? Vt^2 : decay*S + (1-decay)*Vt^2 (in place);
 *   out = QG (Vt / (S + lam)) QA^T.
 * QG m x m, QA n x n (the factors' eigenbases), S and out m x n, all fp32
 * row-major with the given pitches; products on split-tf32 operands.
 * ---------------------------------------------------------------------- */
size_t po_ekfac_workspace_bytes(long long m, long long n);
int po_ekfac_precondition(const float* QG, long long qg_ld, const float* QA, long long qa_ld, const float* V,
                          long long v_ld, float* S, long long s_ld, float* out, long long out_ld, long long m,
                          long long n, int first, float decay, float lam, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ------------------------------------------------------------------------
 * Elementwise halves of the Muon step, flat over n elements of `dtype`
 * (PO_F32 / PO_BF16), rounding after each in-place op like the reference's
 * pytorch_opt/optim/muon.py:82-83 and :87-92.
 *   po_muon_momentum: buf <- buf*momentum + g; u <- nesterov ? g + momentum*buf : buf
 *   po_muon_apply:    p <- p*decay (when decay != 1); p <- p - lr_eff*o;
 *                     *sq_sum (device fp64, nullable) += sum(o^2)
 * ---------------------------------------------------------------------- */
int po_muon_momentum(const void* g, void* buf, void* u, int dtype, long long n, float momentum, int nesterov,
                     void* stream);
int po_muon_apply(void* p, const void* o, int dtype, long long n, float lr_eff, float decay, double* sq_sum,
                  void* stream);

/* ------------------------------------------------------------------------
 * One fused Muon step of a group of same-shape matrices: replaces, per
 * matrix, pytorch_opt/optim/muon.py:79-93 (momentum :82, Nesterov :83,
 * newton_schulz_orthogonalize :85, decoupled decay :87-88, update :91 and
 * the update_rms sum :92). g, buf, p: [batch][rows][cols] contiguous of
 * `dtype` (PO_BF16 / PO_F32); buf and p are updated in place:
 *   buf <- buf*momentum + g;  u <- nesterov ? g + momentum*buf : buf
 *   O = NS_steps(u) (as po_newton_schulz, default schedule, cast to dtype)
 *   p <- p*decay (when decay != 1);  p <- p - lr_eff*O;  *sq_sum += sum(O^2)
 * with the reference's roundings (every in-place op rounds to dtype; the
 * add's alpha is rounded to dtype). The momentum pass also sums each
 * matrix's ||u||_F^2, bf16 u is read directly by the first products (no
 * packed copy), and the last product's epilogue updates p, so O is never
 * stored. o_out (nullable, [batch][rows][cols] of dtype) also receives O.
 * sq_sum: device fp64, nullable, accumulated (not reset).
 * ---------------------------------------------------------------------- */
size_t po_muon_step_workspace_bytes(long long batch, long long rows, long long cols, int dtype);
int po_muon_step(const void* g, void* buf, void* p, int dtype, long long batch, long long rows, long long cols,
                 float momentum, int nesterov, int ns_steps, float a, float b, float c, float eps, float lr_eff,
                 float decay, double* sq_sum, void* o_out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * General batched product used by the ops above, exported for tests:
 *   C[b] = alpha * op(A[b]) @ op(B[b]) + beta * C[b]
 * A: M x K (trans_a: stored K x M), B: K x N (trans_b: stored N x K), all of
 * `dtype` PO_BF16 (bf16 products; precision 1 = sum K in chunks outside the
 * truncating tensor-core accumulator, for long K) or PO_F32 (precision:
 * 0 = tf32, 1 = split-bf16 (~2^-16 relative), 2 = split-tf32 (~2^-21,
 * fp32-grade); 1 and 2 chunked). C is fp32. Pitches in elements.
 * ---------------------------------------------------------------------- */
size_t po_matmul_workspace_bytes(long long batch, long long M, long long N, long long K, int dtype, int precision);
int po_matmul(const void* A, long long lda, long long sa, int trans_a, const void* B, long long ldb, long long sb,
              int trans_b, float* C, long long ldc, long long sc, int dtype, int precision, long long batch,
              long long M, long long N, long long K, float alpha, float beta, void* workspace,
              size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PYTORCH_OPT_B200_H_ */
