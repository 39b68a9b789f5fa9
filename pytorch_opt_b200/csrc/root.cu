// Inverse p-th matrix root by the coupled Newton iteration, on the tensor cores.
//
// Mirrors pytorch_opt/ops/reference.py:17-40 (_coupled_newton) and :43-68
// (inverse_matrix_root, method="newton"); ATen version
// pytorch_opt/ops/csrc/pytorch_opt_ops.cpp:15-39, :41-63.
//
// Reference iteration (M = sym(A) + damping I, z = (1+p)/(2||M||_F)):
//   X0 = z^(1/p) I, M0 = z M
//   Mi = (1 + 1/p) I - Mk/p ;  X <- X Mi ;  Mk <- Mi^p Mk ;  err = max|Mk - I|
//   stop when err < tol; if err > 1.2 * previous err keep the previous X.
//
// Increment form used here. With Mk = I - p D (D = (I - Mk)/p, so Mi = I + D):
//   X_{k+1} = X_k + X_k D_k
//   Mi^p    = I + T_k           (T by binary powering: (I+U)(I+V) = I + U + V + U V)
//   D_{k+1} = D_k - T_k/p + T_k D_k
//   err     = p * max|D_{k+1}|
// Every product is a polynomial in M, hence symmetric: only the lower
// triangle of tiles is computed and stored mirrored. Products of the small
// increments keep their relative accuracy, so the error test sees the same
// values as the fp64 reference and stops after the same number of steps.
// Precision: split-bf16 (hi*hi + hi*lo + lo*hi) while err > 1e-3, single bf16
// afterwards, fp32 accumulation. The iterates are SPD-like with dominant
// diagonals; the tensor cores see them with zeroed diagonals and the epilogue
// adds the diagonal terms exactly (the accumulator truncates, which would
// otherwise bias the many small off-diagonal terms summed next to one large
// diagonal term). Convergence bookkeeping stays on the device; converged
// batch items are skipped by later launches. Iterations are enqueued in
// blocks of kIterBlock; after each block the host reads one 4-byte count of
// items still iterating and stops enqueueing once it is zero (the reference
// reads its error back after every iteration). Under stream capture no read
// is possible, so all max_iter iterations are enqueued.
#include <math.h>

#include "elementwise.cuh"
#include "gemm_host.cuh"

namespace po {
namespace {

constexpr float kSplitUntil = 1e-3f;  // use split-bf16 products while err exceeds this
constexpr int kIterBlock = 4;         // iterations enqueued between two reads of the active count

struct Slot {
  float* f;
  __nv_bfloat16* h;
  __nv_bfloat16* l;
};

struct RootState {
  float* red;       // per batch: max|D_{k+1}| of the current step (fp32 bits, atomicMax)
  float* prev_err;  // per batch: err of the previous step (< 0: none yet)
  int* active;      // per batch: still iterating
  int* passes;      // per batch: 3 (split) or 1
  int* result;      // per batch: X slot holding the answer
  int* iters;       // per batch: steps taken
  double* sums;     // per batch: ||M||_F^2
  int* count;       // items still active after the last block (read by the host)
};

struct RootBufs {
  Slot X[2], D[2], T[3];
  RootState st;
  long long ld;
  unsigned int* sched;  // tile queue of the products
};

constexpr int kTmpSlots = 3;

void root_layout(Arena& ar, long long batch, long long d, int p, RootBufs& B) {
  B.ld = round_up(d, 64);
  const size_t n = static_cast<size_t>(batch * d * B.ld);
  auto slot = [&](Slot& s) {
    s.f = static_cast<float*>(ar.take(n * 4));
    s.h = static_cast<__nv_bfloat16*>(ar.take(n * 2));
    s.l = static_cast<__nv_bfloat16*>(ar.take(n * 2));
  };
  for (auto& s : B.X) slot(s);
  for (auto& s : B.D) slot(s);
  const int ntmp = p == 1 ? 0 : (p == 2 ? 1 : kTmpSlots);
  for (int i = 0; i < kTmpSlots; ++i) {
    if (i < ntmp) slot(B.T[i]);
    else B.T[i] = Slot{nullptr, nullptr, nullptr};
  }
  const size_t b = static_cast<size_t>(batch);
  B.st.red = static_cast<float*>(ar.take(b * 4));
  B.st.prev_err = static_cast<float*>(ar.take(b * 4));
  B.st.active = static_cast<int*>(ar.take(b * 4));
  B.st.passes = static_cast<int*>(ar.take(b * 4));
  B.st.result = static_cast<int*>(ar.take(b * 4));
  B.st.iters = static_cast<int*>(ar.take(b * 4));
  B.st.sums = static_cast<double*>(ar.take(b * 8));
  B.st.count = static_cast<int*>(ar.take(4));
  B.sched = take_sched(ar);
}

template <int DT>
__device__ __forceinline__ double ld_elem(const void* p, long long i) {
  if (DT == PO_F32) return static_cast<const float*>(p)[i];
  if (DT == PO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<const double*>(p)[i];
}

// fp32 master gets v; the tensor-core operand copies (hi, lo) get v with the
// diagonal zeroed (its contribution is added exactly by the epilogue).
__device__ __forceinline__ void put_slot(const Slot& s, long long o, float v, bool diag) {
  s.f[o] = v;
  const float w = diag ? 0.0f : v;
  const __nv_bfloat16 h = __float2bfloat16_rn(w);
  s.h[o] = h;
  s.l[o] = __float2bfloat16_rn(w - __bfloat162float(h));
}

// Tiled pass over M = sym(A) + damping I (32x32 tiles, 32x8 threads).
//   PHASE 0: sums[b] += sum M_ij^2 (fp64)
//   PHASE 1: D0 = (I - z M)/p, X0 = z^(1/p) I, with z = (1+p)/(2||M||_F)
template <int DT, int PHASE>
__global__ void root_prep_kernel(const void* A, long long ld, long long bs, long long d, double damping, int p,
                                 double* sums, Slot X0, Slot D0, long long ldw) {
  __shared__ double tile[32][33];
  __shared__ double part[8];
  const int b = blockIdx.z;
  const long long r0 = static_cast<long long>(blockIdx.y) * 32, c0 = static_cast<long long>(blockIdx.x) * 32;
  // transposed tile: At(i, j) = A(c0 + i, r0 + j)
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = c0 + i, c = r0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < d && c < d) ? ld_elem<DT>(A, b * bs + r * ld + c) : 0.0;
  }
  __syncthreads();
  double acc = 0.0;
  double z = 0.0, x0 = 0.0;
  if (PHASE == 1) {
    const double fro = fmax(sqrt(sums[b]), 2.2250738585072014e-308);
    z = (1.0 + p) / (2.0 * fro);
    x0 = pow(z, 1.0 / p);
  }
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = r0 + i, c = c0 + threadIdx.x;
    if (r >= d || c >= d) continue;
    double m = 0.5 * (ld_elem<DT>(A, b * bs + r * ld + c) + tile[threadIdx.x][i]);
    if (r == c) m += damping;
    if (PHASE == 0) {
      acc += m * m;
    } else {
      const long long o = b * d * ldw + r * ldw + c;
      const double dd = ((r == c ? 1.0 : 0.0) - z * m) / p;
      put_slot(D0, o, static_cast<float>(dd), r == c);
      put_slot(X0, o, r == c ? static_cast<float>(x0) : 0.0f, r == c);
    }
  }
  if (PHASE == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const int tid = threadIdx.y * 32 + threadIdx.x;
    if ((tid & 31) == 0) part[tid >> 5] = acc;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int w = 0; w < 8; ++w) t += part[w];
      atomicAdd(sums + b, t);
    }
  }
}

__global__ void root_state_init(RootState st, int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  st.red[b] = 0.0f;
  st.prev_err[b] = -1.0f;
  st.active[b] = 1;
  st.passes[b] = 3;
  st.result[b] = 0;
  st.iters[b] = 0;
}

// After step k (X_{k+1} in slot (k+1)&1): apply the reference's stopping rules.
__global__ void root_control(RootState st, int batch, int step, int p, float tol) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch || !st.active[b]) return;
  const float err = static_cast<float>(p) * st.red[b];
  st.red[b] = 0.0f;
  st.iters[b] = step + 1;
  const float prev = st.prev_err[b];
  if (prev >= 0.0f && err > prev * 1.2f) {  // diverging: keep the last good iterate
    st.result[b] = step & 1;
    st.active[b] = 0;
    return;
  }
  st.prev_err[b] = err;
  st.result[b] = (step + 1) & 1;
  if (err < tol || !(err == err)) st.active[b] = 0;
  st.passes[b] = err > kSplitUntil ? 3 : 1;
}

// st.count = number of batch items still iterating (one block).
__global__ void root_count_active(RootState st, int batch) {
  __shared__ int part[32];
  int n = 0;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) n += st.active[b] != 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
    *st.count = t;
  }
}

// out[b] = sym(X[result[b]][b]) cast to the output type.
template <int DT>
__global__ void root_final_kernel(Slot X0, Slot X1, const int* result, long long d, long long ldw, void* out,
                                  long long ld, long long bs) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const float* X = result[b] ? X1.f : X0.f;
  const long long r0 = static_cast<long long>(blockIdx.y) * 32, c0 = static_cast<long long>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = c0 + i, c = r0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < d && c < d) ? X[b * d * ldw + r * ldw + c] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = r0 + i, c = c0 + threadIdx.x;
    if (r >= d || c >= d) continue;
    const float v = 0.5f * (X[b * d * ldw + r * ldw + c] + tile[threadIdx.x][i]);
    const long long o = b * bs + r * ld + c;
    if (DT == PO_F32) static_cast<float*>(out)[o] = v;
    else if (DT == PO_BF16) static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(v);
    else static_cast<double*>(out)[o] = static_cast<double>(v);
  }
}

MatView slot_view(const __nv_bfloat16* p, long long d, long long ld) {
  MatView v;
  v.ptr = p;
  v.dtype = PO_BF16;
  v.rows = d;
  v.cols = d;
  v.ld = ld;
  v.bstride = d * ld;
  return v;
}

// out = alpha U V + beta1 C1 + beta2 C2 (symmetric), written to all three parts of `out`.
int slot_gemm(const RootBufs& B, long long batch, long long d, const Slot& U, const Slot& V, const Slot& out,
              const Slot* c1, float beta1, const Slot* c2, float beta2, float* red, cudaStream_t s) {
  GemmDesc g;
  g.kind = KIND_BF16;
  g.M = g.N = g.K = static_cast<int>(d);
  g.batch = static_cast<int>(batch);
  g.a[0] = slot_view(U.h, d, B.ld);
  g.a[1] = slot_view(U.l, d, B.ld);
  g.b[0] = slot_view(V.h, d, B.ld);
  g.b[1] = slot_view(V.l, d, B.ld);
  g.npass = 3;
  g.passes = B.st.passes;
  g.active = B.st.active;
  g.tri = true;
  g.sched = B.sched;
  const long long bsw = d * B.ld;
  g.epi.alpha = 1.0f;
  if (c1 != nullptr) g.epi.in[g.epi.nin++] = epi_in(c1->f, IN_F32, B.ld, bsw, beta1);
  if (c2 != nullptr) g.epi.in[g.epi.nin++] = epi_in(c2->f, IN_F32, B.ld, bsw, beta2);
  g.epi.nout = 3;
  g.epi.out[0] = epi_out(out.f, OUT_F32, B.ld, bsw);
  g.epi.out[1] = epi_out(out.h, OUT_BF16, B.ld, bsw);
  g.epi.out[2] = epi_out(out.l, OUT_BF16_LO, B.ld, bsw);
  g.epi.out[1].zero_diag = 1;
  g.epi.out[2].zero_diag = 1;
  // The operands' diagonals dominate their rows; keeping them out of the
  // tensor cores' truncating accumulation and adding them exactly here keeps
  // the products accurate to the split-bf16 representation.
  g.epi.diag_split = 1;
  g.epi.dU = epi_in(U.f, IN_F32, B.ld, bsw, 1.0f);
  g.epi.dV = epi_in(V.f, IN_F32, B.ld, bsw, 1.0f);
  g.epi.red_absmax = red;
  g.epi.red_ident = 0.0f;
  return launch_gemm(g, s);
}

bool same(const Slot& a, const Slot& b) { return a.f == b.f; }

}  // namespace
}  // namespace po

using namespace po;

extern "C" size_t po_root_workspace_bytes(long long batch, long long d, int p) {
  if (batch <= 0 || d <= 0 || p < 1) return 0;
  Arena ar(nullptr, 0);
  RootBufs B;
  root_layout(ar, batch, d, p, B);
  return ar.used + 256;
}

extern "C" int po_inverse_root(const void* A, int dtype, long long batch, long long d, long long ld, long long bstride,
                               void* out, long long out_ld, long long out_bstride, int p, double damping,
                               int max_iter, double tol, int* iters_out, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (p < 1) return set_error(PO_ERR_ARG, "p must be a positive integer");
  if (dtype != PO_F32 && dtype != PO_BF16 && dtype != PO_F64)
    return set_error(PO_ERR_ARG, "inverse_root: dtype must be fp32, bf16 or fp64");
  if (batch < 0 || d < 0 || max_iter < 0) return set_error(PO_ERR_ARG, "inverse_root: negative size");
  if (batch == 0 || d == 0) return PO_OK;
  if (A == nullptr || out == nullptr) return set_error(PO_ERR_ARG, "inverse_root: null pointer");
  if (ld < d || out_ld < d) return set_error(PO_ERR_ARG, "inverse_root: row pitch smaller than d");
  if (batch > 65535 || d > 65536) return set_error(PO_ERR_ARG, "inverse_root: size too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Arena ar(workspace, workspace_bytes);
  RootBufs B;
  root_layout(ar, batch, d, p, B);
  if (workspace == nullptr || ar.overflow())
    return set_error(PO_ERR_WORKSPACE, "inverse_root: workspace too small (query po_root_workspace_bytes)");

  int r;
  const int nb = static_cast<int>(batch);
  if ((r = check_cuda(cudaMemsetAsync(B.st.sums, 0, batch * 8, s), "memset"))) return r;
  if ((r = zero_sched(B.sched, s))) return r;
  root_state_init<<<cdiv(batch, 128), 128, 0, s>>>(B.st, nb);
  dim3 grid(cdiv(d, 32), cdiv(d, 32), nb), block(32, 8);
#define PO_ROOT_PREP(DT)                                                                                        \
  root_prep_kernel<DT, 0><<<grid, block, 0, s>>>(A, ld, bstride, d, damping, p, B.st.sums, B.X[0], B.D[0], B.ld); \
  root_prep_kernel<DT, 1><<<grid, block, 0, s>>>(A, ld, bstride, d, damping, p, B.st.sums, B.X[0], B.D[0], B.ld);
  if (dtype == PO_F32) { PO_ROOT_PREP(PO_F32) }
  else if (dtype == PO_BF16) { PO_ROOT_PREP(PO_BF16) }
  else { PO_ROOT_PREP(PO_F64) }
#undef PO_ROOT_PREP
  if ((r = check_cuda(cudaGetLastError(), "root prep"))) return r;

  const float ftol = static_cast<float>(tol);
  const float inv_p = 1.0f / static_cast<float>(p);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if ((r = check_cuda(cudaStreamIsCapturing(s, &cap), "cudaStreamIsCapturing"))) return r;
  const bool can_read = cap == cudaStreamCaptureStatusNone;
  for (int k = 0; k < max_iter; ++k) {
    const Slot& Dk = B.D[k & 1];
    const Slot& Dn = B.D[(k + 1) & 1];
    const Slot& Xk = B.X[k & 1];
    const Slot& Xn = B.X[(k + 1) & 1];
    // T = Mi^p - I by binary powering of (I + D_k).
    Slot base = Dk, res{nullptr, nullptr, nullptr};
    bool have_res = false;
    for (int e = p; e > 0; e >>= 1) {
      if (e & 1) {
        if (!have_res) {
          res = base;
          have_res = true;
        } else {
          Slot nr{nullptr, nullptr, nullptr};
          for (int i = 0; i < kTmpSlots; ++i)
            if (!same(B.T[i], res) && !same(B.T[i], base)) { nr = B.T[i]; break; }
          if ((r = slot_gemm(B, batch, d, res, base, nr, &res, 1.0f, &base, 1.0f, nullptr, s))) return r;
          res = nr;
        }
      }
      if (e > 1) {
        Slot nbs{nullptr, nullptr, nullptr};
        for (int i = 0; i < kTmpSlots; ++i)
          if (!same(B.T[i], res) && !same(B.T[i], base)) { nbs = B.T[i]; break; }
        if ((r = slot_gemm(B, batch, d, base, base, nbs, &base, 2.0f, nullptr, 0.0f, nullptr, s))) return r;
        base = nbs;
      }
    }
    // X_{k+1} = X_k + X_k D_k
    if ((r = slot_gemm(B, batch, d, Xk, Dk, Xn, &Xk, 1.0f, nullptr, 0.0f, nullptr, s))) return r;
    // D_{k+1} = D_k - T/p + T D_k   (p == 1: T = D_k, so D_{k+1} = D_k D_k)
    if (p == 1) r = slot_gemm(B, batch, d, Dk, Dk, Dn, nullptr, 0.0f, nullptr, 0.0f, B.st.red, s);
    else r = slot_gemm(B, batch, d, res, Dk, Dn, &Dk, 1.0f, &res, -inv_p, B.st.red, s);
    if (r) return r;
    root_control<<<cdiv(batch, 128), 128, 0, s>>>(B.st, nb, k, p, ftol);
    if ((r = check_cuda(cudaGetLastError(), "root control"))) return r;
    if (can_read && (k + 1) % kIterBlock == 0 && k + 1 < max_iter) {
      root_count_active<<<1, 256, 0, s>>>(B.st, nb);
      if ((r = check_cuda(cudaGetLastError(), "root count"))) return r;
      int active = 0;
      if ((r = check_cuda(cudaMemcpyAsync(&active, B.st.count, sizeof(int), cudaMemcpyDeviceToHost, s), "count")))
        return r;
      if ((r = check_cuda(cudaStreamSynchronize(s), "root block sync"))) return r;
      if (active == 0) break;
    }
  }

  dim3 fgrid(cdiv(d, 32), cdiv(d, 32), nb);
  if (dtype == PO_F32) root_final_kernel<PO_F32><<<fgrid, block, 0, s>>>(B.X[0], B.X[1], B.st.result, d, B.ld, out, out_ld, out_bstride);
  else if (dtype == PO_BF16) root_final_kernel<PO_BF16><<<fgrid, block, 0, s>>>(B.X[0], B.X[1], B.st.result, d, B.ld, out, out_ld, out_bstride);
  else root_final_kernel<PO_F64><<<fgrid, block, 0, s>>>(B.X[0], B.X[1], B.st.result, d, B.ld, out, out_ld, out_bstride);
  if ((r = check_cuda(cudaGetLastError(), "root final"))) return r;
  if (iters_out != nullptr)
    if ((r = check_cuda(cudaMemcpyAsync(iters_out, B.st.iters, batch * 4, cudaMemcpyDeviceToDevice, s), "iters")))
      return r;
  return PO_OK;
}
