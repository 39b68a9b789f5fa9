// Warp-specialised, persistent tcgen05 GEMM for sm_100a.
//
//   D[b] = epilogue( A[b] (M x K) * B[b]^T (N x K) )      for b in [0, batch)
//
// * Operands are read by TMA (128-byte swizzle) into a STAGES-deep shared
//   memory ring; each operand is either K-major (rows of K contiguous) or
//   MN-major (the M/N index contiguous, i.e. the transposed view).
// * One elected thread issues tcgen05.mma into a double-buffered TMEM
//   accumulator (2 x BN fp32 columns), so the epilogue of tile i overlaps the
//   main loop of tile i+1.
// * Eight epilogue warps drain TMEM with tcgen05.ld and apply a fused
//   "alpha*acc + sum(beta_i*C_i) + gamma*I" with up to three typed outputs,
//   optional mirrored stores (symmetric products computed on the lower
//   triangle of tiles only), an optional per-batch max|D - ident*I| or
//   sum of D^2, the exact diagonal split (both operands' diagonals, or the
//   left operand's as a per-row scale of the addend), the diagonal written
//   out or summed (trace), and the EKFAC rescaling.
// * Split-bf16 ("bf16x3") products: npass = 3 runs the K loop three times,
//   hi*hi + hi*lo + lo*hi, into the same accumulator.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA
// issuer, warps 2..9 = epilogue (warp w owns TMEM lanes 32*(w%4) .. +31 and
// half of the tile's columns: the first half for warps 2..5, the second for 6..9).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace po {

enum OperandKind : int { KIND_BF16 = 0, KIND_TF32 = 1 };

enum OutKind : int {
  OUT_F32 = 0,      // fp32 as computed
  OUT_BF16 = 1,     // bf16, round to nearest even
  OUT_TF32 = 2,     // fp32 rounded (nearest, ties away) to the tf32 grid
  OUT_BF16_LO = 3,  // bf16(v - float(bf16(v))): low half of a split-bf16 pair
  OUT_F16 = 4,      // fp16
  OUT_F64 = 5,      // fp64 (scalar stores)
  OUT_TF32_LO = 6,  // tf32(v - tf32(v)): low half of a split-tf32 pair
};
enum InKind : int { IN_F32 = 0, IN_BF16 = 1 };

struct EpiIn {
  const void* ptr;
  long long ld;       // elements between rows
  long long bstride;  // elements between batch items
  int kind;           // InKind
  int vec;            // 16-byte vector access legal
  float beta;
};

struct EpiOut {
  void* ptr;
  long long ld;
  long long bstride;
  int kind;       // OutKind
  int trans;      // write element (i, j) to ptr[j*ld + i]
  int vec;
  int zero_diag;  // store 0 on the diagonal (operand copies for the diagonal split)
  int lower_only; // symmetric product: skip the mirrored copy (readers use only lower-triangle
                  // tiles and whole diagonal tiles of a product tiled the same way)
};

constexpr int kGemmThreads = 320;                  // 10 warps
constexpr int kEpilogueThreads = kGemmThreads - 64;  // warps 2..9
constexpr int kMaxEpiIn = 2;
constexpr int kMaxEpiOut = 3;

struct Epilogue {
  float alpha;  // scale of the accumulator
  float gamma;  // added on the diagonal (i == j)
  int nin;
  int nout;
  EpiIn in[kMaxEpiIn];
  EpiOut out[kMaxEpiOut];
  float* red_absmax;  // per batch: max |D_ij - red_ident * [i==j]| (nullable), fp32 bits >= 0
  float red_ident;
  // Per batch: += sum of D_ij^2 over the stored values (nullable; products
  // without mirrored tiles only, and never together with red_absmax: the
  // per-thread reduction register serves one of the two).
  double* red_sumsq;
  // EKFAC rescaling of the product Vt (pytorch_opt/optim/ekfac.py:51-58), on
  // plain products only: in place S <- first ? Vt^2 : decay*S + (1-decay)*Vt^2
  // (fp32, S shaped like the output), then the outputs receive Vt / (S + lam).
  float* ek_s;
  long long ek_ld, ek_bstride;
  float ek_decay, ek_lam;
  int ek_first;
  // Diagonal split of a symmetric product U V whose operands were passed to
  // the tensor cores with zeroed diagonals: the epilogue adds the diagonal's
  // exact contribution alpha * (u_i V_ij + U_ij v_j - [i==j] u_i v_i) from
  // the fp32 masters U, V (u, v = their diagonals), and the mirrored half of
  // the tile reuses the same values.
  int diag_split;
  EpiIn dU, dV;
  // The addends are exactly symmetric (written by mirrored stores), so the
  // mirrored half of an off-diagonal tile takes the same values as the tile.
  int mirror_same;
  // Row-diagonal split of a plain product U X whose left operand U reached
  // the tensor cores with a zeroed diagonal, X being the addend in[0]: the
  // epilogue adds u_i X_ij exactly, i.e. in[0] is scaled by
  // beta + in0_rowcoef[b][i] instead of beta (nullable).
  const float* in0_rowcoef;
  long long in0_rowcoef_bs;
  // The same for the right operand's diagonal, U X with X on the left (X D):
  // in[0]'s coefficient for column j is beta + in0_colcoef[b][j] (nullable).
  const float* in0_colcoef;
  long long in0_colcoef_bs;
  // Diagonal of the stored result: diag_out[b][i] = D_ii (nullable; written by
  // the thread holding the diagonal element, on diagonal tiles).
  float* diag_out;
  long long diag_out_bs;
  // Per batch: += sum of the stored diagonal values D_ii (nullable): the
  // trace of the result, for KFAC's pi-split damping.
  double* red_trace;
  // Symmetric diagonal split against the addend (nullable): in[0] is the
  // fp32 master of a symmetric operand A whose diagonal was zeroed for the
  // tensor cores (the product is F F, F = A off its diagonal) and dsym is
  // that diagonal, contiguous [batch][M]. With one row read of A the
  // epilogue forms alpha*acc + (beta0 + alpha*(d_i + d_j)) A_ij - [i==j]
  // alpha d_i^2 = alpha*(A A) + beta0*A.
  const float* dsym;
  long long dsym_bs;
  // Product S T of two symmetric matrices held split (nullable s2_ds = off):
  // the operands are F_S, F_T (zero diagonals), s2_fs / s2_ft the same bf16
  // arrays read by rows, s2_ds / s2_dt their diagonals ([batch][M], plus the
  // constants s2_ds_add / s2_dt_add: P = a I + B keeps B's arrays). The
  // epilogue forms alpha*(acc + d_S,i F_T,ij + F_S,ij d_T,j + [i==j] d_S,i d_T,i)
  // = alpha*(S T); with S, T polynomials in one matrix S T is symmetric.
  EpiIn s2_fs, s2_ft;
  const float* s2_ds;
  const float* s2_dt;
  long long s2_d_bs;
  float s2_ds_add, s2_dt_add;
  // Per-batch scales read on the device (nullable): alpha is multiplied by
  // alpha_scale[b], in[0]'s coefficient (beta, plus in0_rowcoef) by in_scale[b].
  const float* alpha_scale;
  const float* in_scale;
  // red_sumsq: 1 = every batch item adds into red_sumsq[0].
  int red_sumsq_shared;
  // Muon's parameter update from the product's values (nullable mu_p):
  // o = v rounded to the parameter type, p <- round(round(p * mu_decay) +
  // mu_alpha * o) (the decay only when mu_use_decay), and red_sumsq gets o^2.
  // p is [batch][..] with pitch mu_ld, batch pitch mu_bs, laid out like the
  // product. Outputs, if any, are still written.
  void* mu_p;
  long long mu_ld, mu_bs;
  int mu_bf16;  // parameter type: 1 = bf16, 0 = fp32
  int mu_vec;   // 16-byte vector access legal
  int mu_use_decay;
  float mu_decay, mu_alpha;
  // Triangular products: on diagonal tiles store only j <= i and mirror the
  // lower half to the upper (bit-symmetric results when the (i, j) and
  // (j, i) accumulations differ, as for split passes hi*lo + lo*hi).
  int sym_diag;
};

struct alignas(64) GemmParams {
  CUtensorMap mapA[2];  // [0] = plain / hi, [1] = lo (split-bf16 only)
  CUtensorMap mapB[2];
  int M, N, K, batch;
  int tiles_m, tiles_n, tiles_per_batch, total_tiles;
  int tri;    // compute only tiles with nt <= mt (M == N, BN == 128) and mirror-store
  int npass;  // 1 or 3
  int a4d, b4d;  // MN-major operand mapped as 4-D [batch][MN / (128 B)][K][128 B]: one TMA copy per stage
  int group;     // row tiles per raster band (tiles of a band share A panels through L2)
  unsigned int* sched;  // {next tile, CTAs finished}: dynamic tile queue (two-SM kernel), null = static
  const int* active;  // per batch: nonzero = compute (nullable: all)
  const int* passes;  // per batch pass count (nullable: npass)
  int* err;           // device error word
  // Measurement only (nullable): cycles each role of the two-SM kernel spends
  // in its waits, summed over CTAs (see po_gemm_profile).
  unsigned long long* prof;
  int no_prefetch;  // 1: no L2 prefetch of the epilogue's row reads (measurement)
  Epilogue epi;
};

// Slots of GemmParams::prof.
enum GemmProf : int {
  kProfMmaFullWait = 0,    // MMA issuer waiting for operand stages (TMA not ahead)
  kProfMmaTemptyWait = 1,  // MMA issuer waiting for a free accumulator (epilogue behind)
  kProfMmaTotal = 2,       // MMA issuer's whole loop
  kProfProdEmptyWait = 3,  // TMA producer waiting for a free stage (MMA behind)
  kProfProdTotal = 4,
  kProfEpiFullWait = 5,    // epilogue waiting for an accumulator (MMA behind)
  kProfEpiWork = 6,        // epilogue draining and storing tiles
  kProfEpiTotal = 7,
  kProfTiles = 8,          // tiles processed (by the MMA issuers)
  kProfSlots = 16
};

template <int KIND, int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int ES = (KIND == KIND_BF16) ? 2 : 4;  // bytes per element in smem
  static constexpr int BK = 128 / ES;                     // K elements per stage (one 128 B swizzle row)
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int MMA_K = (KIND == KIND_BF16) ? 16 : 8;  // 32 bytes of K per instruction
  static constexpr int KSTEPS = BK / MMA_K;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

struct TileCoord {
  int b, mt, nt;
};

__device__ __forceinline__ TileCoord decode_tile(const GemmParams& P, int t) {
  TileCoord c;
  c.b = t / P.tiles_per_batch;
  int r = t - c.b * P.tiles_per_batch;
  if (P.tri) {
    int mt = static_cast<int>((sqrtf(8.0f * static_cast<float>(r) + 1.0f) - 1.0f) * 0.5f);
    while ((mt + 1) * (mt + 2) / 2 <= r) ++mt;
    while (mt * (mt + 1) / 2 > r) --mt;
    c.mt = mt;
    c.nt = r - mt * (mt + 1) / 2;
  } else {
    // Rasterise in bands of 8 row-tiles so concurrently running CTAs share
    // operand panels in L2.
    const int GROUP = P.group;
    const int band = r / (GROUP * P.tiles_n);
    const int first = band * GROUP;
    const int rows = min(P.tiles_m - first, GROUP);
    const int in_band = r - band * GROUP * P.tiles_n;
    c.mt = first + in_band % rows;
    c.nt = in_band / rows;
  }
  return c;
}

__device__ __forceinline__ bool tile_active(const GemmParams& P, int b) {
  return P.active == nullptr || __ldg(P.active + b) != 0;
}
__device__ __forceinline__ int tile_passes(const GemmParams& P, int b) {
  return P.passes == nullptr ? P.npass : __ldg(P.passes + b);
}

// ------------------------------------------------------------ epilogue I/O
// The epilogue works on chunks of EC consecutive accumulator columns of one
// row (one thread per row).
constexpr int EC = 16;

__device__ __forceinline__ float round_tf32(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

__device__ __forceinline__ float bf16_lo(float v) {
  const float hi = __bfloat162float(__float2bfloat16_rn(v));
  return v - hi;
}

__device__ __forceinline__ float tf32_lo(float v) { return round_tf32(v - round_tf32(v)); }

// x[j] += beta * in(row, col0 + j) (columns >= ncols contribute 0).
__device__ __forceinline__ void add_row(const EpiIn& in, float beta, int b, int row, int col0, int ncols,
                                        float (&x)[EC]) {
  const long long base = static_cast<long long>(b) * in.bstride + static_cast<long long>(row) * in.ld + col0;
  if (in.kind == IN_F32) {
    const float* p = static_cast<const float*>(in.ptr) + base;
    if (in.vec && col0 + EC <= ncols) {
#pragma unroll
      for (int q = 0; q < EC / 4; ++q) {
        const float4 f = reinterpret_cast<const float4*>(p)[q];
        x[4 * q] += beta * f.x;
        x[4 * q + 1] += beta * f.y;
        x[4 * q + 2] += beta * f.z;
        x[4 * q + 3] += beta * f.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < EC; ++j)
        if (col0 + j < ncols) x[j] += beta * p[j];
    }
  } else {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(in.ptr) + base;
    if (in.vec && col0 + EC <= ncols) {
#pragma unroll
      for (int q = 0; q < EC / 8; ++q) {
        const uint4 u = reinterpret_cast<const uint4*>(p)[q];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          x[8 * q + 2 * e] += beta * f.x;
          x[8 * q + 2 * e + 1] += beta * f.y;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < EC; ++j)
        if (col0 + j < ncols) x[j] += beta * __bfloat162float(p[j]);
    }
  }
}

// x[j] += beta * in(col0 + j, row): the transposed position (coalesced
// across the warp, whose lanes hold consecutive rows).
template <typename T>
__device__ __forceinline__ void add_col_typed(const T* p, long long ld, int nv, float beta, float (&x)[EC]) {
  if (nv >= EC) {
#pragma unroll
    for (int j = 0; j < EC; ++j) x[j] += beta * static_cast<float>(p[j * ld]);
  } else {
#pragma unroll
    for (int j = 0; j < EC; ++j)
      if (j < nv) x[j] += beta * static_cast<float>(p[j * ld]);
  }
}

__device__ __forceinline__ void add_col(const EpiIn& in, float beta, int b, int row, int col0, int ncols,
                                        float (&x)[EC]) {
  const long long off = static_cast<long long>(b) * in.bstride + row + static_cast<long long>(col0) * in.ld;
  const int nv = ncols - col0;
  if (in.kind == IN_F32) add_col_typed(static_cast<const float*>(in.ptr) + off, in.ld, nv, beta, x);
  else add_col_typed(static_cast<const __nv_bfloat16*>(in.ptr) + off, in.ld, nv, beta, x);
}

__device__ __forceinline__ void store_elem(const EpiOut& o, long long off, float v) {
  switch (o.kind) {
    case OUT_F32: static_cast<float*>(o.ptr)[off] = v; break;
    case OUT_TF32: static_cast<float*>(o.ptr)[off] = round_tf32(v); break;
    case OUT_TF32_LO: static_cast<float*>(o.ptr)[off] = tf32_lo(v); break;
    case OUT_BF16: static_cast<__nv_bfloat16*>(o.ptr)[off] = __float2bfloat16_rn(v); break;
    case OUT_BF16_LO: static_cast<__nv_bfloat16*>(o.ptr)[off] = __float2bfloat16_rn(bf16_lo(v)); break;
    case OUT_F64: static_cast<double*>(o.ptr)[off] = static_cast<double>(v); break;
    default: static_cast<__half*>(o.ptr)[off] = __float2half_rn(v); break;
  }
}

// Store EC values of row `row` at columns col0.. (row-major orientation).
template <typename Cvt>
__device__ __forceinline__ void store_row_f32x4(float* p, const float (&v)[EC], Cvt cvt) {
#pragma unroll
  for (int q = 0; q < EC / 4; ++q)
    reinterpret_cast<float4*>(p)[q] = make_float4(cvt(v[4 * q]), cvt(v[4 * q + 1]), cvt(v[4 * q + 2]), cvt(v[4 * q + 3]));
}
template <typename Cvt>
__device__ __forceinline__ void store_row_bf16x8(__nv_bfloat16* p, const float (&v)[EC], Cvt cvt) {
#pragma unroll
  for (int q = 0; q < EC / 8; ++q) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(cvt(v[8 * q + 2 * e]), cvt(v[8 * q + 2 * e + 1]));
    reinterpret_cast<uint4*>(p)[q] = u;
  }
}

__device__ __forceinline__ void store_row(const EpiOut& o, int b, int row, int col0, int ncols, const float (&v)[EC]) {
  const long long base = static_cast<long long>(b) * o.bstride + static_cast<long long>(row) * o.ld + col0;
  if (o.vec && col0 + EC <= ncols) {
    switch (o.kind) {
      case OUT_F32:
        store_row_f32x4(static_cast<float*>(o.ptr) + base, v, [](float x) { return x; });
        return;
      case OUT_TF32:
        store_row_f32x4(static_cast<float*>(o.ptr) + base, v, [](float x) { return round_tf32(x); });
        return;
      case OUT_TF32_LO:
        store_row_f32x4(static_cast<float*>(o.ptr) + base, v, [](float x) { return tf32_lo(x); });
        return;
      case OUT_BF16:
        store_row_bf16x8(static_cast<__nv_bfloat16*>(o.ptr) + base, v, [](float x) { return x; });
        return;
      case OUT_BF16_LO:
        store_row_bf16x8(static_cast<__nv_bfloat16*>(o.ptr) + base, v, [](float x) { return bf16_lo(x); });
        return;
      default:
        break;
    }
  }
#pragma unroll
  for (int j = 0; j < EC; ++j)
    if (col0 + j < ncols) store_elem(o, base + j, v[j]);
}

// Store element (row, col0+j) at the transposed position [col0+j][row]: one
// store per column, coalesced across the warp. The output kind is resolved
// once per chunk, not per element.
template <typename T, typename Cvt>
__device__ __forceinline__ void store_col_typed(T* p, long long ld, int nv, const float (&v)[EC], Cvt cvt) {
  if (nv >= EC) {
#pragma unroll
    for (int j = 0; j < EC; ++j) p[j * ld] = cvt(v[j]);
  } else {
#pragma unroll
    for (int j = 0; j < EC; ++j)
      if (j < nv) p[j * ld] = cvt(v[j]);
  }
}

__device__ __forceinline__ void store_col(const EpiOut& o, int b, int row, int col0, int ncols, const float (&v)[EC]) {
  const long long off = static_cast<long long>(b) * o.bstride + row + static_cast<long long>(col0) * o.ld;
  const int nv = ncols - col0;
  switch (o.kind) {
    case OUT_F32:
      store_col_typed(static_cast<float*>(o.ptr) + off, o.ld, nv, v, [](float x) { return x; });
      break;
    case OUT_TF32:
      store_col_typed(static_cast<float*>(o.ptr) + off, o.ld, nv, v, [](float x) { return round_tf32(x); });
      break;
    case OUT_TF32_LO:
      store_col_typed(static_cast<float*>(o.ptr) + off, o.ld, nv, v, [](float x) { return tf32_lo(x); });
      break;
    case OUT_BF16:
      store_col_typed(static_cast<__nv_bfloat16*>(o.ptr) + off, o.ld, nv, v,
                      [](float x) { return __float2bfloat16_rn(x); });
      break;
    case OUT_BF16_LO:
      store_col_typed(static_cast<__nv_bfloat16*>(o.ptr) + off, o.ld, nv, v,
                      [](float x) { return __float2bfloat16_rn(bf16_lo(x)); });
      break;
    case OUT_F64:
      store_col_typed(static_cast<double*>(o.ptr) + off, o.ld, nv, v, [](float x) { return static_cast<double>(x); });
      break;
    default:
      store_col_typed(static_cast<__half*>(o.ptr) + off, o.ld, nv, v, [](float x) { return __float2half_rn(x); });
      break;
  }
}

// Load EC consecutive fp32 elements of row `row` (zeros past ncols).
__device__ __forceinline__ void load_row_f32(const EpiIn& in, int b, int row, int col0, int ncols, float (&x)[EC]) {
  const float* p = static_cast<const float*>(in.ptr) + static_cast<long long>(b) * in.bstride +
                   static_cast<long long>(row) * in.ld + col0;
  if (in.vec && col0 + EC <= ncols) {
#pragma unroll
    for (int q = 0; q < EC / 4; ++q) {
      const float4 f = reinterpret_cast<const float4*>(p)[q];
      x[4 * q] = f.x; x[4 * q + 1] = f.y; x[4 * q + 2] = f.z; x[4 * q + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < EC; ++j) x[j] = (col0 + j < ncols) ? p[j] : 0.0f;
  }
}

// Load EC consecutive elements of row `row` of an fp32 or bf16 input as fp32
// (zeros past ncols).
__device__ __forceinline__ void load_row_any(const EpiIn& in, int b, int row, int col0, int ncols, float (&x)[EC]) {
  if (in.kind == IN_F32) {
    load_row_f32(in, b, row, col0, ncols, x);
    return;
  }
  const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(in.ptr) + static_cast<long long>(b) * in.bstride +
                           static_cast<long long>(row) * in.ld + col0;
  if (in.vec && col0 + EC <= ncols) {
#pragma unroll
    for (int q = 0; q < EC / 8; ++q) {
      const uint4 u = reinterpret_cast<const uint4*>(p)[q];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        x[8 * q + 2 * e] = f.x;
        x[8 * q + 2 * e + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < EC; ++j) x[j] = (col0 + j < ncols) ? __bfloat162float(p[j]) : 0.0f;
  }
}

// EC consecutive fp32 values of a vector from index col0 (zeros past n).
__device__ __forceinline__ void load_vec_f32(const float* d, int col0, int n, float (&x)[EC]) {
  if (col0 + EC <= n && (reinterpret_cast<uintptr_t>(d + col0) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < EC / 4; ++q) {
      const float4 f = reinterpret_cast<const float4*>(d + col0)[q];
      x[4 * q] = f.x; x[4 * q + 1] = f.y; x[4 * q + 2] = f.z; x[4 * q + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < EC; ++j) x[j] = (col0 + j < n) ? d[col0 + j] : 0.0f;
  }
}

// Store to output `o`, honouring its zero-diagonal flag (jd: column of the
// diagonal within this chunk, or out of range).
__device__ __forceinline__ void store_out(const EpiOut& o, int b, int row, int col0, int ncols, int jd,
                                          const float (&v)[EC]) {
  if (o.zero_diag && jd >= 0 && jd < EC) {
    float w[EC];
#pragma unroll
    for (int j = 0; j < EC; ++j) w[j] = (j == jd) ? 0.0f : v[j];
    if (o.trans) store_col(o, b, row, col0, ncols, w);
    else store_row(o, b, row, col0, ncols, w);
    return;
  }
  if (o.trans) store_col(o, b, row, col0, ncols, v);
  else store_row(o, b, row, col0, ncols, v);
}

// Ask L2 for the addend bytes of one row segment [col0, col0 + ncols) before
// the accumulator is ready, so the epilogue's loads hit L2 instead of DRAM.
__device__ __forceinline__ void prefetch_row_segment(const void* base, int es, long long ld, long long bstride, int b,
                                                     int row, int col0, int ncols) {
  if (ncols <= 0) return;
  const char* p = static_cast<const char*>(base) +
                  (static_cast<long long>(b) * bstride + static_cast<long long>(row) * ld + col0) * es;
  const char* end = p + static_cast<long long>(ncols) * es;
  for (const char* q = reinterpret_cast<const char*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(127)); q < end;
       q += 128)
    prefetch_l2(q);
}

// Prefetch every row-oriented addend this thread's epilogue will read for
// columns [col0, col0 + ncols) of `row`.
__device__ __forceinline__ void epilogue_prefetch(const GemmParams& P, int b, int row, int col0, int ncols) {
  const Epilogue& E = P.epi;
  if (row >= P.M || P.no_prefetch) return;
  ncols = min(ncols, P.N - col0);
#pragma unroll
  for (int i = 0; i < kMaxEpiIn; ++i)
    if (i < E.nin)
      prefetch_row_segment(E.in[i].ptr, E.in[i].kind == IN_F32 ? 4 : 2, E.in[i].ld, E.in[i].bstride, b, row, col0,
                           ncols);
  if (E.mu_p != nullptr)
    prefetch_row_segment(E.mu_p, E.mu_bf16 ? 2 : 4, E.mu_ld, E.mu_bs, b, row, col0, ncols);
  if (E.diag_split) {
    prefetch_row_segment(E.dU.ptr, 4, E.dU.ld, E.dU.bstride, b, row, col0, ncols);
    prefetch_row_segment(E.dV.ptr, 4, E.dV.ld, E.dV.bstride, b, row, col0, ncols);
  }
  if (E.s2_ds != nullptr) {
    prefetch_row_segment(E.s2_fs.ptr, 2, E.s2_fs.ld, E.s2_fs.bstride, b, row, col0, ncols);
    if (E.s2_ft.ptr != E.s2_fs.ptr)
      prefetch_row_segment(E.s2_ft.ptr, 2, E.s2_ft.ld, E.s2_ft.bstride, b, row, col0, ncols);
  }
}

// Running max of |values| for the convergence test; NaN counts as +inf.
__device__ __forceinline__ void red_update(float& red, float d) {
  red = (d != d) ? __int_as_float(0x7f800000) : fmaxf(red, d);
}

// Muon's in-place parameter update from the chunk's values v (see
// Epilogue::mu_p); red += sum of the rounded update squared. The roundings
// follow the reference's in-place ops on the parameter dtype
// (pytorch_opt/optim/muon.py:87-91): O is the Newton-Schulz result cast to
// the parameter dtype, p.mul_(decay) rounds, p.add_(O, alpha) rounds once.
__device__ __forceinline__ float mu_round(float x, int bf16) {
  return bf16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

__device__ __forceinline__ void muon_apply_chunk(const Epilogue& E, int b, int row, int col0, int ncols,
                                                 const float (&v)[EC], float& red) {
  const long long base = static_cast<long long>(b) * E.mu_bs;
  float o[EC];
#pragma unroll
  for (int j = 0; j < EC; ++j) {
    o[j] = (col0 + j < ncols) ? mu_round(v[j], E.mu_bf16) : 0.0f;
    red = fmaf(o[j], o[j], red);
  }
  if (E.mu_vec && col0 + EC <= ncols) {
    if (E.mu_bf16) {
      __nv_bfloat16* p = static_cast<__nv_bfloat16*>(E.mu_p) + base + static_cast<long long>(row) * E.mu_ld + col0;
#pragma unroll
      for (int q = 0; q < EC / 8; ++q) {
        uint4 u = reinterpret_cast<const uint4*>(p)[q];
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __bfloat1622float2(h[e]);
          if (E.mu_use_decay) {
            f.x = mu_round(f.x * E.mu_decay, 1);
            f.y = mu_round(f.y * E.mu_decay, 1);
          }
          h[e] = __floats2bfloat162_rn(fmaf(E.mu_alpha, o[8 * q + 2 * e], f.x), fmaf(E.mu_alpha, o[8 * q + 2 * e + 1], f.y));
        }
        reinterpret_cast<uint4*>(p)[q] = u;
      }
    } else {
      float* p = static_cast<float*>(E.mu_p) + base + static_cast<long long>(row) * E.mu_ld + col0;
#pragma unroll
      for (int q = 0; q < EC / 4; ++q) {
        float4 f = reinterpret_cast<const float4*>(p)[q];
        float* fx = reinterpret_cast<float*>(&f);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float pd = E.mu_use_decay ? fx[e] * E.mu_decay : fx[e];
          fx[e] = fmaf(E.mu_alpha, o[4 * q + e], pd);
        }
        reinterpret_cast<float4*>(p)[q] = f;
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < EC; ++j) {
    if (col0 + j >= ncols) continue;
    const long long off = base + static_cast<long long>(row) * E.mu_ld + col0 + j;
    if (E.mu_bf16) {
      __nv_bfloat16* p = static_cast<__nv_bfloat16*>(E.mu_p) + off;
      float f = __bfloat162float(*p);
      if (E.mu_use_decay) f = mu_round(f * E.mu_decay, 1);
      *p = __float2bfloat16_rn(fmaf(E.mu_alpha, o[j], f));
    } else {
      float* p = static_cast<float*>(E.mu_p) + off;
      const float f = E.mu_use_decay ? *p * E.mu_decay : *p;
      *p = fmaf(E.mu_alpha, o[j], f);
    }
  }
}

// Epilogue for one EC-column chunk held by one thread (one row).
__device__ __forceinline__ void epilogue_chunk(const GemmParams& P, const TileCoord& tc, int row, int col0,
                                               bool mirror, const float (&acc)[EC], float& red) {
  const Epilogue& E = P.epi;
  const int N = P.N;
  if (row >= P.M) return;
  const int jd = row - col0;  // diagonal column within this chunk, if any
  float v[EC];
  const bool same = E.diag_split || E.mirror_same || E.dsym != nullptr || E.s2_ds != nullptr;
  if (mirror && !same) {
    // Element (row, c) of an off-diagonal tile of a symmetric product is also
    // element (c, row): rebuild it with the addends read at (c, row) and
    // store it there. Off-diagonal tiles hold no diagonal entries.
#pragma unroll
    for (int j = 0; j < EC; ++j) v[j] = E.alpha * acc[j];
#pragma unroll
    for (int i = 0; i < kMaxEpiIn; ++i)
      if (i < E.nin) add_col(E.in[i], E.in[i].beta, tc.b, row, col0, N, v);
#pragma unroll
    for (int o = 0; o < kMaxEpiOut; ++o)
      if (o < E.nout) store_col(E.out[o], tc.b, row, col0, N, v);
    if (E.red_absmax != nullptr) {
#pragma unroll
      for (int j = 0; j < EC; ++j)
        if (col0 + j < N) red_update(red, fabsf(v[j]));
    }
  }
  const float alpha = E.alpha_scale != nullptr ? E.alpha * E.alpha_scale[tc.b] : E.alpha;
#pragma unroll
  for (int j = 0; j < EC; ++j) v[j] = alpha * acc[j];
  int first_in = 0;
  if (E.dsym != nullptr) {
    // alpha*(F F) + alpha*(D A + A D - D^2) + beta0*A from one row of A.
    const float* d = E.dsym + static_cast<long long>(tc.b) * E.dsym_bs;
    const float di = d[row];
    float a_row[EC], dj[EC];
    load_row_f32(E.in[0], tc.b, row, col0, N, a_row);
    load_vec_f32(d, col0, N, dj);
    const float beta0 = E.in[0].beta;
#pragma unroll
    for (int j = 0; j < EC; ++j) {
      v[j] = fmaf(fmaf(alpha, di + dj[j], beta0), a_row[j], v[j]);
      if (j == jd) v[j] -= alpha * di * di;
    }
    first_in = 1;
  } else if (E.diag_split) {
    const float* U = static_cast<const float*>(E.dU.ptr) + static_cast<long long>(tc.b) * E.dU.bstride;
    const float* V = static_cast<const float*>(E.dV.ptr) + static_cast<long long>(tc.b) * E.dV.bstride;
    const float u = U[static_cast<long long>(row) * (E.dU.ld + 1)];
    float ur[EC], vr[EC];
    load_row_f32(E.dU, tc.b, row, col0, N, ur);
    load_row_f32(E.dV, tc.b, row, col0, N, vr);
#pragma unroll
    for (int j = 0; j < EC; ++j) {
      const float vj = (col0 + j < N) ? V[static_cast<long long>(col0 + j) * (E.dV.ld + 1)] : 0.0f;
      float t = fmaf(u, vr[j], ur[j] * vj);
      if (j == jd) t -= u * vj;
      v[j] = fmaf(alpha, t, v[j]);
    }
  }
  if (E.s2_ds != nullptr) {
    const long long db = static_cast<long long>(tc.b) * E.s2_d_bs;
    const float dsi = E.s2_ds[db + row] + E.s2_ds_add;
    float fs[EC], ft[EC], dtj[EC];
    load_row_any(E.s2_fs, tc.b, row, col0, N, fs);
    load_row_any(E.s2_ft, tc.b, row, col0, N, ft);
    load_vec_f32(E.s2_dt + db, col0, N, dtj);
#pragma unroll
    for (int j = 0; j < EC; ++j) {
      const float dt = dtj[j] + E.s2_dt_add;
      float t = fmaf(dsi, ft[j], fs[j] * dt);
      if (j == jd) t = fmaf(dsi, dt, t);
      v[j] = fmaf(alpha, t, v[j]);
    }
  }
  if (E.gamma != 0.0f) {
#pragma unroll
    for (int j = 0; j < EC; ++j)
      if (j == jd) v[j] += E.gamma;
  }
#pragma unroll
  for (int i = 0; i < kMaxEpiIn; ++i) {
    if (i < E.nin && i >= first_in) {
      float beta = E.in[i].beta;
      if (i == 0) {
        if (E.in0_rowcoef != nullptr) beta += E.in0_rowcoef[static_cast<long long>(tc.b) * E.in0_rowcoef_bs + row];
        if (E.in0_colcoef != nullptr) {
          // x_j += (beta + cc_j) * scale * C0(row, j)
          const float sc = E.in_scale != nullptr ? E.in_scale[tc.b] : 1.0f;
          float cc[EC], cv[EC];
          load_vec_f32(E.in0_colcoef + static_cast<long long>(tc.b) * E.in0_colcoef_bs, col0, N, cc);
          load_row_any(E.in[0], tc.b, row, col0, N, cv);
#pragma unroll
          for (int j = 0; j < EC; ++j) v[j] = fmaf((beta + cc[j]) * sc, cv[j], v[j]);
          continue;
        }
        if (E.in_scale != nullptr) beta *= E.in_scale[tc.b];
      }
      add_row(E.in[i], beta, tc.b, row, col0, N, v);
    }
  }
  if (E.ek_s != nullptr) {
    float* sp = E.ek_s + static_cast<long long>(tc.b) * E.ek_bstride + static_cast<long long>(row) * E.ek_ld + col0;
#pragma unroll
    for (int j = 0; j < EC; ++j) {
      if (col0 + j < N) {
        const float sq = v[j] * v[j];                                            // Vt.pow(2)
        const float sn = E.ek_first ? sq : fmaf(1.0f - E.ek_decay, sq, sp[j] * E.ek_decay);  // s.mul_().add_()
        sp[j] = sn;
        v[j] = v[j] / (sn + E.ek_lam);                                           // Vt / (s + lam)
      }
    }
  }
  if ((E.diag_out != nullptr || E.red_trace != nullptr) && jd >= 0 && jd < EC && col0 + jd < N) {
#pragma unroll
    for (int j = 0; j < EC; ++j) {
      if (j == jd) {
        if (E.diag_out != nullptr) E.diag_out[static_cast<long long>(tc.b) * E.diag_out_bs + row] = v[j];
        if (E.red_trace != nullptr) atomicAdd(E.red_trace + tc.b, static_cast<double>(v[j]));
      }
    }
  }
  if (E.mu_p != nullptr) {
    muon_apply_chunk(E, tc.b, row, col0, N, v, red);
#pragma unroll
    for (int o = 0; o < kMaxEpiOut; ++o)
      if (o < E.nout) store_out(E.out[o], tc.b, row, col0, N, jd, v);
    return;  // plain products only: no mirrored half
  }
  if (E.sym_diag && P.tri && !mirror) {
    // Diagonal tile: keep the lower half, written to both (i, j) and (j, i).
#pragma unroll
    for (int o = 0; o < kMaxEpiOut; ++o) {
      if (o >= E.nout) continue;
      const EpiOut& eo = E.out[o];
      const long long base = static_cast<long long>(tc.b) * eo.bstride;
#pragma unroll
      for (int j = 0; j < EC; ++j) {
        const int c = col0 + j;
        if (c >= N || c > row) continue;
        const float w = (eo.zero_diag && c == row) ? 0.0f : v[j];
        store_elem(eo, base + static_cast<long long>(row) * eo.ld + c, w);
        if (c < row) store_elem(eo, base + static_cast<long long>(c) * eo.ld + row, w);
      }
    }
  } else {
#pragma unroll
    for (int o = 0; o < kMaxEpiOut; ++o)
      if (o < E.nout) store_out(E.out[o], tc.b, row, col0, N, jd, v);
  }
  if (E.red_absmax != nullptr) {
#pragma unroll
    for (int j = 0; j < EC; ++j)
      if (col0 + j < N) red_update(red, fabsf(v[j] - (j == jd ? E.red_ident : 0.0f)));
  } else if (E.red_sumsq != nullptr) {
#pragma unroll
    for (int j = 0; j < EC; ++j)
      if (col0 + j < N) red = fmaf(v[j], v[j], red);
  }
  if (mirror && same) {
    // The full product is symmetric: the mirrored element takes the same value.
#pragma unroll
    for (int o = 0; o < kMaxEpiOut; ++o)
      if (o < E.nout && !E.out[o].lower_only) store_col(E.out[o], tc.b, row, col0, N, v);
  }
}

// ------------------------------------------------------------------ kernel
// CHUNKED (BN == 128 only): the K loop is cut into chunks of KCHUNK k-blocks,
// each accumulated into its own (double-buffered) TMEM accumulator and summed
// by the epilogue in registers with round-to-nearest fp32 adds. The tensor
// core adds every MMA result into its accumulator with truncation, so long
// K loops drift low; chunking bounds that drift independently of K.
constexpr int KCHUNK = 4;

template <int KIND, int BN, bool A_MN, bool B_MN, bool CHUNKED>
__global__ void __launch_bounds__(kGemmThreads, 1) tc_gemm_kernel(const __grid_constant__ GemmParams P) {
  using C = GemmCfg<KIND, BN>;
  constexpr int BM = C::BM;
  static_assert(!CHUNKED || BN == 128, "chunked accumulation keeps a 128-column row in registers");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, kEpilogueThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&P.mapA[0]);
    prefetch_tensormap(&P.mapB[0]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_holder;
  const int nkb = (P.K + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t armed = 0;  // bit s: stage s has been armed; bit 8+s: parity of its last arming
      for (int t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(P, t);
        if (!tile_active(P, tc.b)) continue;
        const int nv = tile_passes(P, tc.b) * nkb;
        for (int v = 0; v < nv; ++v) {
          const int pass = v / nkb;
          const int k0 = (v - pass * nkb) * C::BK;
          if (!mbar_wait_bounded(empty + stage, phase ^ 1u, abort_flag, P.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + stage, C::STAGE_BYTES);
          armed = (armed & ~(0x101u << stage)) | (1u << stage) | (phase << (8 + stage));
          const CUtensorMap* ma = &P.mapA[pass == 2 ? 1 : 0];
          const CUtensorMap* mb = &P.mapB[pass == 1 ? 1 : 0];
          uint8_t* sa = tiles + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          if (!A_MN) {
            tma_load_3d(sa, ma, full + stage, k0, tc.mt * BM, tc.b);
          } else if (P.a4d) {
            tma_load_4d(sa, ma, full + stage, 0, k0, tc.mt * BM / (128 / C::ES), tc.b);
          } else {
#pragma unroll
            for (int i = 0; i < BM * C::ES / 128; ++i)
              tma_load_3d(sa + i * C::BK * 128, ma, full + stage, tc.mt * BM + i * (128 / C::ES), k0, tc.b);
          }
          if (!B_MN) {
            tma_load_3d(sb, mb, full + stage, k0, tc.nt * BN, tc.b);
          } else if (P.b4d) {
            tma_load_4d(sb, mb, full + stage, 0, k0, tc.nt * BN / (128 / C::ES), tc.b);
          } else {
#pragma unroll
            for (int i = 0; i < BN * C::ES / 128; ++i)
              tma_load_3d(sb + i * C::BK * 128, mb, full + stage, tc.nt * BN + i * (128 / C::ES), k0, tc.b);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the last load issued into each stage land before the CTA can
        // exit (earlier loads into a stage completed before it was re-armed).
        for (int s = 0; s < C::STAGES; ++s) {
          if (!(armed & (1u << s))) continue;
          const uint32_t par = (armed >> (8 + s)) & 1u;
          const unsigned long long t0 = global_timer_ns();
          while (!mbar_try_wait(full + s, par)) {
            if (global_timer_ns() - t0 > kWaitTimeoutNs) {
              atomicCAS(P.err, 0, kErrTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t fmt = (KIND == KIND_BF16) ? 1u : 2u;
      constexpr uint32_t idesc = make_idesc(fmt, BM, BN, A_MN ? 1u : 0u, B_MN ? 1u : 0u);
      // Byte advance of the descriptor start address per MMA_K step.
      constexpr uint32_t A_STEP = A_MN ? C::MMA_K * 128 : 32;
      constexpr uint32_t B_STEP = B_MN ? C::MMA_K * 128 : 32;
      constexpr uint32_t A_LBO = A_MN ? C::BK * 128 : 16;
      constexpr uint32_t B_LBO = B_MN ? C::BK * 128 : 16;
      // MN-major 32-bit operands use the 128 B swizzle with 32 B granules (4-row atoms).
      constexpr bool MN32 = (KIND == KIND_TF32);
      constexpr uint32_t A_LAY = (A_MN && MN32) ? kSwizzle128BAtom32B : kSwizzle128B;
      constexpr uint32_t B_LAY = (B_MN && MN32) ? kSwizzle128BAtom32B : kSwizzle128B;
      constexpr uint32_t A_SBO = (A_MN && MN32) ? 512 : 1024;
      constexpr uint32_t B_SBO = (B_MN && MN32) ? 512 : 1024;
      int stage = 0;
      uint32_t phase = 0;
      int ucount = 0;  // accumulator units issued (tiles, or chunks of tiles)
      bool ok = true;
      for (int t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(P, t);
        if (!tile_active(P, tc.b)) continue;
        const int nv = tile_passes(P, tc.b) * nkb;
        const int chunk = CHUNKED ? KCHUNK : nv;
        for (int v0 = 0; v0 < nv && ok; v0 += chunk) {
          const int v1 = min(nv, v0 + chunk);
          const int acc = ucount & 1;
          const uint32_t acc_phase = (ucount >> 1) & 1;
          if (!mbar_wait_bounded(tempty + acc, acc_phase ^ 1u, abort_flag, P.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t dtmem = tmem_base + static_cast<uint32_t>(acc * BN);
          for (int v = v0; v < v1; ++v) {
            if (!mbar_wait_bounded(full + stage, phase, abort_flag, P.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            // TMA writes and tensor-core reads are both async-proxy operations ordered
            // by the mbarrier: no tcgen05 fence is needed between them.
            const uint32_t sa = smem_u32(tiles + stage * C::STAGE_BYTES);
            const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
            for (int ks = 0; ks < C::KSTEPS; ++ks) {
              const uint64_t ad = make_sw128_desc(sa + ks * A_STEP, A_LBO, A_SBO, A_LAY);
              const uint64_t bd = make_sw128_desc(sb + ks * B_STEP, B_LBO, B_SBO, B_LAY);
              const uint32_t accumulate = (v > v0 || ks > 0) ? 1u : 0u;
              if (KIND == KIND_BF16) mma_f16(dtmem, ad, bd, idesc, accumulate);
              else mma_tf32(dtmem, ad, bd, idesc, accumulate);
            }
            mma_commit(empty + stage);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          mma_commit(tfull + acc);
          ++ucount;
        }
      }
      // Wait until every MMA issued by this thread has completed.
      mma_commit(drain);
      {
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_timer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(P.err, 0, kErrTimeoutDrain);
            break;
          }
        }
      }
    }
  } else {
    // -------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    constexpr int HC = BN / EC / 2;        // chunks per column half
    const int c_lo = ((warp - 2) >> 2) * HC;  // first chunk of this warp's half
    int ucount = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x) {
      const TileCoord tc = decode_tile(P, t);
      if (!tile_active(P, tc.b)) continue;
      const int row = tc.mt * BM + q * 32 + lane;
      const bool mirror = P.tri && tc.mt != tc.nt;
      float red = 0.0f;
      epilogue_prefetch(P, tc.b, row, tc.nt * BN + c_lo * EC, HC * EC);
      if (CHUNKED) {
        const int nv = tile_passes(P, tc.b) * nkb;
        float racc[BN / 2];
#pragma unroll
        for (int j = 0; j < BN / 2; ++j) racc[j] = 0.0f;
        for (int v0 = 0; v0 < nv; v0 += KCHUNK) {
          const int acc = ucount & 1;
          const uint32_t acc_phase = (ucount >> 1) & 1;
          const bool ready = mbar_wait_bounded_sleep(tfull + acc, acc_phase, abort_flag, P.err, kErrTimeoutEpilogue);
          if (!__all_sync(0xffffffffu, ready)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (int c = 0; c < HC; ++c) {
            uint32_t r[EC];
            tmem_ld_32x16(tmem_base + lane_base + static_cast<uint32_t>(acc * BN + (c_lo + c) * EC), r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < EC; ++j) racc[c * EC + j] += __uint_as_float(r[j]);
          }
          tc_fence_before_sync();
          mbar_arrive(tempty + acc);
          ++ucount;
        }
        if (!ok) break;
        // One inlined copy of the epilogue: the chunk's registers are picked
        // by a switch over compile-time offsets (racc stays in registers).
#pragma unroll 1
        for (int c = 0; c < HC; ++c) {
          float f[EC];
          static_assert(!CHUNKED || HC == 4, "chunked epilogue: four chunks per column half");
          switch (c) {
            case 0: {
#pragma unroll
              for (int j = 0; j < EC; ++j) f[j] = racc[j];
              break;
            }
            case 1: {
#pragma unroll
              for (int j = 0; j < EC; ++j) f[j] = racc[EC + j];
              break;
            }
            case 2: {
#pragma unroll
              for (int j = 0; j < EC; ++j) f[j] = racc[2 * EC + j];
              break;
            }
            default: {
#pragma unroll
              for (int j = 0; j < EC; ++j) f[j] = racc[3 * EC + j];
              break;
            }
          }
          epilogue_chunk(P, tc, row, tc.nt * BN + (c_lo + c) * EC, mirror, f, red);
        }
      } else {
        const int acc = ucount & 1;
        const uint32_t acc_phase = (ucount >> 1) & 1;
        // Keep the warp converged for tcgen05.ld: leave together if any lane gave up.
        const bool ready = mbar_wait_bounded_sleep(tfull + acc, acc_phase, abort_flag, P.err, kErrTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, ready)) break;
        tc_fence_after_sync();
#pragma unroll 1
        for (int c = c_lo; c < c_lo + HC; ++c) {
          uint32_t r[EC];
          tmem_ld_32x16(tmem_base + lane_base + static_cast<uint32_t>(acc * BN + c * EC), r);
          tmem_ld_wait();
          float f[EC];
#pragma unroll
          for (int j = 0; j < EC; ++j) f[j] = __uint_as_float(r[j]);
          epilogue_chunk(P, tc, row, tc.nt * BN + c * EC, mirror, f, red);
        }
        tc_fence_before_sync();
        mbar_arrive(tempty + acc);
        ++ucount;
      }
      if (P.epi.red_absmax != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) red = fmaxf(red, __shfl_xor_sync(0xffffffffu, red, o));
        if (lane == 0 && red > 0.0f)
          atomicMax(reinterpret_cast<int*>(P.epi.red_absmax) + tc.b, __float_as_int(red));
      } else if (P.epi.red_sumsq != nullptr) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) red += __shfl_xor_sync(0xffffffffu, red, o);
        if (lane == 0) atomicAdd(P.epi.red_sumsq + (P.epi.red_sumsq_shared ? 0 : tc.b), static_cast<double>(red));
      }
    }
  }

  __syncwarp();
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace po
