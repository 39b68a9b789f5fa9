// Tensor-map encoding, kernel instantiation and launch of the tcgen05 GEMM,
// plus the library-wide error plumbing.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "gemm_launch.cuh"
#include "gemm_pair_launch.cuh"

namespace po {

// ----------------------------------------------------------- error plumbing
static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PO_OK;
  return set_error(PO_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Written by kernels whose bounded waits gave up; read by po_device_error().
__device__ int g_device_error = 0;

static constexpr int kMaxDevices = 64;

int* device_error_word() {
  static int* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

// Wait-cycle counters of the two-SM kernel, filled while po_gemm_profile has
// switched them on (measurement only).
__device__ unsigned long long g_gemm_prof[kProfSlots];
static std::atomic<bool> g_gemm_prof_on{false};

unsigned long long* gemm_prof_word() {
  if (!g_gemm_prof_on.load(std::memory_order_relaxed)) return nullptr;
  static unsigned long long* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_prof) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<unsigned long long*>(p);
  }
  return ptrs[dev];
}

int sm_count() {
  static int counts[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

// ------------------------------------------------------------- tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Map over a [batch][outer][inner] array, box = {box_inner, box_outer, 1},
// 128-byte swizzle, zero fill out of bounds.
static int encode_map(CUtensorMap* map, const MatView& v, int batch, int box_inner, int box_outer,
                      CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(PO_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int es = dtype_size(v.dtype);
  if (v.dtype != PO_BF16 && v.dtype != PO_F32) return set_error(PO_ERR_ARG, "operand dtype must be bf16 or fp32");
  if (reinterpret_cast<uintptr_t>(v.ptr) % 16 != 0 || (v.ld * es) % 16 != 0 ||
      (batch > 1 && (v.bstride * es) % 16 != 0))
    return set_error(PO_ERR_ARG, "tensor-core operand needs 16-byte aligned base and pitches");
  const long long bstride_bytes = batch > 1 ? v.bstride * es : v.ld * es * (v.rows > 0 ? v.rows : 1);
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(v.cols), static_cast<cuuint64_t>(v.rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(v.ld * es), static_cast<cuuint64_t>(bstride_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, v.dtype == PO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                  const_cast<void*>(v.ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu, ld %lld", int(r),
             (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2], v.ld);
    return set_error(PO_ERR_CUDA, buf);
  }
  return PO_OK;
}

// MN-major operand stored [batch][K][MN] viewed as [batch][MN / w][K][w] with
// w = 128 B of elements, so that one box {w, box_k, nblk, 1} brings all of a
// stage's MN blocks in one copy. Only when MN is a multiple of w (the view
// then covers exactly the stored elements). Returns 1 when not applicable.
static int encode_map_mn4d(CUtensorMap* map, const MatView& v, int batch, int box_k, int nblk,
                           CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) return 1;
  const int es = dtype_size(v.dtype);
  const int w = 128 / es;
  if (v.cols % w != 0 || reinterpret_cast<uintptr_t>(v.ptr) % 16 != 0 || (v.ld * es) % 16 != 0 ||
      (batch > 1 && (v.bstride * es) % 16 != 0))
    return 1;
  const long long bstride_bytes = batch > 1 ? v.bstride * es : v.ld * es * (v.rows > 0 ? v.rows : 1);
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(v.rows),
                        static_cast<cuuint64_t>(v.cols / w), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(v.ld * es), 128, static_cast<cuuint64_t>(bstride_bytes)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(w), static_cast<cuuint32_t>(box_k), static_cast<cuuint32_t>(nblk), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, v.dtype == PO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                  const_cast<void*>(v.ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 1;
}

EpiIn epi_in(const void* ptr, int in_kind, long long ld, long long bstride, float beta) {
  EpiIn e{};
  e.ptr = ptr;
  e.kind = in_kind;
  e.ld = ld;
  e.bstride = bstride;
  e.beta = beta;
  const int es = in_kind == IN_F32 ? 4 : 2;
  e.vec = (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && (ld * es) % 16 == 0 && (bstride * es) % 16 == 0;
  return e;
}

EpiOut epi_out(void* ptr, int out_kind, long long ld, long long bstride, bool trans) {
  EpiOut e{};
  e.ptr = ptr;
  e.kind = out_kind;
  e.ld = ld;
  e.bstride = bstride;
  e.trans = trans ? 1 : 0;
  const int es = (out_kind == OUT_F32 || out_kind == OUT_TF32 || out_kind == OUT_TF32_LO) ? 4
                 : (out_kind == OUT_F64 ? 8 : 2);
  e.vec = (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && (ld * es) % 16 == 0 && (bstride * es) % 16 == 0;
  return e;
}

// Tile shape choice. A one-SM CTA streams 128 x BN operand panels per k-block
// for its own 128 x BN tile; a pair of SMs computing one 256 x 256 tile
// streams half as many bytes per SM per MMA, so pair tiles run closer to the
// tensor-core rate. They are four times larger than 128 x 128 tiles, so on
// small problems the one-SM kernel can still win by filling more SMs. The
// estimate: per-SM work of one tile x waves, divided by the measured relative
// throughput of each tile shape (128x128: 0.55, 128x256: 0.7, pair: 0.85).
// PO_GEMM_PAIR=0/1 in the environment forces the choice (for measurement).
static int pair_override() {
  const char* e = getenv("PO_GEMM_PAIR");
  if (e == nullptr || *e == 0) return -1;
  return atoi(e) != 0 ? 1 : 0;
}

static bool use_pair(const GemmDesc& d, int bn) {
  int want = d.pair;
  if (want < 0) want = pair_override();
  if (want >= 0) return want != 0;
  const long long sms = sm_count();
  auto tiles = [&](int tm, int tn) {
    const long long a = cdiv(d.M, tm), b = cdiv(d.N, tn);
    return (d.tri ? a * (a + 1) / 2 : a * b) * d.batch;
  };
  const long long t1 = tiles(128, bn);
  const long long t2 = tiles(256, 256);
  const double eff1 = bn == 256 ? 0.7 : 0.55;
  const double cost1 = static_cast<double>((t1 + sms - 1) / sms) * 128.0 * bn / eff1;
  const double cost2 = static_cast<double>((t2 + sms / 2 - 1) / (sms / 2)) * 128.0 * 256.0 / 0.85;
  return cost2 <= cost1;
}

bool gemm_uses_pair(const GemmDesc& d) {
  int bn = d.bn;
  if (bn == 0) bn = (d.tri || d.N <= 128) ? 128 : 256;
  if (d.tri || d.chunked) bn = 128;
  return !d.chunked && use_pair(d, bn);
}

int launch_gemm(const GemmDesc& d, cudaStream_t stream) {
  if (d.M <= 0 || d.N <= 0 || d.batch <= 0) return PO_OK;
  if (d.K <= 0) return set_error(PO_ERR_ARG, "launch_gemm: K must be positive");
  if (d.tri && d.M != d.N) return set_error(PO_ERR_ARG, "launch_gemm: triangular product needs M == N");
  if (d.epi.ek_s != nullptr && d.tri) return set_error(PO_ERR_ARG, "launch_gemm: the EKFAC epilogue needs a plain product");
  if (d.epi.red_sumsq != nullptr && (d.tri || d.epi.red_absmax != nullptr))
    return set_error(PO_ERR_ARG, "launch_gemm: the sum-of-squares reduction needs a plain product");
  if (d.npass != 1 && d.npass != 3) return set_error(PO_ERR_ARG, "launch_gemm: npass must be 1 or 3");
  const int want_dtype = d.kind == KIND_BF16 ? PO_BF16 : PO_F32;
  const int nmaps = d.npass == 3 ? 2 : 1;
  for (int i = 0; i < nmaps; ++i)
    if (d.a[i].dtype != want_dtype || d.b[i].dtype != want_dtype)
      return set_error(PO_ERR_ARG, "launch_gemm: operand dtype does not match the product kind");
  int bn = d.bn;
  if (bn == 0) bn = (d.tri || d.N <= 128) ? 128 : 256;
  if (d.tri || d.chunked) bn = 128;
  const bool pair = !d.chunked && use_pair(d, bn);
  const int tm = pair ? 256 : 128;
  if (pair) bn = 256;

  GemmParams P;
  memset(&P, 0, sizeof(P));
  const int es = d.kind == KIND_BF16 ? 2 : 4;
  const int bk = 128 / es;
  // Rows of A and of B one CTA loads per stage; the two-SM kernel's stages
  // hold two 128-byte K atoms (MN-major boxes span 2 * bk rows of K).
  const int kbox = pair ? 2 * bk : bk;
  const int a_rows = 128, b_rows = pair ? bn / 2 : bn;
  // MN-major 32-bit operands: 128 B swizzle with 32 B granules (the only
  // shared-memory layout the tensor cores accept for MN-major tf32).
  const CUtensorMapSwizzle mn_swz = es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  // PO_GEMM_MN4D=0 in the environment forces the block-by-block loads (for measurement).
  const char* mn4d_env = getenv("PO_GEMM_MN4D");
  const bool no_mn4d = d.no_mn4d || (mn4d_env != nullptr && mn4d_env[0] == '0');
  P.a4d = !d.a_kmajor && !no_mn4d;
  P.b4d = !d.b_kmajor && !no_mn4d;
  for (int i = 0; i < nmaps; ++i) {
    if (P.a4d && encode_map_mn4d(&P.mapA[i], d.a[i], d.batch, kbox, a_rows * es / 128, mn_swz)) P.a4d = 0;
    if (P.b4d && encode_map_mn4d(&P.mapB[i], d.b[i], d.batch, kbox, b_rows * es / 128, mn_swz)) P.b4d = 0;
  }
  for (int i = 0; i < 2; ++i) {
    const int src = i < nmaps ? i : 0;
    int r = 0;
    // A: logical M x K.
    if (d.a_kmajor) r = encode_map(&P.mapA[i], d.a[src], d.batch, bk, a_rows);
    else if (!P.a4d) r = encode_map(&P.mapA[i], d.a[src], d.batch, 128 / es, kbox, mn_swz);
    else if (i >= nmaps) P.mapA[i] = P.mapA[0];
    if (r) return r;
    if (d.b_kmajor) r = encode_map(&P.mapB[i], d.b[src], d.batch, bk, b_rows);
    else if (!P.b4d) r = encode_map(&P.mapB[i], d.b[src], d.batch, 128 / es, kbox, mn_swz);
    else if (i >= nmaps) P.mapB[i] = P.mapB[0];
    if (r) return r;
  }
  P.M = d.M;
  P.N = d.N;
  P.K = d.K;
  P.batch = d.batch;
  P.tiles_m = cdiv(d.M, tm);
  P.tiles_n = cdiv(d.N, bn);
  P.tri = d.tri ? 1 : 0;
  // Raster band height (8 measured best on the Newton-Schulz products:
  // 4, 16 and 32 all read more from DRAM).
  P.group = 8;
  P.tiles_per_batch = d.tri ? P.tiles_m * (P.tiles_m + 1) / 2 : P.tiles_m * P.tiles_n;
  const long long total = static_cast<long long>(P.tiles_per_batch) * d.batch;
  if (total > 0x7fffffffLL) return set_error(PO_ERR_ARG, "launch_gemm: too many tiles");
  P.total_tiles = static_cast<int>(total);
  P.npass = d.npass;
  P.active = d.active;
  P.passes = d.passes;
  // PO_GEMM_DYN=0 in the environment forces the static schedule (for measurement).
  const char* dyn_env = getenv("PO_GEMM_DYN");
  P.sched = (pair && !(dyn_env != nullptr && dyn_env[0] == '0')) ? d.sched : nullptr;
  P.err = device_error_word();
  if (P.err == nullptr) return set_error(PO_ERR_CUDA, "device error word unavailable");
  P.prof = pair ? gemm_prof_word() : nullptr;
  // The epilogue's L2 prefetch of the rows it reads is off: measured on the
  // power-capped Llama step it cost 1-2 % (334-336 ms without, 338-339 ms
  // with, same box). PO_GEMM_PREFETCH=1 in the environment turns it on (for
  // measurement).
  const char* pf_env = getenv("PO_GEMM_PREFETCH");
  P.no_prefetch = (pf_env != nullptr && pf_env[0] == '1') ? 0 : 1;
  P.epi = d.epi;

  const bool a_mn = !d.a_kmajor, b_mn = !d.b_kmajor;
  if (pair) {
    return d.kind == KIND_BF16 ? dispatch_pair<KIND_BF16>(P, a_mn, b_mn, stream)
                               : dispatch_pair<KIND_TF32>(P, a_mn, b_mn, stream);
  }
  if (d.chunked) {
    return d.kind == KIND_BF16 ? dispatch_major<KIND_BF16, 128, true>(P, a_mn, b_mn, stream)
                               : dispatch_major<KIND_TF32, 128, true>(P, a_mn, b_mn, stream);
  }
  if (d.kind == KIND_BF16) {
    return bn == 128 ? dispatch_major<KIND_BF16, 128, false>(P, a_mn, b_mn, stream)
                     : dispatch_major<KIND_BF16, 256, false>(P, a_mn, b_mn, stream);
  }
  return bn == 128 ? dispatch_major<KIND_TF32, 128, false>(P, a_mn, b_mn, stream)
                   : dispatch_major<KIND_TF32, 256, false>(P, a_mn, b_mn, stream);
}

}  // namespace po

// ------------------------------------------------------------------ C ABI
extern "C" const char* po_last_error(void) { return po::g_last_error.c_str(); }

extern "C" int po_device_error(int reset) {
  int* p = po::device_error_word();
  if (p == nullptr) return -1;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (reset && v != 0) cudaMemset(p, 0, sizeof(int));
  return v;
}

extern "C" int po_gemm_profile(int enable, unsigned long long* out, int n) {
  if (out != nullptr) {
    if (n < 0 || n > po::kProfSlots) return po::set_error(PO_ERR_ARG, "po_gemm_profile: n out of range");
    void* p = nullptr;
    if (int r = po::check_cuda(cudaGetSymbolAddress(&p, po::g_gemm_prof), "po_gemm_profile")) return r;
    if (int r = po::check_cuda(cudaDeviceSynchronize(), "po_gemm_profile")) return r;
    if (n > 0)
      if (int r = po::check_cuda(cudaMemcpy(out, p, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost),
                                 "po_gemm_profile"))
        return r;
    if (int r = po::check_cuda(cudaMemset(p, 0, po::kProfSlots * sizeof(unsigned long long)), "po_gemm_profile"))
      return r;
  }
  po::g_gemm_prof_on.store(enable != 0);
  return PO_OK;
}

extern "C" const char* po_version(void) { return "pytorch_opt_b200 0.1 (sm_100a)"; }
