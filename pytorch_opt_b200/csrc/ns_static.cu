// Newton–Schulz for callers that cannot allocate device memory.
//
// po_newton_schulz() needs a caller-provided workspace. Some callers have no
// way to provide one: code running inside a host framework that owns every
// byte of device memory through its own pool (a cudaMalloc there bypasses the
// pool's accounting and synchronises the device in the middle of a step), or
// plug-in code that is handed device pointers but no allocator. For them this
// entry point runs the same computation on a scratch area that lives in the
// library itself: a file-scope device array of fixed size, reserved on every
// GPU that loads the library until the process exits. It calls no
// cudaMalloc / cudaFree and no allocating library routine.
#include <mutex>
#include <string>

#include "common.cuh"

// Scratch shared by every call on a device (it fits, for example, one
// 1024 x 1024 matrix, or a batch of small ones; see the header).
static __device__ __align__(256) unsigned char g_ns_scratch[PO_NS_STATIC_SCRATCH_BYTES];

namespace po {
namespace {

constexpr int kMaxScratchDevices = 64;

// Device address of g_ns_scratch on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up
// once per device with cudaGetSymbolAddress (with that device current).
int scratch_address(void** out) {
  static void* ptrs[kMaxScratchDevices] = {};
  static std::mutex mu;
  int dev = 0;
  int r = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (r) return r;
  if (dev < 0 || dev >= kMaxScratchDevices) return set_error(PO_ERR_UNSUPPORTED, "newton_schulz_static: device id");
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    r = check_cuda(cudaGetSymbolAddress(&p, g_ns_scratch), "cudaGetSymbolAddress(newton_schulz scratch)");
    if (r) return r;
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return PO_OK;
}

}  // namespace
}  // namespace po

using namespace po;

extern "C" int po_newton_schulz_static(const void* G, int dtype, long long batch, long long rows, long long cols,
                                       long long ld, long long bstride, void* out, long long out_ld,
                                       long long out_bstride, int steps, float a, float b, float c, float eps,
                                       int tf32_tail, void* stream) {
  if (batch < 0 || rows < 0 || cols < 0) return set_error(PO_ERR_ARG, "newton_schulz_static: negative size");
  if (batch == 0 || rows == 0 || cols == 0) return PO_OK;
  const size_t need = po_ns_workspace_bytes(batch, rows, cols);
  if (need > static_cast<size_t>(PO_NS_STATIC_SCRATCH_BYTES)) {
    return set_error(PO_ERR_ARG, "newton_schulz_static: this problem needs " + std::to_string(need) +
                                     " bytes of scratch, more than the library's built-in " +
                                     std::to_string(PO_NS_STATIC_SCRATCH_BYTES) +
                                     " bytes; use po_newton_schulz with a workspace");
  }
  void* scratch = nullptr;
  const int r = scratch_address(&scratch);
  if (r) return r;
  // The driver zeroes what must start at zero (the per-matrix norms) at the
  // start of every call and writes every other buffer before reading it.
  return po_newton_schulz(G, dtype, batch, rows, cols, ld, bstride, out, out_ld, out_bstride, steps, a, b, c, eps,
                          tf32_tail, scratch, static_cast<size_t>(PO_NS_STATIC_SCRATCH_BYTES), stream);
}
