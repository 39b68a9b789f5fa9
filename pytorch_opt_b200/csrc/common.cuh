// Host-side plumbing shared by the op drivers: status codes, the per-thread
// error message behind po_last_error(), the device error word that kernels
// write when a bounded wait gives up, and small launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/pytorch_opt_b200.h"

namespace po {

// Record a message for po_last_error() and return the status code.
int set_error(int code, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);

// Address (on the current device) of the library's device error word.
int* device_error_word();
// Streaming-multiprocessor count of the current device.
int sm_count();

inline int cdiv(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }
inline long long round_up(long long a, long long b) { return (a + b - 1) / b * b; }

// Element type codes used across the C ABI (see include/pytorch_opt_b200.h).
inline int dtype_size(int dt) {
  switch (dt) {
    case PO_F32: return 4;
    case PO_BF16: return 2;
    case PO_F16: return 2;
    case PO_F64: return 8;
    default: return 0;
  }
}

// Bump allocator over a caller-provided device workspace.
struct Arena {
  char* base;
  size_t size;
  size_t used = 0;
  bool dry;  // size-query mode: only count bytes
  Arena(void* b, size_t s) : base(static_cast<char*>(b)), size(s), dry(b == nullptr) {}
  void* take(size_t bytes) {
    used = static_cast<size_t>(round_up(static_cast<long long>(used), 256));
    void* p = dry ? nullptr : base + used;
    used += bytes;
    return p;
  }
  bool overflow() const { return !dry && used > size; }
};

}  // namespace po
