// Shared host-side helpers of the GDN C ABI: error text, argument checks and
// launch-status translation.  Every entry point validates its arguments with
// these before it makes any CUDA call.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace gdn {

// Record a message for gdn_last_error() on this thread and return `code`.
int fail(int code, const char* fmt, ...);
// Clear the thread's last error (called at the start of every entry point).
void clear_error();
// Translate a CUDA status into GDN_OK or GDN_ERR_CUDA with the CUDA text.
int cuda_status(cudaError_t e, const char* what);

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// True when [p, p+n) and [q, q+m) share at least one byte.
inline bool overlap(const void* p, size_t n, const void* q, size_t m) {
  if (!p || !q || n == 0 || m == 0) return false;
  auto a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(q);
  return a < b + m && b < a + n;
}

// Address of this device's error word (set by kernels whose bounded waits
// give up), cached per device; GDN_OK or GDN_ERR_CUDA.
int device_error_ptr(int** out);

// cuTensorMapEncodeTiled, looked up once through the runtime's driver entry
// point (so that the library loads on a machine without a driver): *fn is
// the function, to be cast to its CUDA signature; GDN_OK or GDN_ERR_CUDA.
int tensor_map_encoder(void** fn);

constexpr int kD = 128;  // Dk = Dv, fixed by the model (TextConfig, python/qwen35.py:88-91)

}  // namespace gdn
