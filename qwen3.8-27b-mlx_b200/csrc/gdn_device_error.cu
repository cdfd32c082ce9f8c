// The library's device-side error word (one per device that loads the
// library).  Kernels with bounded waits receive its address and set it when a
// wait gives up; gdn_take_device_error() reads and clears it.
#include <cuda_runtime.h>

#include <mutex>

#include "gdn_internal.h"

namespace gdn {

__device__ int g_device_error = 0;

int device_error_ptr(int** out) {
  static int* cache[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != GDN_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev & 63]) {
    void* p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_device_error), "device error word address");
    if (rc != GDN_OK) return rc;
    cache[dev & 63] = static_cast<int*>(p);
  }
  *out = cache[dev & 63];
  return GDN_OK;
}

}  // namespace gdn

extern "C" int gdn_take_device_error(void* stream, int* code) {
  gdn::clear_error();
  if (!code) return gdn::fail(GDN_ERR_NULL, "code is NULL");
  int* word = nullptr;
  int rc = gdn::device_error_ptr(&word);
  if (rc != GDN_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  rc = gdn::cuda_status(cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, st), "read device error word");
  if (rc != GDN_OK) return rc;
  rc = gdn::cuda_status(cudaStreamSynchronize(st), "synchronize");
  if (rc != GDN_OK) return rc;
  if (v != 0) {
    rc = gdn::cuda_status(cudaMemsetAsync(word, 0, sizeof(int), st), "clear device error word");
    if (rc != GDN_OK) return rc;
    rc = gdn::cuda_status(cudaStreamSynchronize(st), "synchronize");
    if (rc != GDN_OK) return rc;
  }
  *code = v;
  return GDN_OK;
}
