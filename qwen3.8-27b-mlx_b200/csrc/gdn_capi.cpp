// Error reporting and version of the GDN C ABI.
#include <cstdarg>
#include <cstdio>

#include "gdn_internal.h"

namespace gdn {

namespace {
thread_local char g_err[512] = {0};
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_err[0] = 0; }

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GDN_OK;
  return fail(GDN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

}  // namespace gdn

extern "C" const char* gdn_last_error(void) { return gdn::g_err; }

extern "C" int gdn_version(void) { return 100; }  // 0.1.0
