// CUDA IPC helpers for head-sharded layers whose kernels write into other
// ranks' buffers (gdn_chunked_norm_gather_ws): a rank exports a device
// pointer as (handle of its allocation, offset), a peer process opens it with
// its own device current, so the mapping lives in that device's context and
// peer access from it is enabled.  Plain peer mappings; no multicast object.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "gdn_internal.h"

using namespace gdn;

extern "C" int gdn_ipc_export(const void* ptr, void* handle_out, size_t* offset_out) {
  clear_error();
  if (!ptr || !handle_out || !offset_out) return fail(GDN_ERR_NULL, "ptr, handle_out and offset_out are required");
  // the allocation's base, through the runtime's driver entry point so that
  // the library does not link the driver library (it loads without a GPU)
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  int rc = cuda_status(cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &q),
                       "driver entry point cuMemGetAddressRange");
  if (rc != GDN_OK) return rc;
  if (!fn || q != cudaDriverEntryPointSuccess) return fail(GDN_ERR_CUDA, "cuMemGetAddressRange not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (reinterpret_cast<RangeFn>(fn)(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(GDN_ERR_CUDA, "cuMemGetAddressRange failed for %p", ptr);
  cudaIpcMemHandle_t h;
  rc = cuda_status(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (rc != GDN_OK) return rc;
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return GDN_OK;
}

extern "C" int gdn_ipc_open(const void* handle, size_t offset, void** base_out, void** ptr_out) {
  clear_error();
  if (!handle || !base_out || !ptr_out) return fail(GDN_ERR_NULL, "handle, base_out and ptr_out are required");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  int rc = cuda_status(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  if (rc != GDN_OK) return rc;
  *base_out = base;
  *ptr_out = static_cast<unsigned char*>(base) + offset;
  return GDN_OK;
}

extern "C" int gdn_ipc_close(void* base) {
  clear_error();
  if (!base) return GDN_OK;
  return cuda_status(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}
