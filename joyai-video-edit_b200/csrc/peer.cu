// Peer-memory plumbing for the sequence-parallel exchange fused into the FP8
// GEMM (jo_fp8_scaled_mm_scatter): each rank exports a CUDA IPC handle for its
// exchange buffer, the other ranks of the node open it and pass the mapped
// base pointers to the GEMM, whose epilogue then stores straight into the
// owning rank's memory over NVLink.
//
// Legacy CUDA IPC (cudaIpcGetMemHandle / cudaIpcOpenMemHandle) is used on
// purpose: it maps plain device memory peer-to-peer and creates no NVLink
// multicast object.  The handle names the whole cudaMalloc allocation that
// holds the pointer, so the byte offset of the pointer inside it is exported
// beside the handle.
#include "jo_common.cuh"

#include <cuda.h>
#include <string.h>

namespace jo {
namespace {

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn get_address_range() {
  static GetAddressRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

}  // namespace
}  // namespace jo

extern "C" {

// Exports the IPC handle (64 bytes, written to handle_out) of the allocation
// holding dev_ptr and the byte offset of dev_ptr inside that allocation.
int jo_ipc_get_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  using namespace jo;
  JO_REQUIRE(dev_ptr && handle_out && offset_out, JO_ERR_INVALID, "jo_ipc_get_handle: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  GetAddressRangeFn range = get_address_range();
  JO_REQUIRE(range != nullptr, JO_ERR_CUDA, "jo_ipc_get_handle: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) {
    set_error("jo_ipc_get_handle: %p is not device memory of this context", dev_ptr);
    return JO_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("jo_ipc_get_handle: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
    return JO_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<uintptr_t>(dev_ptr) - (uintptr_t)base);
  return JO_OK;
}

// Maps a peer's allocation (64-byte handle from jo_ipc_get_handle on another
// process of this node) into this process on the current device; *base_out
// receives the mapped base (add the exported offset).  Peer access is enabled
// lazily by the driver.
int jo_ipc_open(const void* handle, void** base_out) {
  using namespace jo;
  JO_REQUIRE(handle && base_out, JO_ERR_INVALID, "jo_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("jo_ipc_open: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
    return JO_ERR_CUDA;
  }
  *base_out = p;
  return JO_OK;
}

// Unmaps a base pointer returned by jo_ipc_open.
int jo_ipc_close(void* base) {
  using namespace jo;
  JO_REQUIRE(base, JO_ERR_INVALID, "jo_ipc_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("jo_ipc_close: cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(e));
    return JO_ERR_CUDA;
  }
  return JO_OK;
}

}  // extern "C"
