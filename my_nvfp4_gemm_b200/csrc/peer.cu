// peer.cu — sharing device buffers between the processes of one node (one process per GPU), so
// that a kernel on one GPU can store into another GPU's buffer over NVLink.
//
// A buffer handed out by an allocator (torch's caching allocator, for one) usually sits inside
// a larger device allocation; CUDA IPC handles name whole allocations. Export therefore finds
// the allocation base and returns the handle plus the buffer's offset in it; open maps the
// allocation on the current device (peer access enabled lazily) and adds the offset back.
#include <cstdint>
#include <cstring>
#include <cuda.h>

#include "capi_util.h"

namespace {

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = []() -> GetAddressRangeFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<GetAddressRangeFn>(p);
  }();
  return fn;
}

}  // namespace

extern "C" {

int nvfp4_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return NVFP4_ERR_INVALID_VALUE;
  GetAddressRangeFn range = address_range_fn();
  if (!range) return NVFP4_ERR_NO_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return NVFP4_ERR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return nvfp4::status_from_cuda(e);
  static_assert(sizeof(h) == NVFP4_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return NVFP4_OK;
}

int nvfp4_ipc_open(const void* handle, int64_t offset, void** ptr_out) {
  if (!handle || !ptr_out || offset < 0) return NVFP4_ERR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return nvfp4::status_from_cuda(e);
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return NVFP4_OK;
}

int nvfp4_ipc_close(void* ptr, int64_t offset) {
  if (!ptr || offset < 0) return NVFP4_ERR_INVALID_VALUE;
  return nvfp4::status_from_cuda(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset));
}

}  // extern "C"
