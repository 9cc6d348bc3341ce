// Peer-memory plumbing for the expert-parallel exchange: CUDA IPC handles for
// receive buffers and device-to-device copies that the copy engines execute.
// With the "peer" transport rows cross NVLink as plain DMA copies from this
// GPU into another GPU's buffer; the fused dispatch/combine kernels
// (ep_fused.cu) instead store to / load from the mapped peer buffers with
// ordinary vector accesses (no TMA, no bulk copies).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <mutex>

#include "moe_common.cuh"

namespace moe {
namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_ipc_get_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  MOE_REQUIRE(dev_ptr != nullptr && handle_out != nullptr && offset_out != nullptr,
              "ipc_get_handle: null argument");
  auto range = address_range_fn();
  if (range == nullptr) {
    set_last_error("ipc_get_handle: cuMemGetAddressRange unavailable");
    return MOE_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  if (r != CUDA_SUCCESS) {
    set_last_error("ipc_get_handle: cuMemGetAddressRange failed (%d)", static_cast<int>(r));
    return MOE_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  MOE_CUDA_CALL(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return MOE_OK;
}

extern "C" int moe_ipc_open_handle(const void* handle, void** base_out) {
  MOE_REQUIRE(handle != nullptr && base_out != nullptr, "ipc_open_handle: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  MOE_CUDA_CALL(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                "cudaIpcOpenMemHandle");
  *base_out = p;
  return MOE_OK;
}

extern "C" int moe_ipc_close_handle(void* base) {
  MOE_REQUIRE(base != nullptr, "ipc_close_handle: null pointer");
  MOE_CUDA_CALL(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
  return MOE_OK;
}

extern "C" int moe_copy_async(void* dst, const void* src, size_t bytes, moe_stream_t stream) {
  if (bytes == 0) return MOE_OK;
  MOE_REQUIRE(dst != nullptr && src != nullptr, "copy_async: null pointer");
  MOE_CUDA_CALL(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault,
                                reinterpret_cast<cudaStream_t>(stream)),
                "cudaMemcpyAsync");
  return MOE_OK;
}
