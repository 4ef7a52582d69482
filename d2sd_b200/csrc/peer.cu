// CUDA IPC helpers for the head-sharded output exchange of d2sd_suffix_merge_gather:
// each rank exports its output buffer and arrival counter, opens its peers' and
// hands the resulting device pointers to the kernel, which stores rows and
// increments counters over NVLink. Plain point-to-point mappings (no multicast
// objects).
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace d2sd {
namespace {
PFN_cuMemGetAddressRange_v3020 get_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 3020, cudaEnableDefault,
                                         &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
    }
  });
  return fn;
}
}  // namespace
}  // namespace d2sd

extern "C" int d2sd_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  using namespace d2sd;
  if (!ptr || !handle_out || !offset_out)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_ipc_handle: null argument");
  auto range = get_range_fn();
  if (!range) return fail(D2SD_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_ipc_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return fail(D2SD_ERR_CUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - base);
  return D2SD_OK;
}

extern "C" int d2sd_ipc_open(const void* handle, void** base_out) {
  using namespace d2sd;
  if (!handle || !base_out) return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return fail(D2SD_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return D2SD_OK;
}

extern "C" int d2sd_ipc_close(void* base) {
  using namespace d2sd;
  if (!base) return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_ipc_close: null argument");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess)
    return fail(D2SD_ERR_CUDA, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return D2SD_OK;
}
