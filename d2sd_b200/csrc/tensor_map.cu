// Host-side TMA descriptor encoding shared by the kernels.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace d2sd {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}
}  // namespace

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      const char* what) {
  auto fn = get_encode_fn();
  if (!fn) return fail(D2SD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const uint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult res = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims,
                    strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) {
    return fail(D2SD_ERR_INVALID_ARGUMENT, std::string("cuTensorMapEncodeTiled failed for ") +
                                               what + " (CUresult " +
                                               std::to_string(static_cast<int>(res)) + ")");
  }
  return D2SD_OK;
}

}  // namespace d2sd
