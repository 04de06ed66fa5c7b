// Host side of TMA: tensor-map encoding via the runtime's driver entry
// point (no link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace ortc {

int encode_tma_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0,
                  uint64_t d1, uint64_t stride1, uint32_t b0, uint32_t b1,
                  CUtensorMapSwizzle swz) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) return fail(ORT_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride1};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ORT_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) +
                                       ")");
  return ORT_CUDA_OK;
}

}  // namespace ortc
