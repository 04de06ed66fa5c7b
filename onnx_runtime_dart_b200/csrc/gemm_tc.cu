// tcgen05 tensor-core path (16-bit operands, fp32 accumulation in TMEM).
// Until the kernel lands every MMA-mode call routes to the exact path.
#include "common.cuh"

namespace ortc {

int mma_supported_shape(int64_t, int64_t) { return 0; }

int launch_mma_nbits(ort_cuda_session*, Weight&, const float*, int64_t, float*, int64_t, int,
                     cudaStream_t) {
  return fail(ORT_CUDA_ERR_UNSUPPORTED, "MMA path not built");
}

int launch_mma_dense(ort_cuda_session*, Weight&, const float*, int64_t, bool, float*, int64_t,
                     int, float, float, const float*, int64_t, int64_t, int64_t, cudaStream_t) {
  return fail(ORT_CUDA_ERR_UNSUPPORTED, "MMA path not built");
}

}  // namespace ortc
