// MatMulNBits for callers that cannot allocate device memory.
//
// Some hosts must not allocate device memory once they are running: a
// serving process that reserves its whole memory budget at start-up, an
// application whose device memory is owned by another runtime's allocator,
// or a latency-critical path where cudaMalloc's implicit device
// synchronisation is not acceptable.  ort_cuda_matmul_nbits may grow the
// session's split-K scratch with cudaMalloc; this entry point never does.
// It runs the same decode GEMV kernels with their scratch (the split-K
// partial sums) in the file-scope array below, which every GPU that loads
// this library holds until the process exits.
//
// Host code must not use the array's name as a device address (on the host
// it is a stand-in); the device address comes from cudaGetSymbolAddress,
// taken once per device with that device current, on the first call of the
// entry point on that device.
#include <mutex>

#include "common.cuh"

namespace ortc {
namespace {

// 4 MiB of partial sums per GPU.
constexpr size_t kNoAllocPartialFloats = size_t(1) << 20;

static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartialFloats];

struct Slot {
  float* partials = nullptr;
  bool ready = false;
};
std::mutex g_mu;
Slot g_slots[64];

// Device address of the array on `device` (which must be current).  The
// lookup can load the module lazily, which would invalidate a stream
// capture in progress, so a session that is capturing gets an error
// instead when the address is not known yet.
int slot_for(int device, bool capturing, Slot** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= 64) return fail(ORT_CUDA_ERR_INVALID_ARG, "device index >= 64");
  Slot& sl = g_slots[device];
  if (!sl.ready) {
    if (capturing)
      return fail(ORT_CUDA_ERR_INVALID_ARG,
                  "the first no-allocation MatMulNBits call on a device sets it up and cannot "
                  "be captured; make one call before the capture");
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(partials)");
    sl.partials = static_cast<float*>(p);
    sl.ready = true;
  }
  *out = &sl;
  return ORT_CUDA_OK;
}

}  // namespace
}  // namespace ortc

using namespace ortc;

extern "C" ORT_CUDA_API int ort_cuda_matmul_nbits_noalloc(ort_cuda_session* s, const char* name,
                                                          const float* A, int64_t M, float* Y) {
  ORTC_CHECK(s && name && A && Y, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  const Weight& w = it->second;
  ORTC_CHECK(w.kind == W_NBITS, ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + name + "' is not a MatMulNBits weight");
  ORTC_CHECK(s->world == 1, ORT_CUDA_ERR_UNSUPPORTED,
             "no-allocation MatMulNBits runs on single-GPU sessions only");
  ORTC_CHECK(s->mode != ORT_CUDA_MODE_STRICT, ORT_CUDA_ERR_UNSUPPORTED,
             "no-allocation MatMulNBits runs the exact-mode GEMV; this session's mode is "
             "STRICT, whose bit-for-bit reference rounding it does not reproduce");
  ORTC_CHECK(M >= 1 && M <= 4, ORT_CUDA_ERR_INVALID_ARG,
             "no-allocation MatMulNBits takes 1 <= M <= 4, got M=" + std::to_string(M));
  ORTC_CHECK(tc_gemv_ok(w, M), ORT_CUDA_ERR_UNSUPPORTED,
             "no-allocation MatMulNBits needs 32 <= block_size <= 512");
  // The plan the regular entry point would use, unless its partial sums do
  // not fit the static scratch; then the heuristic's choice among the plans
  // that fit.  Every plan gives the same bits, and the tile-major plan
  // needs no partial sums, so only a shape no plan fits is refused.
  const int plan = tc_gemv_plan(w, M, s->sm_count, kNoAllocPartialFloats);
  if (plan < 0) {
    const size_t pf = tc_gemv_partial_floats(w, M, s->sm_count, tc_gemv_plan(w, M, s->sm_count));
    ORTC_CHECK(false, ORT_CUDA_ERR_INVALID_ARG,
               "no-allocation MatMulNBits: this shape needs " + std::to_string(pf) +
                   " partial floats; the static scratch holds " +
                   std::to_string(kNoAllocPartialFloats));
  }
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != s->device) ORTC_CUDA(cudaSetDevice(s->device));
  Slot* sl = nullptr;
  // The array keeps the previous call's contents; nothing in it needs a
  // starting value (every partial is written before it is read).
  int rc = slot_for(s->device, s->capturing, &sl);
  if (rc == ORT_CUDA_OK)
    rc = launch_tc_gemv(w, plan, A, M, Y, w.nl, sl->partials, s->err_dev, s->sm_count,
                        s->stream, &s->launches, nullptr);
  if (prev >= 0 && prev != s->device) cudaSetDevice(prev);
  return rc;
}
