// Measured fp32 FFMA throughput of the session's GPU: the denominator of
// the exact mode's CUDA-core roofline (the dense fp32 Gemm/MatMul of the
// exact and strict modes runs on FFMA, not on tensor cores).  No
// counterpart in the reference, which has no device.
//
// Every thread runs kChains independent multiply-add chains (enough to
// cover the FFMA latency with every warp slot of the SM filled), and the
// grid holds 8 CTAs of 256 threads per SM.  The values stay finite and the
// result is stored only under a condition the host never meets, so the
// compiler keeps every FFMA.  Timed with CUDA events on the session stream
// after one untimed launch.
#include "common.cuh"

namespace ortc {
namespace {

constexpr int kChains = 16;
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) ffma_probe_kernel(int iters, float b, float c,
                                                              float never, float* sink) {
  float a[kChains];
#pragma unroll
  for (int i = 0; i < kChains; i++) a[i] = (float)(threadIdx.x + i) * 1e-3f;
  for (int it = 0; it < iters; it++) {
#pragma unroll
    for (int r = 0; r < 8; r++) {
#pragma unroll
      for (int i = 0; i < kChains; i++) a[i] = fmaf(a[i], b, c);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kChains; i++) s += a[i];
  if (s == never) sink[blockIdx.x * kThreads + threadIdx.x] = s;
}

}  // namespace
}  // namespace ortc

using namespace ortc;

extern "C" ORT_CUDA_API int ort_cuda_probe_ffma(ort_cuda_session* s, double* tflops) {
  ORTC_CHECK(s && tflops, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG, "cannot probe during a capture");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != s->device) ORTC_CUDA(cudaSetDevice(s->device));
  const int blocks = s->sm_count * 8, iters = 4096;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int rc = ORT_CUDA_OK;
  float ms = 0.f;
  cudaError_t e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  for (int rep = 0; rep < 2 && e == cudaSuccess; rep++) {
    if (rep == 1) e = cudaEventRecord(e0, s->stream);
    if (e == cudaSuccess) {
      ffma_probe_kernel<<<blocks, kThreads, 0, s->stream>>>(iters, 0.9999999f, 1e-7f, -1.0f,
                                                             nullptr);
      e = cudaGetLastError();
    }
    if (rep == 1 && e == cudaSuccess) e = cudaEventRecord(e1, s->stream);
  }
  if (e == cudaSuccess) e = cudaEventSynchronize(e1);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  if (e != cudaSuccess) rc = cuda_fail(e, "ffma probe");
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (prev >= 0 && prev != s->device) cudaSetDevice(prev);
  if (rc) return rc;
  const double flops = 2.0 * kChains * 8.0 * iters * (double)blocks * kThreads;
  *tflops = flops / (ms * 1e-3) / 1e12;
  return ORT_CUDA_OK;
}
