// DynamicQuantizeLinear on the device (opDynamicQuantizeLinear,
// lib/src/onnx_ops.dart:2556-2580): the uint8 input of MatMulInteger in the
// int8 dynamic-quantisation path, so the chain stays on the GPU.
//
// The reference takes the range [min(0, min x), max(0, max x)] with plain
// comparisons (a NaN never updates it), then, in double arithmetic rounded
// to float32 where it stores: scale = fp32((mx - mn) / 255), zero point =
// round-half-even(clamp(fp32(-mn / scale), 0, 255)), and per element
// y = saturate(round-half-even(fp32(x / scale)) + zp) (zp alone when scale
// is 0).  IEEE double division and rint give the same bits here.  The
// reference raises on an inf or NaN element (its rounding converts NaN to
// an int); those inputs are left undefined.
//
// Kernel 1: CTAs reduce strided slices to (min, max); the last CTA (atomic
// ticket) combines them and writes scale and zero point.  Kernel 2: the
// quantisation, reading them from device memory.
#include "common.cuh"

namespace ortc {
namespace {

constexpr int kDqThreads = 512;

__global__ void __launch_bounds__(kDqThreads)
    dq_range_kernel(const float* __restrict__ X, int64_t n, float2* part, unsigned* ticket,
                    float* scale_out, uint8_t* zp_out, double* params) {
  float mn = 0.0f, mx = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * kDqThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kDqThreads) {
    const float v = __ldg(X + i);
    if (v < mn) mn = v;
    if (v > mx) mx = v;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float a = __shfl_xor_sync(0xffffffffu, mn, off), b = __shfl_xor_sync(0xffffffffu, mx, off);
    if (a < mn) mn = a;
    if (b > mx) mx = b;
  }
  __shared__ float2 wr[kDqThreads / 32];
  __shared__ bool last;
  if ((threadIdx.x & 31) == 0) wr[threadIdx.x >> 5] = make_float2(mn, mx);
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < kDqThreads / 32; w++) {
    if (wr[w].x < mn) mn = wr[w].x;
    if (wr[w].y > mx) mx = wr[w].y;
  }
  part[blockIdx.x] = make_float2(mn, mx);
  __threadfence();
  last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  if (!last) return;
  __threadfence();
  for (unsigned b = 0; b < gridDim.x; b++) {
    const float lo = __ldcg(&part[b].x), hi = __ldcg(&part[b].y);
    if (lo < mn) mn = lo;
    if (hi > mx) mx = hi;
  }
  *ticket = 0;  // ready for the next call
  const float scale = (float)(((double)mx - (double)mn) / 255.0);
  double zp = 0.0;
  if (scale != 0.0f) {
    const double zf = (double)(float)(-(double)mn / (double)scale);
    zp = rint(fmin(fmax(zf, 0.0), 255.0));  // round half to even
  }
  *scale_out = scale;
  *zp_out = (uint8_t)zp;
  params[0] = (double)scale;
  params[1] = zp;
}

__global__ void __launch_bounds__(kDqThreads)
    dq_quantize_kernel(const float* __restrict__ X, int64_t n, const double* params,
                       uint8_t* __restrict__ Y) {
  const double scale = params[0], zp = params[1];
  for (int64_t i = (int64_t)blockIdx.x * kDqThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kDqThreads) {
    double q = zp;
    if (scale != 0.0) q = rint((double)(float)((double)__ldg(X + i) / scale)) + zp;
    Y[i] = (uint8_t)(q < 0.0 ? 0.0 : (q > 255.0 ? 255.0 : q));
  }
}

}  // namespace

size_t dynamic_quant_scratch_bytes(int sm_count) {
  return 256 + (size_t)sm_count * 4 * sizeof(float2);
}

int launch_dynamic_quant(const float* X, int64_t n, uint8_t* Y, float* scale, uint8_t* zp,
                         void* scratch, int sm_count, cudaStream_t st, int64_t* launches) {
  // scratch: [0] ticket, [16] params (2 doubles), [256] per-CTA partials
  unsigned* ticket = static_cast<unsigned*>(scratch);
  double* params = reinterpret_cast<double*>(static_cast<char*>(scratch) + 16);
  float2* part = reinterpret_cast<float2*>(static_cast<char*>(scratch) + 256);
  const int64_t want = (n + kDqThreads * 8 - 1) / (kDqThreads * 8);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count * 4));
  dq_range_kernel<<<grid, kDqThreads, 0, st>>>(X, n, part, ticket, scale, zp, params);
  ORTC_CUDA(cudaGetLastError());
  dq_quantize_kernel<<<grid, kDqThreads, 0, st>>>(X, n, params, Y);
  ORTC_CUDA(cudaGetLastError());
  *launches += 2;
  return ORT_CUDA_OK;
}

}  // namespace ortc
