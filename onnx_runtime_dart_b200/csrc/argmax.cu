// ArgMax / ArgMin over the last axis of a device-resident [rows, cols] fp32
// matrix: the device counterpart of opArgMinMax (lib/src/onnx_ops.dart:
// 2198-2237) for the case a decode step needs, greedy selection over the
// lm_head logits, so that a step reads back one int64 per row instead of the
// whole logits row.
//
// The reference scans from element 0 with plain comparisons: a candidate
// replaces the best only if strictly better (or also equal, with
// select_last_index), so ties keep the first (last) index and a NaN never
// wins unless it is element 0 (comparisons with NaN are false).  The same
// result is the best of the non-NaN elements under the order "larger
// (smaller) value, then smaller (larger) index" — an order in which any
// grouping of the scan gives the same answer — replaced by 0 when element 0
// is NaN.  CTAs reduce 16K-column segments of a row to one candidate each;
// the last CTA of a row (an atomic ticket) combines the row's candidates in
// segment order and writes the index.
#include <climits>

#include "common.cuh"

namespace ortc {
namespace {

constexpr int kArgThreads = 512;
constexpr int64_t kArgSeg = 16384;  // columns per CTA

// Whether candidate (v, i) replaces the current best (bv, bi); `ok` marks a
// non-NaN candidate.
__device__ __forceinline__ bool replaces(float v, int i, bool ok, float bv, int bi, bool bok,
                                         bool is_min, bool last) {
  if (!ok) return false;
  if (!bok) return true;
  if (v != bv) return is_min ? v < bv : v > bv;
  return last ? i > bi : i < bi;
}

struct ArgCand {
  float v;
  int i;
  int ok;
};

__device__ __forceinline__ void take(ArgCand& b, const ArgCand& c, bool is_min, bool last) {
  if (replaces(c.v, c.i, c.ok != 0, b.v, b.i, b.ok != 0, is_min, last)) b = c;
}

__global__ void __launch_bounds__(kArgThreads)
    argminmax_kernel(const float* __restrict__ X, int64_t ldx, int cols, int nseg, int is_min,
                     int last, ArgCand* part, unsigned* tickets, int64_t* out) {
  const int row = (int)(blockIdx.x / nseg), seg = (int)(blockIdx.x % nseg);
  const float* x = X + (int64_t)row * ldx;
  const int c0 = (int)(seg * kArgSeg), c1 = (int)min((int64_t)cols, (seg + 1) * kArgSeg);
  ArgCand b = {0.0f, 0, 0};
  // each thread's indices increase, so its own scan order is the reference's
  for (int c = c0 + threadIdx.x; c < c1; c += kArgThreads) {
    const float v = __ldg(x + c);
    const ArgCand cand = {v, c, isnan(v) ? 0 : 1};
    take(b, cand, is_min, last);
  }
  for (int off = 16; off > 0; off >>= 1) {
    ArgCand o;
    o.v = __shfl_xor_sync(0xffffffffu, b.v, off);
    o.i = __shfl_xor_sync(0xffffffffu, b.i, off);
    o.ok = __shfl_xor_sync(0xffffffffu, b.ok, off);
    take(b, o, is_min, last);
  }
  __shared__ ArgCand warp_best[kArgThreads / 32];
  __shared__ bool finisher;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_best[warp] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgThreads / 32; w++) take(b, warp_best[w], is_min, last);
    finisher = true;
    if (nseg > 1) {
      part[(int64_t)row * nseg + seg] = b;
      __threadfence();  // the candidate is visible before the ticket is taken
      finisher = atomicAdd(&tickets[row], 1u) == (unsigned)(nseg - 1);
    }
  }
  __syncthreads();
  if (threadIdx.x != 0 || !finisher) return;
  if (nseg > 1) {
    __threadfence();
    b.ok = 0;
    for (int s = 0; s < nseg; s++) {  // segment order, as the scan visits them
      const ArgCand* q = part + (int64_t)row * nseg + s;
      ArgCand c;
      c.v = __ldcg(&q->v);
      c.i = __ldcg(&q->i);
      c.ok = __ldcg(&q->ok);
      take(b, c, is_min, last);
    }
    tickets[row] = 0;  // ready for the next call
  }
  out[row] = isnan(__ldg(x)) || !b.ok ? 0 : (int64_t)b.i;
}

}  // namespace

int64_t argminmax_candidates(int64_t rows, int64_t cols) {
  const int64_t nseg = (cols + kArgSeg - 1) / kArgSeg;
  return nseg <= 1 ? 0 : rows * nseg;
}
size_t argminmax_candidate_bytes() { return sizeof(ArgCand); }

int launch_argminmax(const float* X, int64_t rows, int64_t cols, int64_t ldx, bool is_min,
                     bool last, int64_t* out, unsigned* tickets, void* candidates,
                     cudaStream_t st, int64_t* launches) {
  if (rows == 0) return ORT_CUDA_OK;
  ORTC_CHECK(cols >= 1 && cols <= INT_MAX && ldx >= cols && rows <= INT_MAX,
             ORT_CUDA_ERR_INVALID_ARG, "ArgMax: need 1 <= cols <= ldx and cols < 2^31");
  const int nseg = (int)((cols + kArgSeg - 1) / kArgSeg);
  ORTC_CHECK(rows * nseg <= INT_MAX, ORT_CUDA_ERR_INVALID_ARG, "ArgMax: too many rows");
  ArgCand* part = static_cast<ArgCand*>(candidates);
  argminmax_kernel<<<(unsigned)(rows * nseg), kArgThreads, 0, st>>>(
      X, ldx, (int)cols, nseg, is_min ? 1 : 0, last ? 1 : 0, part, tickets, out);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

}  // namespace ortc
