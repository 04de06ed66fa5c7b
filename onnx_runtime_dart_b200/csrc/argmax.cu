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
#include <algorithm>
#include <atomic>
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

// ---- TopK over the last axis ----------------------------------------------
// The device counterpart of opTopK (lib/src/onnx_ops.dart:2261-2303) for the
// candidates of top-k sampling after lm_head: per row the k entries in the
// reference's order -- value descending (ascending with `largest` 0), ties
// to the smaller index, NaN above every number (Dart's compareTo), -0.0
// equal to 0.0.  Each value maps to a 32-bit key whose unsigned order is
// that ranking (largest first); one CTA per row finds the k-th key by radix
// selection (four 8-bit histogram passes), gathers the keys above it and,
// in index order, the first ties at it, and sorts the k (key, index) pairs
// with a bitonic network in shared memory.
namespace ortc {
namespace {

constexpr int kTkThreads = 1024;
constexpr int kTkMaxK = 1024;
constexpr int kTkSeg = 8192;        // columns per segment CTA of a long row
constexpr int kTkMaxCand = 4096;    // candidates merged per row
constexpr int kTkMaxKeyBytes = 160 * 1024;  // a row segment's keys in shared memory

__device__ __forceinline__ uint32_t topk_key(float v, bool largest) {
  uint32_t u;
  if (isnan(v)) {
    u = 0xffffffffu;
  } else {
    if (v == 0.0f) v = 0.0f;  // -0.0 ties with 0.0
    u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order-preserving
  }
  return largest ? u : ~u;
}

// (key, index) as one 64-bit word that orders key descending, then index
// ascending; 0 ranks below every entry.
__device__ __forceinline__ unsigned long long topk_pair(uint32_t key, uint32_t c) {
  return ((unsigned long long)key << 32) | (0xffffffffu - c);
}

// The k largest keys of columns [c0, c0 + len) of row x, unordered, into
// out[0..k) as pairs (slots past len hold 0).  Radix selection of the k-th
// key T with warp-aggregated histogram counts, then the keys above T and,
// in index order, the first ties at T.  All threads of the CTA take part.
__device__ void topk_select(const float* __restrict__ x, int c0, int len, int k, bool largest,
                            uint32_t* keys, unsigned long long* out, unsigned* hist,
                            unsigned* wsum, unsigned& s_bin, unsigned& s_left, unsigned& n_gt) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int iters = (len + kTkThreads - 1) / kTkThreads;
  if (len <= k) {  // every column is a candidate
    for (int i = tid; i < k; i += kTkThreads)
      out[i] = i < len ? topk_pair(topk_key(__ldg(x + c0 + i), largest), (uint32_t)(c0 + i)) : 0ull;
    __syncthreads();
    return;
  }
  // the keys into shared memory once (independent loads), read by every pass
#pragma unroll 8
  for (int c = tid; c < len; c += kTkThreads) keys[c] = topk_key(__ldg(x + c0 + c), largest);
  uint32_t prefix = 0, mask = 0;
  unsigned left = (unsigned)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kTkThreads) hist[i] = 0;
    __syncthreads();
    for (int it = 0; it < iters; it++) {
      const int c = it * kTkThreads + tid;
      unsigned bin = 256u;
      if (c < len) {
        const uint32_t key = keys[c];
        if ((key & mask) == prefix) bin = (key >> shift) & 255u;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin != 256u && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
    }
    __syncthreads();
    // the bin holding the left-th largest key: a suffix scan of the counts
    // (thread t takes bin 255 - t), one thread finds the crossing
    unsigned h = 0, v = 0;
    if (tid < 256) {
      h = hist[255 - tid];
      v = h;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const unsigned n = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += n;
      }
      if (lane == 31) wsum[warp] = v;
    }
    __syncthreads();
    if (tid < 256) {
      unsigned base = 0;
      for (int w2 = 0; w2 < warp; w2++) base += wsum[w2];
      const unsigned incl = base + v, excl = incl - h;
      if (excl < left && incl >= left) {
        s_bin = 255u - (unsigned)tid;
        s_left = left - excl;
      }
    }
    __syncthreads();
    prefix |= s_bin << shift;
    mask |= 255u << shift;
    left = s_left;
  }
  const uint32_t T = prefix;
  const unsigned ngt = (unsigned)k - left;  // keys above T, all taken
  if (tid == 0) n_gt = 0;
  __syncthreads();
  unsigned ties = 0;  // ties taken before this tile (uniform)
  for (int it = 0; it < iters; it++) {
    const int c = it * kTkThreads + tid;
    const uint32_t key = c < len ? keys[c] : 0u;
    const bool gt = c < len && key > T, tie = c < len && key == T;
    if (gt) out[atomicAdd(&n_gt, 1u)] = topk_pair(key, (uint32_t)(c0 + c));
    const unsigned bal = __ballot_sync(0xffffffffu, tie);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    unsigned before = ties;
    for (int w2 = 0; w2 < warp; w2++) before += wsum[w2];
    before += __popc(bal & ((1u << lane) - 1u));
    if (tie && before < left) out[ngt + before] = topk_pair(key, (uint32_t)(c0 + c));
    unsigned tile = 0;
    for (int w2 = 0; w2 < kTkThreads / 32; w2++) tile += wsum[w2];
    ties += tile;
    __syncthreads();  // wsum is rewritten by the next tile
  }
}

// Sorts n pairs in shared memory descending (bitonic, n padded to a power
// of two with 0) and writes the first k as values and indices of row x.
__device__ void topk_sort_out(unsigned long long* cand, int n, int k, const float* __restrict__ x,
                              float* vals, int64_t* idx) {
  const int tid = threadIdx.x;
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = n + tid; i < P; i += kTkThreads) cand[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += kTkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const unsigned long long a = cand[i], b = cand[j];
          const bool desc = (i & size) == 0;
          if (desc ? a < b : a > b) {
            cand[i] = b;
            cand[j] = a;
          }
        }
      }
      __syncthreads();
    }
  for (int i = tid; i < k; i += kTkThreads) {
    const uint32_t c = 0xffffffffu - (uint32_t)(cand[i] & 0xffffffffull);
    vals[i] = x[c];
    idx[i] = (int64_t)c;
  }
}

// One CTA per row (rows up to a few segments long).
__global__ void __launch_bounds__(kTkThreads)
    topk_kernel(const float* __restrict__ X, int64_t ldx, int cols, int k, int largest,
                float* __restrict__ vals, int64_t* __restrict__ idx) {
  __shared__ unsigned hist[256];
  __shared__ unsigned wsum[kTkThreads / 32];
  __shared__ unsigned s_bin, s_left, n_gt;
  __shared__ unsigned long long cand[kTkMaxK];
  extern __shared__ uint32_t tk_keys[];  // cols keys
  const float* x = X + (int64_t)blockIdx.x * ldx;
  topk_select(x, 0, cols, k, largest != 0, tk_keys, cand, hist, wsum, s_bin, s_left, n_gt);
  __syncthreads();
  topk_sort_out(cand, k, k, x, vals + (int64_t)blockIdx.x * k, idx + (int64_t)blockIdx.x * k);
}

// Long rows, stage 1: CTA (row, segment) writes its segment's k best pairs.
__global__ void __launch_bounds__(kTkThreads)
    topk_seg_kernel(const float* __restrict__ X, int64_t ldx, int cols, int seg, int nseg, int k,
                    int largest, unsigned long long* __restrict__ cand) {
  __shared__ unsigned hist[256];
  __shared__ unsigned wsum[kTkThreads / 32];
  __shared__ unsigned s_bin, s_left, n_gt;
  __shared__ unsigned long long loc[kTkMaxK];
  extern __shared__ uint32_t tk_keys[];  // seg keys
  const int row = blockIdx.x / nseg, sg = blockIdx.x % nseg;
  const int c0 = sg * seg, len = min(seg, cols - c0);
  topk_select(X + (int64_t)row * ldx, c0, len, k, largest != 0, tk_keys, loc, hist, wsum, s_bin,
              s_left, n_gt);
  __syncthreads();
  for (int i = threadIdx.x; i < k; i += kTkThreads)
    cand[((int64_t)row * nseg + sg) * k + i] = loc[i];
}

// Stage 2: one CTA per row sorts the segments' nseg * k pairs.
__global__ void __launch_bounds__(kTkThreads)
    topk_merge_kernel(const float* __restrict__ X, int64_t ldx, int nseg, int k,
                      const unsigned long long* __restrict__ cand, float* __restrict__ vals,
                      int64_t* __restrict__ idx) {
  __shared__ unsigned long long all[kTkMaxCand];
  const int row = blockIdx.x, n = nseg * k;
  for (int i = threadIdx.x; i < n; i += kTkThreads) all[i] = cand[(int64_t)row * n + i];
  __syncthreads();
  topk_sort_out(all, n, k, X + (int64_t)row * ldx, vals + (int64_t)row * k, idx + (int64_t)row * k);
}

}  // namespace

int topk_segments(int64_t cols, int64_t k) {
  if (cols <= 2 * kTkSeg) return 1;
  int64_t nseg = (cols + kTkSeg - 1) / kTkSeg;
  nseg = std::min<int64_t>(nseg, kTkMaxCand / std::max<int64_t>(k, 1));
  return (int)std::max<int64_t>(1, nseg);
}

// Largest k a row of `cols` columns takes: a segment holds at most
// kTkMaxKeyBytes / 4 = 40960 columns and a row at most kTkMaxCand / k
// segments, so cols <= 40960 * floor(4096 / k).
int64_t topk_max_k(int64_t cols) {
  const int64_t seg_cols = kTkMaxKeyBytes / 4;
  if (cols <= 2 * kTkSeg || cols <= seg_cols) return std::min<int64_t>(cols, kTkMaxK);
  const int64_t nseg_needed = (cols + seg_cols - 1) / seg_cols;
  return std::min<int64_t>({cols, (int64_t)kTkMaxK, kTkMaxCand / nseg_needed});
}

size_t topk_scratch_bytes(int64_t rows, int64_t cols, int64_t k) {
  const int nseg = topk_segments(cols, k);
  return nseg > 1 ? (size_t)rows * nseg * k * 8 : 0;
}

int launch_topk(const float* X, int64_t rows, int64_t cols, int64_t ldx, int64_t k, bool largest,
                float* vals, int64_t* idx, void* scratch, cudaStream_t st, int64_t* launches) {
  if (rows == 0 || k == 0) return ORT_CUDA_OK;
  ORTC_CHECK(k >= 1 && k <= kTkMaxK && k <= cols && cols <= INT_MAX && ldx >= cols &&
                 rows <= INT_MAX,
             ORT_CUDA_ERR_INVALID_ARG, "TopK: need 1 <= k <= min(cols, 1024) and cols < 2^31");
  const int nseg = topk_segments(cols, k);
  // per device: keys above 48 KB of shared memory.  Sessions may run on
  // several host threads; setting the attribute twice is harmless, so an
  // atomic bit per device only saves the repeated calls.
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  ORTC_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !(attr_set.load(std::memory_order_acquire) >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kTkMaxKeyBytes));
    ORTC_CUDA(cudaFuncSetAttribute(topk_seg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kTkMaxKeyBytes));
    if (dev < 64) attr_set.fetch_or(1ull << dev, std::memory_order_acq_rel);
  }
  if (nseg == 1) {
    topk_kernel<<<(unsigned)rows, kTkThreads, (size_t)cols * 4, st>>>(
        X, ldx, (int)cols, (int)k, largest ? 1 : 0, vals, idx);
    ORTC_CUDA(cudaGetLastError());
    (*launches)++;
    return ORT_CUDA_OK;
  }
  ORTC_CHECK(scratch != nullptr, ORT_CUDA_ERR_INVALID_ARG, "TopK: scratch missing");
  ORTC_CHECK(rows * nseg <= INT_MAX, ORT_CUDA_ERR_INVALID_ARG, "TopK: too many rows");
  const int seg = (int)((cols + nseg - 1) / nseg);
  ORTC_CHECK((size_t)seg * 4 <= (size_t)kTkMaxKeyBytes, ORT_CUDA_ERR_UNSUPPORTED,
             "TopK: rows of " + std::to_string(cols) + " columns take k <= " +
                 std::to_string(topk_max_k(cols)) + " (each of at most 4096 / k segments "
                 "holds 40960 columns), got k = " + std::to_string(k));
  unsigned long long* cand = static_cast<unsigned long long*>(scratch);
  topk_seg_kernel<<<(unsigned)(rows * nseg), kTkThreads, (size_t)seg * 4, st>>>(
      X, ldx, (int)cols, seg, nseg, (int)k, largest ? 1 : 0, cand);
  ORTC_CUDA(cudaGetLastError());
  topk_merge_kernel<<<(unsigned)rows, kTkThreads, 0, st>>>(X, ldx, nseg, (int)k, cand, vals, idx);
  ORTC_CUDA(cudaGetLastError());
  *launches += 2;
  return ORT_CUDA_OK;
}

}  // namespace ortc
