// Peer-memory all-gather of Y for N-sharded sessions.
//
// The reference's GemmPool writes every worker's output columns straight
// into the shared result (parallel_pool.dart:121-205); across GPUs the
// equivalent is each rank reading the other ranks' column slices over
// NVLink.  Every rank owns an exchange buffer (ready flags, an epoch
// counter, two halves); at session start the buffers are exported with CUDA
// IPC and the handles swapped once through NCCL.  Per operation, with
// e = counter + 1 read on the device:
//   p2p_stage_kernel    copies the rank's [M, Ns] slice into half (e & 1)
//                       (skipped when the producing kernel wrote it there,
//                       see YSel)
//   p2p_gather_kernel   posts e into every peer's flag slot for this rank,
//                       waits (bounded) until every peer has posted e here,
//                       reads all slices with plain peer loads into Y [M, N],
//                       and its last CTA stores counter = e.
// A rank's next write into a half that a peer may still be reading is two
// epochs later, after that peer has posted the intervening epoch, which it
// does only after its own read finished: two halves are enough.  The epoch
// lives on the device, so the sequence replays unchanged from a CUDA graph.
// No NCCL and no multicast is on the per-operation path.
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "nccl_dl.cuh"
#include "ptx.cuh"

namespace ortc {
namespace {

constexpr size_t kFlagBytes = 256;
constexpr int kCtrSlot = 8, kDoneSlot = 9;  // 64-bit words in the flag area
constexpr int kPull = 4;                    // elements per thread and round
constexpr size_t kDefaultCapFloats = size_t(4) << 20;  // 16 MB per half
constexpr size_t kDefaultLLWords = size_t(4) << 20;    // tagged area: 32 MB per half
constexpr int kLand = 4;                               // words per thread and round

struct P2PArgs {
  const float* src[8];            // rank r's half 0 (half 1 follows at + cap)
  unsigned long long* flag[8];    // rank r's flag slot for this rank
  unsigned long long* mine;       // this rank's flag area (slot r written by rank r)
  int64_t cap;
  float* Y;
  int64_t ldy;
  int M, Ns, N, rank, world;
  int* err;
  uint64_t wait_ns;  // bound of the wait for the peers' flags
};

__device__ __forceinline__ unsigned long long next_epoch(const unsigned long long* mine) {
  return *reinterpret_cast<const volatile unsigned long long*>(mine + kCtrSlot) + 1;
}

__global__ void __launch_bounds__(256) p2p_stage_kernel(const float* __restrict__ local,
                                                        float* xhalf0, int64_t cap,
                                                        const unsigned long long* mine,
                                                        int64_t n) {
  float* dst = xhalf0 + (next_epoch(mine) & 1) * cap;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = local[i];
}

__global__ void __launch_bounds__(256) p2p_gather_kernel(const P2PArgs a) {
  __shared__ int ok;
  __shared__ unsigned long long epoch;
  // launched as a programmatic dependent: the slice is complete, and the
  // epoch counter final, only after the producing grid has finished
  griddep_launch_dependents();
  griddep_wait();
  if (threadIdx.x == 0) {
    ok = 1;
    epoch = next_epoch(a.mine);
  }
  __syncthreads();
  const unsigned long long e = epoch;
  if (threadIdx.x == 0) {
    // The slice lives in this GPU's memory and peers read it through this
    // GPU's L2; griddepcontrol.wait has made the producing grid's writes
    // complete and visible, so the flag needs no further fence (a
    // system-scope fence here cost 4-12 us per operation).
    for (int r = 0; r < a.world; r++)
      if (r != a.rank)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a.flag[r]), "l"(e)
                     : "memory");
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < a.world && ok; r++) {
      if (r == a.rank) continue;
      for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a.mine + r) : "memory");
        if (v >= e) break;
        if (globaltimer() - t0 > a.wait_ns) {
          record_error(a.err, KERR_WAIT_PEER);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  if (ok) {
    // up to kPull elements per thread and round, all loads in flight before
    // any store (peer loads take microseconds)
    const int64_t half = (int64_t)(e & 1) * a.cap;
    const int64_t total = (int64_t)a.M * a.N;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total;
         i0 += stride * kPull) {
      float v[kPull];
#pragma unroll
      for (int u = 0; u < kPull; u++) {
        const int64_t i = i0 + u * stride;
        if (i < total) {
          const int m = (int)(i / a.N), n = (int)(i % a.N);
          const int r = n / a.Ns, j = n - r * a.Ns;
          v[u] = __ldcv(a.src[r] + half + (int64_t)m * a.Ns + j);
        }
      }
#pragma unroll
      for (int u = 0; u < kPull; u++) {
        const int64_t i = i0 + u * stride;
        if (i < total) a.Y[(i / a.N) * a.ldy + i % a.N] = v[u];
      }
    }
  }
  // the last CTA to finish advances the epoch counter (every CTA has read it)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.mine + kDoneSlot, 1ull) == gridDim.x - 1) {
      a.mine[kDoneSlot] = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(a.mine + kCtrSlot) = e;
    }
  }
}

// Push mode's consumer (see YSel): copies the peers' columns of this
// epoch's [M, N] output from this rank's tagged area into Y, waiting
// (bounded) for each word's tag; the rank's own columns [n0, n0 + nl) are
// in Y already.  Launched as a programmatic dependent of the producer: the
// epoch is read and advanced only after the producer grid has finished
// (it read the same counter).
__global__ void __launch_bounds__(256) p2p_land_kernel(const unsigned long long* ll0,
                                                       int64_t llcap, unsigned long long* mine,
                                                       float* Y, int M, int N, int n0, int nl,
                                                       int* err, uint64_t wait_ns) {
  __shared__ unsigned long long epoch;
  griddep_launch_dependents();
  griddep_wait();
  if (threadIdx.x == 0) epoch = next_epoch(mine);
  __syncthreads();
  const unsigned long long e = epoch;
  const unsigned tag = (unsigned)e;
  const unsigned long long* src = ll0 + (int64_t)(e & 1) * llcap;
  const int other = N - nl;  // peers' columns per row
  const int total = M * other;
  const int stride = (int)(gridDim.x * blockDim.x);
  uint64_t t0 = 0;
  bool ok = true;
  for (int i0 = (int)(blockIdx.x * blockDim.x + threadIdx.x); i0 < total && ok;
       i0 += stride * kLand) {
    int64_t at[kLand];
    unsigned long long w[kLand];
#pragma unroll
    for (int u = 0; u < kLand; u++) {
      const int i = i0 + u * stride;
      at[u] = -1;
      if (i < total) {
        const int m = i / other, j = i - m * other;
        at[u] = (int64_t)m * N + (j < n0 ? j : j + nl);
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[u]) : "l"(src + at[u]) : "memory");
      }
    }
#pragma unroll
    for (int u = 0; u < kLand; u++) {
      if (at[u] < 0 || !ok) continue;
      while ((unsigned)(w[u] >> 32) != tag) {
        if (t0 == 0) t0 = globaltimer();
        if (globaltimer() - t0 > wait_ns) {
          record_error(err, KERR_WAIT_PEER);
          ok = false;
          break;
        }
        __nanosleep(32);
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[u]) : "l"(src + at[u]) : "memory");
      }
      if (ok) Y[at[u]] = __uint_as_float((unsigned)w[u]);
    }
  }
  // the last CTA to finish advances the epoch counter (every CTA has read it)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(mine + kDoneSlot, 1ull) == gridDim.x - 1) {
      mine[kDoneSlot] = 0;
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(mine + kCtrSlot) = e;
    }
  }
}

// Prefill-sized outputs (push mode, see PrefillPush): the fused GEMM of
// every rank stores its [M, Ns] block straight into each peer's big
// exchange buffer (half epoch & 1, block [source rank]) from its epilogue
// and its last CTA posts the epoch into the peer's ready slot for it.  The
// header of a rank's big buffer holds 64-bit slots: [0, 8) ready epoch
// posted by source r; [8, 16) consumed epoch posted by reader r (the
// reader finished copying this rank's block); 16: the GEMM's CTA ticket;
// 17: the landing kernel's CTA ticket.
constexpr int kReadySlot = 0, kConsumedSlot = 8, kGemmTicketSlot = 16, kLandTicketSlot = 17;
constexpr int kLandV = 8;          // float4 per thread and round
constexpr int kLandThreads = 512;

// Copies rank r's [m, Ns] block (src[r], row pitch Ns) into columns
// r * Ns .. of Y (row pitch ldy, N columns) for every rank but `skip`,
// one (row, rank) slice at a time per CTA.
__device__ void copy_slices(const float* const* src, float* Y, int64_t ldy, int m, int Ns, int N,
                            int world, int skip) {
  const bool vec = (N % 4) == 0 && (Ns % 4) == 0 && (ldy % 4) == 0;
  const int slices = m * world;
  for (int sl = blockIdx.x; sl < slices; sl += gridDim.x) {
    const int row = sl / world, r = sl - row * world;
    if (r == skip) continue;
    const int c0 = r * Ns;
    const int len = min(Ns, N - c0);  // the last rank's slice may be short
    if (len <= 0) continue;
    const float* sp = src[r] + (int64_t)row * Ns;
    float* dst = Y + (int64_t)row * ldy + c0;
    if (vec) {
      const int n4 = len / 4;
      const float4* s4 = reinterpret_cast<const float4*>(sp);
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int j0 = threadIdx.x; j0 < n4; j0 += blockDim.x * kLandV) {
        float4 v[kLandV];
#pragma unroll
        for (int t = 0; t < kLandV; t++) {
          const int j = j0 + t * blockDim.x;
          if (j < n4) v[t] = __ldcg(s4 + j);
        }
#pragma unroll
        for (int t = 0; t < kLandV; t++) {
          const int j = j0 + t * blockDim.x;
          if (j < n4) d4[j] = v[t];
        }
      }
      for (int j = n4 * 4 + threadIdx.x; j < len; j += blockDim.x) dst[j] = __ldcg(sp + j);
    } else {
      for (int j = threadIdx.x; j < len; j += blockDim.x) dst[j] = __ldcg(sp + j);
    }
  }
}

// Waits (bounded) until every peer has posted at least `need` in the slots
// [base, base + world) of this rank's header (not its own).
__device__ bool wait_slots(const unsigned long long* slots, int world, int rank,
                           unsigned long long need, int* err, uint64_t wait_ns) {
  const uint64_t t0 = globaltimer();
  for (int r = 0; r < world; r++) {
    if (r == rank) continue;
    for (;;) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(slots + r) : "memory");
      if (v >= need) break;
      if (globaltimer() - t0 > wait_ns) {
        record_error(err, KERR_WAIT_PEER);
        return false;
      }
      __nanosleep(128);
    }
  }
  return true;
}

// Before a push-mode GEMM: every peer has consumed epoch need from the half
// this epoch overwrites.
__global__ void p2p_push_wait_kernel(const unsigned long long* header, int world, int rank,
                                     unsigned long long need, int* err, uint64_t wait_ns) {
  if (threadIdx.x == 0) wait_slots(header + kConsumedSlot, world, rank, need, err, wait_ns);
}

// A rank holding no columns runs no GEMM: it posts its (empty) block ready.
__global__ void p2p_push_post_kernel(PrefillPush p) {
  if (threadIdx.x == 0)
    for (int r = 0; r < p.world; r++)
      if (r != p.rank)
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.flag[r]), "l"(p.epoch)
                     : "memory");
}

struct LandArgs {
  const float* src[8];             // this rank's half: the block of source r
  unsigned long long* consumed[8];  // source r's consumed slot for this rank
  unsigned long long* header;      // this rank's header
  unsigned long long epoch;
  float* Y;
  int m, Ns, N, rank, world;
  int* err;
  uint64_t wait_ns;
};

__global__ void __launch_bounds__(kLandThreads, 2) p2p_push_land_kernel(const LandArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0)
    ok = wait_slots(a.header + kReadySlot, a.world, a.rank, a.epoch, a.err, a.wait_ns) ? 1 : 0;
  __syncthreads();
  if (ok) copy_slices(a.src, a.Y, a.N, a.m, a.Ns, a.N, a.world, a.rank);
  // the last CTA tells every source that its block of this epoch is consumed
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned* ticket = reinterpret_cast<unsigned*>(a.header + kLandTicketSlot);
    if (atomicAdd(ticket, 1u) == gridDim.x - 1) {
      *ticket = 0u;
      __threadfence_system();
      for (int r = 0; r < a.world; r++)
        if (r != a.rank)
          asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a.consumed[r]), "l"(a.epoch)
                       : "memory");
    }
  }
}

// Bounded completion of a non-blocking NCCL call, then of the stream.
int nccl_finish(ort_cuda_session* s, ncclResult_t r) {
  if (r != ncclSuccess && r != ncclInProgress)
    return fail(ORT_CUDA_ERR_NCCL, std::string("NCCL: ") + nccl()->GetErrorString(r));
  if (r == ncclInProgress) {
    const int rc = nccl_wait_ready((ncclComm_t)s->nccl, s->timeout_ms);
    if (rc) return rc;
  }
  return bounded_sync(s);
}

// Every rank contributes `bytes` at `mine`; returns all ranks' bytes.
int host_allgather(ort_cuda_session* s, const void* mine, size_t bytes, std::vector<char>* all) {
  void* d = nullptr;
  ORTC_CUDA(cudaMalloc(&d, bytes * s->world));
  int rc = ORT_CUDA_OK;
  cudaError_t e = cudaMemcpy((char*)d + bytes * s->rank, mine, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpy");
  if (rc == ORT_CUDA_OK)
    rc = nccl_finish(s, nccl()->AllGather((char*)d + bytes * s->rank, d, bytes, ncclUint8,
                                          (ncclComm_t)s->nccl, s->stream));
  if (rc == ORT_CUDA_OK) {
    all->resize(bytes * s->world);
    e = cudaMemcpy(all->data(), d, bytes * s->world, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpy");
  }
  cudaFree(d);
  return rc;
}

}  // namespace

int p2p_setup(ort_cuda_session* s) {
  s->p2p_ok = false;
  if (s->world < 2 || s->world > 8 || !s->nccl) return ORT_CUDA_OK;
  size_t cap = kDefaultCapFloats;
  if (const char* env = std::getenv("ORT_CUDA_P2P_FLOATS")) cap = std::strtoull(env, nullptr, 10);
  cap = (cap + 63) / 64 * 64;  // keeps the tagged area 256-byte aligned
  const size_t llcap = kDefaultLLWords;
  // [flags][half 0, half 1: cap floats][tagged half 0, half 1: llcap words];
  // the tagged area starts zeroed (tag 0 is never an epoch: e >= 1)
  ORTC_CUDA(cudaMalloc(&s->xbuf, kFlagBytes + 2 * cap * 4 + 2 * llcap * 8));
  ORTC_CUDA(cudaMemset(s->xbuf, 0, kFlagBytes));
  ORTC_CUDA(cudaMemset((char*)s->xbuf + kFlagBytes + 2 * cap * 4, 0, 2 * llcap * 8));
  ORTC_CUDA(cudaDeviceSynchronize());
  s->xcap = cap;
  s->llcap = llcap;
  cudaIpcMemHandle_t h;
  bool ok = cudaIpcGetMemHandle(&h, s->xbuf) == cudaSuccess;
  if (!ok) std::memset(&h, 0, sizeof(h));
  std::vector<char> handles;
  int rc = host_allgather(s, &h, sizeof(h), &handles);
  if (rc) return rc;
  for (int r = 0; r < s->world; r++) {
    if (r == s->rank) {
      s->xpeer[r] = s->xbuf;
      continue;
    }
    cudaIpcMemHandle_t hr;
    std::memcpy(&hr, handles.data() + r * sizeof(hr), sizeof(hr));
    void* p = nullptr;
    if (ok && cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess)
      s->xpeer[r] = p;
    else
      ok = false;
  }
  cudaGetLastError();  // a refused mapping only disables this path
  // every rank must take the same path: use peer memory only if all can
  const char mine = ok ? 1 : 0;
  std::vector<char> oks;
  rc = host_allgather(s, &mine, 1, &oks);
  if (rc) return rc;
  bool all_ok = true;
  for (char c : oks) all_ok = all_ok && c == 1;
  s->p2p_ok = all_ok;
  return ORT_CUDA_OK;
}

namespace {
constexpr size_t kBigFlagBytes = 4096;

void big_unmap(ort_cuda_session* s) {
  for (int r = 0; r < 8; r++) {
    if (s->bpeer[r] && r != s->rank) cudaIpcCloseMemHandle(s->bpeer[r]);
    s->bpeer[r] = nullptr;
  }
  if (s->bbuf) cudaFree(s->bbuf);
  s->bbuf = nullptr;
  s->bcap = 0;
}
}  // namespace

int p2p_big_ensure(ort_cuda_session* s, size_t half_floats, bool* ok) {
  *ok = false;
  if (!s->p2p_ok || !s->nccl) return ORT_CUDA_OK;
  if (s->bbuf && s->bcap >= half_floats) {
    *ok = true;
    return ORT_CUDA_OK;
  }
  // Every rank reaches this with the same size (the shapes are the same on
  // all ranks).  The old buffer goes first: nobody reads it any more once
  // every rank has synchronised its streams and passed the handshake below.
  ORTC_CUDA(cudaDeviceSynchronize());
  std::vector<char> sync;
  const char one = 1;
  int rc = host_allgather(s, &one, 1, &sync);
  if (rc) return rc;
  big_unmap(s);
  const size_t want = (half_floats + 63) / 64 * 64;
  bool mine_ok = cudaMalloc(&s->bbuf, kBigFlagBytes + 2 * want * 4) == cudaSuccess;
  if (!mine_ok) {
    cudaGetLastError();
    s->bbuf = nullptr;
  }
  cudaIpcMemHandle_t h;
  std::memset(&h, 0, sizeof(h));
  if (mine_ok) {
    mine_ok = cudaMemset(s->bbuf, 0, kBigFlagBytes) == cudaSuccess &&
              cudaDeviceSynchronize() == cudaSuccess &&
              cudaIpcGetMemHandle(&h, s->bbuf) == cudaSuccess;
    cudaGetLastError();
  }
  std::vector<char> handles;
  rc = host_allgather(s, &h, sizeof(h), &handles);
  if (rc) return rc;
  for (int r = 0; r < s->world && mine_ok; r++) {
    if (r == s->rank) {
      s->bpeer[r] = s->bbuf;
      continue;
    }
    cudaIpcMemHandle_t hr;
    std::memcpy(&hr, handles.data() + r * sizeof(hr), sizeof(hr));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess)
      s->bpeer[r] = p;
    else
      mine_ok = false;
  }
  cudaGetLastError();
  const char c = mine_ok ? 1 : 0;
  std::vector<char> oks;
  rc = host_allgather(s, &c, 1, &oks);
  if (rc) return rc;
  bool all_ok = true;
  for (char o : oks) all_ok = all_ok && o == 1;
  if (!all_ok) {
    big_unmap(s);
    return ORT_CUDA_OK;  // every rank keeps the NCCL path
  }
  s->bcap = want;
  s->bepoch = 0;  // every rank restarts its epochs with the zeroed header
  *ok = true;
  return ORT_CUDA_OK;
}

namespace {
float* big_half(void* base, size_t cap, unsigned long long epoch) {
  return (float*)((char*)base + kBigFlagBytes) + (size_t)(epoch & 1) * cap;
}
}  // namespace

int p2p_push_prepare(ort_cuda_session* s, unsigned long long epoch, int64_t M, int64_t ns,
                     PrefillPush* push) {
  unsigned long long* header = (unsigned long long*)s->bbuf;
  if (epoch >= 3) {
    p2p_push_wait_kernel<<<1, 32, 0, s->stream>>>(header, s->world, s->rank, epoch - 2,
                                                  s->err_dev,
                                                  (uint64_t)s->peer_wait_ms * 1000000ull);
    ORTC_CUDA(cudaGetLastError());
    s->launches++;
  }
  *push = PrefillPush();
  for (int r = 0; r < s->world; r++) {
    push->land[r] = big_half(s->bpeer[r], s->bcap, epoch) + (size_t)s->rank * M * ns;
    push->flag[r] = (unsigned long long*)s->bpeer[r] + kReadySlot + s->rank;
  }
  push->ticket = reinterpret_cast<unsigned*>(header + kGemmTicketSlot);
  push->epoch = epoch;
  push->ns = ns;
  push->rank = s->rank;
  push->world = s->world;
  return ORT_CUDA_OK;
}

int p2p_push_post(ort_cuda_session* s, const PrefillPush& push) {
  p2p_push_post_kernel<<<1, 32, 0, s->stream>>>(push);
  ORTC_CUDA(cudaGetLastError());
  s->launches++;
  return ORT_CUDA_OK;
}

int p2p_push_land(ort_cuda_session* s, unsigned long long epoch, int64_t M, int64_t ns,
                  int64_t N, float* Y) {
  LandArgs a;
  for (int r = 0; r < 8; r++) {
    a.src[r] = nullptr;
    a.consumed[r] = nullptr;
  }
  for (int r = 0; r < s->world; r++) {
    a.src[r] = big_half(s->bbuf, s->bcap, epoch) + (size_t)r * M * ns;
    a.consumed[r] = (unsigned long long*)s->bpeer[r] + kConsumedSlot + s->rank;
  }
  a.header = (unsigned long long*)s->bbuf;
  a.epoch = epoch;
  a.Y = Y;
  a.m = (int)M;
  a.Ns = (int)ns;
  a.N = (int)N;
  a.rank = s->rank;
  a.world = s->world;
  a.err = s->err_dev;
  a.wait_ns = (uint64_t)s->peer_wait_ms * 1000000ull;
  const unsigned blocks = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>(M * s->world, (int64_t)s->sm_count * 2));
  p2p_push_land_kernel<<<blocks, kLandThreads, 0, s->stream>>>(a);
  ORTC_CUDA(cudaGetLastError());
  s->launches++;
  return ORT_CUDA_OK;
}

void p2p_teardown(ort_cuda_session* s) {
  if (s->xbuf && s->nccl) {
    // no rank unmaps or frees before every rank's last read has finished
    std::vector<char> all;
    const char one = 1;
    host_allgather(s, &one, 1, &all);
  }
  big_unmap(s);
  for (int r = 0; r < 8; r++)
    if (s->xpeer[r] && r != s->rank) cudaIpcCloseMemHandle(s->xpeer[r]);
  if (s->xbuf) cudaFree(s->xbuf);
  s->xbuf = nullptr;
  for (auto& p : s->xpeer) p = nullptr;
  s->p2p_ok = false;
}

bool p2p_fits(ort_cuda_session* s, int64_t floats) {
  return s->p2p_ok && (size_t)floats <= s->xcap;
}

bool p2p_push_fits(ort_cuda_session* s, int64_t M, int64_t N) {
  return s->p2p_ok && s->llcap > 0 && M * N <= (int64_t)s->llcap && N <= INT_MAX / 16 &&
         M * N <= INT_MAX;
}

YSel p2p_ysel_push(ort_cuda_session* s, int64_t n0, int64_t N, int row0) {
  YSel y;
  y.ctr = (const unsigned long long*)s->xbuf + kCtrSlot;
  y.push = true;
  y.rank = s->rank;
  y.world = s->world;
  y.row0 = row0;
  y.n0 = n0;
  y.N = N;
  y.llcap = (int64_t)s->llcap;
  for (int r = 0; r < s->world; r++)
    y.ll[r] = (unsigned long long*)((char*)s->xpeer[r] + kFlagBytes + 2 * s->xcap * 4);
  return y;
}

int p2p_land(ort_cuda_session* s, int64_t M, int64_t N, int64_t n0, int64_t nl, float* Y) {
  unsigned long long* mine = (unsigned long long*)s->xbuf;
  const unsigned long long* ll0 =
      (const unsigned long long*)((char*)s->xbuf + kFlagBytes + 2 * s->xcap * 4);
  const int64_t total = M * (N - nl);
  const unsigned blocks = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>((total + 256 * kLand - 1) / (256 * kLand), s->sm_count));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ORTC_CUDA(cudaLaunchKernelEx(&cfg, p2p_land_kernel, ll0, (int64_t)s->llcap, mine, Y, (int)M,
                               (int)N, (int)n0, (int)nl, s->err_dev,
                               (uint64_t)s->peer_wait_ms * 1000000ull));
  s->launches++;
  return ORT_CUDA_OK;
}

YSel p2p_ysel(ort_cuda_session* s) {
  YSel y;
  y.half0 = (float*)((char*)s->xbuf + kFlagBytes);
  y.cap = (int64_t)s->xcap;
  y.ctr = (const unsigned long long*)s->xbuf + kCtrSlot;
  return y;
}

int p2p_gather(ort_cuda_session* s, const float* local, int64_t M, int64_t Ns, int64_t N,
               float* Y) {
  unsigned long long* mine = (unsigned long long*)s->xbuf;
  float* half0 = (float*)((char*)s->xbuf + kFlagBytes);
  const int64_t n_local = M * Ns;
  if (local) {
    const unsigned sblocks =
        (unsigned)std::max<int64_t>(1, std::min<int64_t>((n_local + 1023) / 1024, s->sm_count));
    p2p_stage_kernel<<<sblocks, 256, 0, s->stream>>>(local, half0, (int64_t)s->xcap, mine,
                                                     n_local);
    ORTC_CUDA(cudaGetLastError());
    s->launches++;
  }
  P2PArgs a;
  for (int r = 0; r < 8; r++) {
    a.src[r] = nullptr;
    a.flag[r] = nullptr;
  }
  for (int r = 0; r < s->world; r++) {
    a.src[r] = (const float*)((char*)s->xpeer[r] + kFlagBytes);
    a.flag[r] = (unsigned long long*)s->xpeer[r] + s->rank;
  }
  a.mine = mine;
  a.cap = (int64_t)s->xcap;
  a.Y = Y;
  a.ldy = N;
  a.M = (int)M;
  a.Ns = (int)Ns;
  a.N = (int)N;
  a.rank = s->rank;
  a.world = s->world;
  a.err = s->err_dev;
  a.wait_ns = (uint64_t)s->peer_wait_ms * 1000000ull;
  const int64_t total = M * N;
  const unsigned blocks = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>((total + 256 * kPull - 1) / (256 * kPull), s->sm_count * 4));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ORTC_CUDA(cudaLaunchKernelEx(&cfg, p2p_gather_kernel, a));
  s->launches++;
  return ORT_CUDA_OK;
}

}  // namespace ortc
