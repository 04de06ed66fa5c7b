// C ABI (include/ort_cuda.h): sessions, weight residency, device tensors
// and operator dispatch for MatMulNBits / MatMul / Gemm.
//
// This is the B200 counterpart of the three OnnxGraphExecutor._dispatch
// cases (lib/src/onnx_graph.dart:1154-1173, :1584-1596) together with the
// state the reference keeps for them (_initializers, _prepackedGemmB,
// onnx_graph.dart:51-56) and its column-split worker pool
// (lib/src/parallel_pool.dart:108-205), which becomes NCCL N-sharding.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "nccl_dl.cuh"

namespace ortc {

static thread_local std::string g_err;

void set_error(const std::string& msg) { g_err = msg; }
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  g_err = std::string("CUDA error ") + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) +
          ") in " + what;
  if (e == cudaErrorMemoryAllocation) return ORT_CUDA_ERR_OOM;
  return ORT_CUDA_ERR_CUDA;
}

int ensure_ws(ort_cuda_session* s, size_t bytes) {
  if (bytes <= s->ws_bytes) return ORT_CUDA_OK;
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
             "a buffer would grow while a CUDA graph is being captured; run every "
             "operation of the graph once before capturing it");
  size_t want = bytes + bytes / 4 + (1 << 20);
  if (s->ws) {
    ORTC_CUDA(cudaStreamSynchronize(s->stream));
    ORTC_CUDA(cudaFree(s->ws));
    s->ws = nullptr;
    s->ws_bytes = 0;
  }
  ORTC_CUDA(cudaMalloc(&s->ws, want));
  s->ws_bytes = want;
  return ORT_CUDA_OK;
}

int ensure_pinned(ort_cuda_session* s, size_t bytes) {
  if (bytes <= s->pinned_bytes) return ORT_CUDA_OK;
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
             "a buffer would grow while a CUDA graph is being captured; run every "
             "operation of the graph once before capturing it");
  size_t want = bytes + bytes / 4 + (1 << 20);
  if (s->pinned) {
    ORTC_CUDA(cudaStreamSynchronize(s->stream));
    ORTC_CUDA(cudaFreeHost(s->pinned));
    s->pinned = nullptr;
    s->pinned_bytes = 0;
  }
  ORTC_CUDA(cudaMallocHost(&s->pinned, want));
  s->pinned_bytes = want;
  return ORT_CUDA_OK;
}

// The decode GEMV times its candidate plans on a weight's first eager call
// for each M (once; results never depend on the plan).
// ORT_CUDA_GEMV_TUNE=0 keeps the heuristic choice instead.
static bool gemv_tuning_enabled() {
  static const bool on = [] {
    const char* v = getenv("ORT_CUDA_GEMV_TUNE");
    return !(v && v[0] == '0');
  }();
  return on;
}

int ensure_kscratch(ort_cuda_session* s, size_t bytes) {
  if (bytes <= s->kscratch_bytes) return ORT_CUDA_OK;
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
             "a buffer would grow while a CUDA graph is being captured; run every "
             "operation of the graph once before capturing it");
  size_t want = bytes + bytes / 4 + (1 << 20);
  if (s->kscratch) {
    ORTC_CUDA(cudaStreamSynchronize(s->stream));
    ORTC_CUDA(cudaFree(s->kscratch));
    s->kscratch = nullptr;
    s->kscratch_bytes = 0;
  }
  ORTC_CUDA(cudaMalloc(&s->kscratch, want));
  s->kscratch_bytes = want;
  return ORT_CUDA_OK;
}

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

bool is_pinned_host(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

int free_weight(ortc::Weight& w) {
  void* ptrs[] = {w.B, w.scales, w.scales16, w.zp, w.W, w.W16, w.col_exp, w.sz16,
                  w.Wi8, w.colsum, w.bzp};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  w = ortc::Weight();
  return ORT_CUDA_OK;
}

int mode_of(ort_cuda_session* s, int flags) {
  if (flags & ORT_CUDA_MODE_OVERRIDE) return (flags >> 12) & 0xF;
  return s->mode;
}

bool valid_mode(int m) { return m >= ORT_CUDA_MODE_EXACT && m <= ORT_CUDA_MODE_MMA_BF16; }

// Per-rank column range of an N-column weight: Ns = ceil(N/world) rounded
// up to 4 (16-byte aligned slices for the all-gather), rank r owns
// [r*Ns, min(N, (r+1)*Ns)).
void shard_cols(int64_t N, int rank, int world, int64_t* n0, int64_t* nl, int64_t* ns) {
  int64_t per = (N + world - 1) / world;
  per = (per + 3) / 4 * 4;
  if (world == 1) per = N;
  int64_t a = per * rank;
  if (a > N) a = N;
  int64_t b = a + per;
  if (b > N) b = N;
  *n0 = a;
  *nl = b - a;
  *ns = per;
}

// Size-based placement on an N-sharded session.  Sharding a weight saves
// (1 - 1/G) of its stream time but adds the exchange of its output and
// leaves the GEMV's fixed per-launch cost (4-7 us) unshrunk, so a
// MatMulNBits weight whose packed bytes stay below replicate_bytes (by
// default kReplicateBytes) is kept whole on every rank and computed locally;
// its results are the 1-GPU results.  Measured at 2, 4 and 8 B200 (cfg3 and
// cfg4 projections of 0.5-8.6 MB: 1.4-1.6x faster replicated; the 9-31 MB
// cfg5 projections: within 2 us either way at M=1, sharded faster at
// M=4096).  The decision depends on the shape and the session setting only,
// so every rank makes it alike (ORT_CUDA_REPLICATE_BYTES must be equal on
// all ranks).
constexpr int64_t kReplicateBytes = 10000000;
bool replicate_nbits(const ort_cuda_session* s, int64_t bytes) {
  if (s->world <= 1) return false;
  return bytes <= (s->replicate_bytes >= 0 ? s->replicate_bytes : kReplicateBytes);
}

// A kernel whose bounded wait gave up wrote a code into the host-mapped
// error word; report it once.
}  // namespace

int check_kernel_error(ort_cuda_session* s) {
  volatile int* e = s->err_host;
  if (!e || *e == 0) return ORT_CUDA_OK;
  const int code = *e;
  *e = 0;
  return fail(ORT_CUDA_ERR_TIMEOUT,
              "a kernel wait exceeded its bound (code " + std::to_string(code) +
                  "); the kernel stopped and returned");
}

// Bounded wait on the session stream.  Polls an event so that a collective
// whose peer never arrives is detected on the host (no device spin); on
// expiry the NCCL communicator is aborted, which ends its kernels.
int bounded_sync(ort_cuda_session* s) {
  if (s->world == 1 || !s->nccl) {
    ORTC_CUDA(cudaStreamSynchronize(s->stream));
    return check_kernel_error(s);
  }
  // One event per session, recorded anew by every call.
  if (!s->sync_ev) ORTC_CUDA(cudaEventCreateWithFlags(&s->sync_ev, cudaEventDisableTiming));
  ORTC_CUDA(cudaEventRecord(s->sync_ev, s->stream));
  // A decode-sized op finishes within tens of microseconds: poll without
  // sleeping for the first 2 ms (a sleep granule would dominate such a
  // call), then back off to 20 us sleeps.
  const auto t0 = std::chrono::steady_clock::now();
  for (int polls = 0;; polls++) {
    const cudaError_t e = cudaEventQuery(s->sync_ev);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return cuda_fail(e, "cudaEventQuery");
    const auto us = std::chrono::duration_cast<std::chrono::microseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if ((polls & 63) == 0 || us > 2000) {
      ncclResult_t ar = ncclSuccess;
      nccl()->CommGetAsyncError((ncclComm_t)s->nccl, &ar);
      if (ar != ncclSuccess && ar != ncclInProgress) {
        nccl()->CommAbort((ncclComm_t)s->nccl);
        s->nccl = nullptr;
        return fail(ORT_CUDA_ERR_NCCL,
                    std::string("NCCL async error: ") + nccl()->GetErrorString(ar));
      }
    }
    if (us > (int64_t)s->timeout_ms * 1000) {
      nccl()->CommAbort((ncclComm_t)s->nccl);
      s->nccl = nullptr;
      return fail(ORT_CUDA_ERR_TIMEOUT, "collective did not complete within " +
                                            std::to_string(s->timeout_ms) +
                                            " ms; communicator aborted");
    }
    if (us > 2000) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return check_kernel_error(s);
}

int nccl_wait_ready(ncclComm_t comm, int timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl()->CommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return fail(ORT_CUDA_ERR_NCCL, nccl()->GetErrorString(r));
    if (st == ncclSuccess) return ORT_CUDA_OK;
    if (st != ncclInProgress) return fail(ORT_CUDA_ERR_NCCL, nccl()->GetErrorString(st));
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > timeout_ms)
      return fail(ORT_CUDA_ERR_TIMEOUT, "NCCL did not finish within " +
                                            std::to_string(timeout_ms) + " ms");
    // an enqueue completes in microseconds: spin first, sleep only when long
    if (ms < 2)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

namespace {

// All-gather this rank's [M, Ns] slice (at `local`) into Y [M, N].
int gather_y(ort_cuda_session* s, const float* local, float* gathered, float* Y, int64_t M,
             int64_t Ns, int64_t N) {
  if (!s->nccl) return fail(ORT_CUDA_ERR_NCCL, "session communicator is not usable");
  ncclResult_t r = nccl()->AllGather(local, gathered, (size_t)(M * Ns), ncclFloat,
                                 (ncclComm_t)s->nccl, s->stream);
  if (r != ncclSuccess && r != ncclInProgress)
    return fail(ORT_CUDA_ERR_NCCL, std::string("ncclAllGather: ") + nccl()->GetErrorString(r));
  if (r == ncclInProgress) {
    // Non-blocking communicator: the collective is on the stream only once
    // the call has completed; nothing may follow it (on the stream or the
    // communicator) before that.
    const int rc = nccl_wait_ready((ncclComm_t)s->nccl, s->timeout_ms);
    if (rc) {
      nccl()->CommAbort((ncclComm_t)s->nccl);
      s->nccl = nullptr;
      return rc;
    }
  }
  return launch_unshard(gathered, Y, s->world, M, Ns, N, s->stream, &s->launches);
}

// Host-IO staging: copies `bytes` from host `src` to device `dst` on the
// session stream (directly if src is pinned, else through the pinned
// staging buffer at offset `pin_off`).
int stage_in(ort_cuda_session* s, void* dst, const void* src, size_t bytes, size_t pin_off) {
  if (bytes == 0) return ORT_CUDA_OK;
  if (is_pinned_host(src)) {
    ORTC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s->stream));
    return ORT_CUDA_OK;
  }
  std::memcpy((char*)s->pinned + pin_off, src, bytes);
  ORTC_CUDA(cudaMemcpyAsync(dst, (char*)s->pinned + pin_off, bytes, cudaMemcpyHostToDevice,
                            s->stream));
  return ORT_CUDA_OK;
}

struct IoPlan {
  // device-side views used by the kernels
  const float* A = nullptr;
  const float* C = nullptr;
  float* Y = nullptr;
  // host destination (HOST_IO)
  float* Yhost = nullptr;
  size_t ybytes = 0;
  bool yhost_pinned = false;
  size_t pin_y_off = 0;
};

}  // namespace
}  // namespace ortc

using namespace ortc;

extern "C" {

ORT_CUDA_API const char* ort_cuda_last_error(void) { return g_err.c_str(); }

ORT_CUDA_API const char* ort_cuda_version(void) { return "ort_cuda_b200 0.1.0 (sm_100a)"; }

ORT_CUDA_API int ort_cuda_device_count(int* count) {
  ORTC_CHECK(count, ORT_CUDA_ERR_INVALID_ARG, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *count = 0;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return ORT_CUDA_OK;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  *count = n;
  return ORT_CUDA_OK;
}

static int open_common(int device, int mode, ort_cuda_session** out) {
  ORTC_CHECK(out, ORT_CUDA_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  ORTC_CHECK(valid_mode(mode), ORT_CUDA_ERR_INVALID_ARG, "unknown mode");
  int n = 0;
  int rc = ort_cuda_device_count(&n);
  if (rc) return rc;
  ORTC_CHECK(n > 0, ORT_CUDA_ERR_CUDA, "no CUDA device visible");
  ORTC_CHECK(device >= 0 && device < n, ORT_CUDA_ERR_INVALID_ARG,
             "device index " + std::to_string(device) + " out of range");
  ORTC_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  ORTC_CUDA(cudaGetDeviceProperties(&prop, device));
  ORTC_CHECK(prop.major == 10 && prop.minor == 0, ORT_CUDA_ERR_UNSUPPORTED,
             std::string("this library is built for sm_100a (B200); device is ") + prop.name);
  auto* s = new ort_cuda_session();
  s->device = device;
  s->mode = mode;
  s->sm_count = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete s;
    return cuda_fail(e, "cudaStreamCreate");
  }
  s->stream = s->own_stream;
  e = cudaHostAlloc((void**)&s->err_host, 64, cudaHostAllocMapped);
  if (e == cudaSuccess) e = cudaHostGetDevicePointer((void**)&s->err_dev, s->err_host, 0);
  if (e != cudaSuccess) {
    cudaStreamDestroy(s->own_stream);
    if (s->err_host) cudaFreeHost(s->err_host);
    delete s;
    return cuda_fail(e, "cudaHostAlloc(error word)");
  }
  *s->err_host = 0;
  *out = s;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_open(int device, int mode, ort_cuda_session** out) {
  return open_common(device, mode, out);
}

ORT_CUDA_API int ort_cuda_nccl_unique_id(void* id128) {
  ORTC_CHECK(id128, ORT_CUDA_ERR_INVALID_ARG, "id buffer is NULL");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  if (!nccl()) return ORT_CUDA_ERR_NCCL;
  ncclUniqueId id;
  ncclResult_t r = nccl()->GetUniqueId(&id);
  if (r != ncclSuccess) return fail(ORT_CUDA_ERR_NCCL, nccl()->GetErrorString(r));
  std::memcpy(id128, &id, 128);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_open_rank(int device, int rank, int world, const void* nccl_id128,
                                    int mode, int timeout_ms, ort_cuda_session** out) {
  ORTC_CHECK(world >= 1 && rank >= 0 && rank < world, ORT_CUDA_ERR_INVALID_ARG,
             "rank/world out of range");
  ORTC_CHECK(world == 1 || nccl_id128, ORT_CUDA_ERR_INVALID_ARG, "NCCL id is NULL");
  ORTC_CHECK(timeout_ms > 0, ORT_CUDA_ERR_INVALID_ARG, "timeout_ms must be > 0");
  if (world > 1 && !nccl()) return ORT_CUDA_ERR_NCCL;
  int rc = open_common(device, mode, out);
  if (rc) return rc;
  ort_cuda_session* s = *out;
  s->rank = rank;
  s->world = world;
  s->timeout_ms = timeout_ms;
  if (const char* env = std::getenv("ORT_CUDA_REPLICATE_BYTES"))
    s->replicate_bytes = std::strtoll(env, nullptr, 10);
  if (world == 1) return ORT_CUDA_OK;
  ncclUniqueId id;
  std::memcpy(&id, nccl_id128, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = nccl()->CommInitRankConfig(&comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    ort_cuda_close(s);
    *out = nullptr;
    return fail(ORT_CUDA_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + nccl()->GetErrorString(r));
  }
  rc = nccl_wait_ready(comm, timeout_ms);
  if (rc) {
    std::string msg = ort_cuda_last_error();
    nccl()->CommAbort(comm);
    ort_cuda_close(s);
    *out = nullptr;
    return fail(rc, "NCCL init (rank " + std::to_string(rank) + "/" + std::to_string(world) +
                        "): " + msg);
  }
  s->nccl = comm;
  rc = p2p_setup(s);
  if (rc) {
    std::string msg = ort_cuda_last_error();
    ort_cuda_close(s);
    *out = nullptr;
    return fail(rc, "peer-memory setup: " + msg);
  }
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_close(ort_cuda_session* s) {
  if (!s) return ORT_CUDA_OK;
  DeviceGuard g(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  for (auto& kv : s->weights) free_weight(kv.second);
  s->weights.clear();
  for (void* p : s->allocs) cudaFree(p);
  s->allocs.clear();
  if (s->ws) cudaFree(s->ws);
  if (s->kscratch) cudaFree(s->kscratch);
  if (s->argscratch) cudaFree(s->argscratch);
  if (s->dqscratch) cudaFree(s->dqscratch);
  if (s->attnscratch) cudaFree(s->attnscratch);
  if (s->pinned) cudaFreeHost(s->pinned);
  if (s->err_host) cudaFreeHost(s->err_host);
  for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second.exec);
  s->graphs.clear();
  profile_free(s);
  if (s->sync_ev) cudaEventDestroy(s->sync_ev);
  if (s->aux) cudaFree(s->aux);
  if (s->amaxbuf) cudaFree(s->amaxbuf);
  for (cudaEvent_t& e : s->chunk_ev)
    if (e) cudaEventDestroy(e);
  if (s->comm_stream) cudaStreamDestroy(s->comm_stream);
  s->comm_stream = nullptr;
  s->sync_ev = nullptr;
  p2p_teardown(s);
  if (s->nccl) {
    nccl()->CommFinalize((ncclComm_t)s->nccl);
    nccl_wait_ready((ncclComm_t)s->nccl, s->timeout_ms);
    nccl()->CommDestroy((ncclComm_t)s->nccl);
  }
  if (s->own_stream) cudaStreamDestroy(s->own_stream);
  delete s;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_set_mode(ort_cuda_session* s, int mode) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  ORTC_CHECK(valid_mode(mode), ORT_CUDA_ERR_INVALID_ARG, "unknown mode");
  s->mode = mode;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_set_stream(ort_cuda_session* s, void* stream) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  s->stream = stream ? (cudaStream_t)stream : s->own_stream;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_sync(ort_cuda_session* s) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG, "cannot synchronise during a capture");
  DeviceGuard g(s->device);
  return bounded_sync(s);
}

ORT_CUDA_API int ort_cuda_set_peer_wait(ort_cuda_session* s, int ms) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  ORTC_CHECK(ms >= 1 && ms <= 600000, ORT_CUDA_ERR_INVALID_ARG,
             "peer wait must be 1 .. 600000 ms");
  s->peer_wait_ms = ms;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_set_replicate_bytes(ort_cuda_session* s, int64_t bytes) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  ORTC_CHECK(bytes >= -1, ORT_CUDA_ERR_INVALID_ARG, "replicate bytes must be >= -1");
  s->replicate_bytes = bytes;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_weight_columns(ort_cuda_session* s, const char* name, int64_t* n0,
                                         int64_t* nl) {
  ORTC_CHECK(s && name && n0 && nl, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  const Weight& w = it->second;
  *n0 = w.group_only ? 0 : w.n0;
  *nl = w.group_only ? 0 : w.nl;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_rank_info(ort_cuda_session* s, int* rank, int* world) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  if (rank) *rank = s->rank;
  if (world) *world = s->world;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_graph_begin(ort_cuda_session* s) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "NULL session");
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG, "a capture is already in progress");
  ORTC_CHECK(s->stream != nullptr && s->stream != cudaStreamLegacy &&
                 s->stream != cudaStreamPerThread,
             ORT_CUDA_ERR_INVALID_ARG, "the legacy default stream cannot be captured");
  DeviceGuard g(s->device);
  ORTC_CUDA(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeRelaxed));
  s->capturing = true;
  s->capture_launch0 = s->launches;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_graph_end(ort_cuda_session* s, int* graph_id) {
  ORTC_CHECK(s && graph_id, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(s->capturing, ORT_CUDA_ERR_INVALID_ARG, "no capture in progress");
  DeviceGuard g(s->device);
  s->capturing = false;
  cudaGraph_t graph = nullptr;
  ORTC_CUDA(cudaStreamEndCapture(s->stream, &graph));
  cudaGraphExec_t exec = nullptr;
  cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
  const int id = s->next_graph++;
  s->graphs[id] = {exec, s->launches - s->capture_launch0};
  s->launches = s->capture_launch0;  // captured launches run when the graph does
  *graph_id = id;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_graph_launch(ort_cuda_session* s, int graph_id) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "NULL session");
  auto it = s->graphs.find(graph_id);
  ORTC_CHECK(it != s->graphs.end(), ORT_CUDA_ERR_NOT_FOUND,
             "no graph with id " + std::to_string(graph_id));
  DeviceGuard g(s->device);
  ORTC_CUDA(cudaGraphLaunch(it->second.exec, s->stream));
  s->launches += it->second.launches;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_graph_drop(ort_cuda_session* s, int graph_id) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "NULL session");
  auto it = s->graphs.find(graph_id);
  ORTC_CHECK(it != s->graphs.end(), ORT_CUDA_ERR_NOT_FOUND,
             "no graph with id " + std::to_string(graph_id));
  DeviceGuard g(s->device);
  cudaGraphExecDestroy(it->second.exec);
  s->graphs.erase(it);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_launch_count(ort_cuda_session* s, int64_t* count) {
  ORTC_CHECK(s && count, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  *count = s->launches;
  return ORT_CUDA_OK;
}

// ---- weights ---------------------------------------------------------------

}  // extern "C"

namespace {
// Fills dst (device) with bytes [off, off + bytes) of the packed B of a
// MatMulNBits weight, on the session stream.
using BSource = std::function<int(void* dst, int64_t off, int64_t bytes)>;

int upload_nbits_impl(ort_cuda_session* s, const char* name, const BSource& Bsrc,
                      const void* scales, const uint8_t* zp, int64_t K, int64_t N, int bits,
                      int block_size, int flags) {
  if (bits != 4)
    return fail(ORT_CUDA_ERR_UNSUPPORTED,
                "MatMulNBits: only bits=4 supported, got " + std::to_string(bits));
  ORTC_CHECK(K > 0 && N > 0 && K < (1ll << 31) && N < (1ll << 31), ORT_CUDA_ERR_INVALID_ARG,
             "MatMulNBits: K and N must be in [1, 2^31)");
  ORTC_CHECK(block_size >= 16 && (block_size & (block_size - 1)) == 0, ORT_CUDA_ERR_INVALID_ARG,
             "MatMulNBits: block_size must be a power of two >= 16, got " +
                 std::to_string(block_size));
  DeviceGuard g(s->device);
  const int64_t nb = (K + block_size - 1) / block_size;
  const int64_t col_bytes = nb * block_size / 2;
  Weight w;
  w.kind = W_NBITS;
  w.K = K;
  w.N = N;
  w.bs = block_size;
  w.nb = (int)nb;
  w.has_zp = zp != nullptr;
  const bool f16 = (flags & ORT_CUDA_SCALES_F16) != 0;
  w.replicated = replicate_nbits(
      s, N * col_bytes + N * nb * (f16 ? 2 : 4) + (w.has_zp ? N * ((nb + 1) / 2) : 0));
  if (w.replicated) {
    w.n0 = 0;
    w.nl = w.ns = N;
  } else {
    shard_cols(N, s->rank, s->world, &w.n0, &w.nl, &w.ns);
  }
  const int64_t nl = w.nl;
  auto cleanup = [&](int rc) {
    free_weight(w);
    return rc;
  };
  cudaError_t e;
  if (nl > 0) {
    // Packed B: this rank's columns are contiguous; upload, then reorder
    // the nibbles of every 32-bit word into the device layout.
    uint8_t* tmpB = nullptr;
    e = cudaMalloc(&tmpB, (size_t)(nl * col_bytes));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(B staging)"));
    e = cudaMalloc(&w.B, (size_t)(nl * col_bytes));
    int rc = e == cudaSuccess ? Bsrc(tmpB, w.n0 * col_bytes, nl * col_bytes)
                              : cuda_fail(e, "cudaMalloc(B)");
    if (!rc)
      rc = launch_permute_nibbles((const uint32_t*)tmpB, (uint32_t*)w.B, nl * col_bytes / 4,
                                  s->stream, &s->launches);
    cudaStreamSynchronize(s->stream);
    cudaFree(tmpB);
    if (rc) return cleanup(rc);
    // Scales: fp32 (fp16 widened bit-exactly on the device), transposed to
    // block-major [nb][s_pitch].
    w.s_pitch = (nl + 3) / 4 * 4;
    float* tmpS = nullptr;
    e = cudaMalloc(&tmpS, (size_t)(nl * nb * 4));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(scale staging)"));
    e = cudaMalloc(&w.scales, (size_t)(nb * w.s_pitch * 4));
    if (e == cudaSuccess) e = cudaMemsetAsync(w.scales, 0, (size_t)(nb * w.s_pitch * 4), s->stream);
    if (e == cudaSuccess) {
      if (f16) {
        uint16_t* tmp16 = nullptr;
        e = cudaMalloc(&tmp16, (size_t)(nl * nb * 2));
        if (e == cudaSuccess)
          e = cudaMemcpyAsync(tmp16, (const uint16_t*)scales + w.n0 * nb, (size_t)(nl * nb * 2),
                              cudaMemcpyHostToDevice, s->stream);
        rc = e == cudaSuccess ? launch_half_to_float(tmp16, tmpS, nl * nb, s->stream, &s->launches)
                              : cuda_fail(e, "copy scales");
        cudaStreamSynchronize(s->stream);
        if (tmp16) cudaFree(tmp16);
      } else {
        e = cudaMemcpyAsync(tmpS, (const float*)scales + w.n0 * nb, (size_t)(nl * nb * 4),
                            cudaMemcpyHostToDevice, s->stream);
        rc = e == cudaSuccess ? ORT_CUDA_OK : cuda_fail(e, "copy scales");
      }
    } else {
      rc = cuda_fail(e, "cudaMalloc(scales)");
    }
    // [nl][nb] -> [nb][s_pitch]: transpose into a padded pitch via a dense
    // [nb][nl] temporary then a pitched copy.
    float* tmpT = nullptr;
    if (!rc) {
      e = cudaMalloc(&tmpT, (size_t)(nl * nb * 4));
      rc = e == cudaSuccess ? launch_transpose(tmpS, tmpT, nl, nb, s->stream, &s->launches)
                            : cuda_fail(e, "cudaMalloc(scale transpose)");
    }
    if (!rc) {
      e = cudaMemcpy2DAsync(w.scales, (size_t)(w.s_pitch * 4), tmpT, (size_t)(nl * 4),
                            (size_t)(nl * 4), (size_t)nb, cudaMemcpyDeviceToDevice, s->stream);
      if (e != cudaSuccess) rc = cuda_fail(e, "pitch scales");
    }
    cudaStreamSynchronize(s->stream);
    cudaFree(tmpS);
    if (tmpT) cudaFree(tmpT);
    if (rc) return cleanup(rc);
    if (f16) {
      // fp16 scales also block-major [nb][s16_pitch] as fp16: the decode
      // GEMV streams these (half the bytes; widened exactly in its epilogue)
      w.s16_pitch = (nl + 7) / 8 * 8;
      std::vector<uint16_t> t((size_t)(nb * w.s16_pitch), 0);
      const uint16_t* src = (const uint16_t*)scales + w.n0 * nb;
      for (int64_t c = 0; c < nl; c++)
        for (int64_t b = 0; b < nb; b++) t[(size_t)(b * w.s16_pitch + c)] = src[c * nb + b];
      e = cudaMalloc(&w.scales16, t.size() * 2);
      if (e == cudaSuccess) e = cudaMemcpy(w.scales16, t.data(), t.size() * 2, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return cleanup(cuda_fail(e, "fp16 scales"));
    }
    if (zp) {
      // Zero points from either input layout (the reference's flat nibble
      // n*nb + blk, onnx_qlinear_ops.dart:135-137, or ORT's per-column
      // padding) into the transposed table [ceil(nb/2)][z_pitch].
      w.z_pitch = (nl + 15) / 16 * 16;
      const int64_t zrows = (nb + 1) / 2;
      std::vector<uint8_t> z((size_t)(zrows * w.z_pitch), 0);
      const bool per_col = (flags & ORT_CUDA_ZP_PER_COLUMN) != 0;
      const int64_t col_zbytes = (nb + 1) / 2;
      for (int64_t c = 0; c < nl; c++) {
        const int64_t gc = w.n0 + c;
        for (int64_t b = 0; b < nb; b++) {
          uint8_t v;
          if (per_col) {
            const uint8_t byte = zp[gc * col_zbytes + (b >> 1)];
            v = (b & 1) ? (byte >> 4) : (byte & 0xF);
          } else {
            const int64_t zi = gc * nb + b;
            const uint8_t byte = zp[zi >> 1];
            v = (zi & 1) ? (byte >> 4) : (byte & 0xF);
          }
          z[(size_t)((b >> 1) * w.z_pitch + c)] |= (uint8_t)(v << ((b & 1) * 4));
        }
      }
      e = cudaMalloc(&w.zp, z.size());
      if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(zp)"));
      e = cudaMemcpy(w.zp, z.data(), z.size(), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return cleanup(cuda_fail(e, "copy zp"));
    }
    e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "upload sync"));
    rc = prepare_nbits_tc(w);
    if (rc) return cleanup(rc);
  }
  auto it = s->weights.find(name);
  if (it != s->weights.end()) {
    free_weight(it->second);
    s->weights.erase(it);
  }
  s->weights.emplace(name, w);
  return ORT_CUDA_OK;
}

// Reads [off, off + len) of an open file completely (pread loops over short
// reads); false on error or end of file.
bool read_at(int fd, void* dst, int64_t off, int64_t len) {
  char* p = static_cast<char*>(dst);
  while (len > 0) {
    const ssize_t r = pread(fd, p, (size_t)std::min<int64_t>(len, 1 << 30), (off_t)off);
    if (r <= 0) return false;
    p += r;
    off += r;
    len -= r;
  }
  return true;
}

struct FdCloser {
  int fd;
  ~FdCloser() {
    if (fd >= 0) close(fd);
  }
};
}  // namespace

extern "C" {

ORT_CUDA_API int ort_cuda_upload_nbits(ort_cuda_session* s, const char* name, const uint8_t* B,
                                       const void* scales, const uint8_t* zp, int64_t K,
                                       int64_t N, int bits, int block_size, int flags) {
  ORTC_CHECK(s && name && B && scales, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  const BSource from_host = [&](void* dst, int64_t off, int64_t bytes) -> int {
    ORTC_CUDA(cudaMemcpyAsync(dst, B + off, (size_t)bytes, cudaMemcpyHostToDevice, s->stream));
    return ORT_CUDA_OK;
  };
  return upload_nbits_impl(s, name, from_host, scales, zp, K, N, bits, block_size, flags);
}

ORT_CUDA_API int ort_cuda_upload_nbits_file(ort_cuda_session* s, const char* name,
                                            const char* path, int64_t b_offset,
                                            int64_t scales_offset, int64_t zp_offset, int64_t K,
                                            int64_t N, int bits, int block_size, int flags) {
  ORTC_CHECK(s && name && path, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
             "weights cannot be uploaded while a CUDA graph is being captured");
  ORTC_CHECK(K > 0 && N > 0 && K < (1ll << 31) && N < (1ll << 31) && block_size >= 16,
             ORT_CUDA_ERR_INVALID_ARG, "MatMulNBits: bad K, N or block_size");
  const int fd = open(path, O_RDONLY);
  ORTC_CHECK(fd >= 0, ORT_CUDA_ERR_INVALID_ARG, std::string("cannot open '") + path + "'");
  FdCloser closer{fd};
  struct stat st;
  ORTC_CHECK(fstat(fd, &st) == 0, ORT_CUDA_ERR_INVALID_ARG, std::string("cannot stat '") + path + "'");
  const int64_t fsize = (int64_t)st.st_size;
  const int64_t nb = (K + block_size - 1) / block_size;
  const int64_t col_bytes = nb * block_size / 2;
  const bool f16 = (flags & ORT_CUDA_SCALES_F16) != 0;
  const int64_t b_bytes = N * col_bytes, s_bytes = N * nb * (f16 ? 2 : 4);
  const int64_t z_bytes =
      (flags & ORT_CUDA_ZP_PER_COLUMN) ? N * ((nb + 1) / 2) : (N * nb + 1) / 2;
  // every range inside the file (the reference rejects a reference outside
  // the companion file, onnx_runtime_dart_io.dart:55-80)
  auto inside = [&](int64_t off, int64_t len) { return off >= 0 && off <= fsize - len; };
  ORTC_CHECK(inside(b_offset, b_bytes) && inside(scales_offset, s_bytes) &&
                 (zp_offset < 0 || inside(zp_offset, z_bytes)),
             ORT_CUDA_ERR_INVALID_ARG,
             std::string("MatMulNBits external data: a range lies outside '") + path + "' (" +
                 std::to_string(fsize) + " bytes)");
  std::vector<uint8_t> sc((size_t)s_bytes), zz(zp_offset >= 0 ? (size_t)z_bytes : 0);
  ORTC_CHECK(read_at(fd, sc.data(), scales_offset, s_bytes) &&
                 (zp_offset < 0 || read_at(fd, zz.data(), zp_offset, z_bytes)),
             ORT_CUDA_ERR_INVALID_ARG, std::string("short read from '") + path + "'");
  DeviceGuard g(s->device);
  // B through two pinned bounce buffers: the read of one chunk overlaps the
  // copy of the previous one
  constexpr int64_t kChunk = 16 << 20;
  int rc = ensure_pinned(s, 2 * kChunk);
  if (rc) return rc;
  cudaEvent_t done[2] = {nullptr, nullptr};
  for (auto& ev : done) ORTC_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  const BSource from_file = [&](void* dst, int64_t off, int64_t bytes) -> int {
    for (int64_t c = 0, i = 0; c < bytes; c += kChunk, i++) {
      const int64_t len = std::min(kChunk, bytes - c);
      char* buf = static_cast<char*>(s->pinned) + (i & 1) * kChunk;
      ORTC_CUDA(cudaEventSynchronize(done[i & 1]));  // its previous copy has ended
      if (!read_at(fd, buf, b_offset + off + c, len))
        return fail(ORT_CUDA_ERR_INVALID_ARG, std::string("short read from '") + path + "'");
      ORTC_CUDA(cudaMemcpyAsync(static_cast<char*>(dst) + c, buf, (size_t)len,
                                cudaMemcpyHostToDevice, s->stream));
      ORTC_CUDA(cudaEventRecord(done[i & 1], s->stream));
    }
    return ORT_CUDA_OK;
  };
  rc = upload_nbits_impl(s, name, from_file, sc.data(), zp_offset >= 0 ? zz.data() : nullptr, K,
                         N, bits, block_size, flags);
  cudaStreamSynchronize(s->stream);
  for (auto& ev : done) cudaEventDestroy(ev);
  return rc;
}

ORT_CUDA_API int ort_cuda_upload_int8(ort_cuda_session* s, const char* name, const void* B,
                                      int64_t K, int64_t N, int b_signed, const void* b_zp,
                                      int64_t b_zp_len) {
  ORTC_CHECK(s && name && B, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(K > 0 && N > 0 && K < (1ll << 30) && N < (1ll << 31), ORT_CUDA_ERR_INVALID_ARG,
             "MatMulInteger: K and N must be positive");
  ORTC_CHECK(b_zp == nullptr || b_zp_len == 1 || b_zp_len == N, ORT_CUDA_ERR_UNSUPPORTED,
             "MatMulInteger: b_zp must be scalar or per-column [N]");
  DeviceGuard g(s->device);
  Weight w;
  w.kind = W_INT8;
  w.K = K;
  w.N = N;
  shard_cols(N, s->rank, s->world, &w.n0, &w.nl, &w.ns);
  w.i8_signed = b_signed ? 1 : 0;
  w.kpitch = (K + 15) / 16 * 16;
  const int64_t nl = w.nl;
  auto cleanup = [&](int rc) {
    free_weight(w);
    return rc;
  };
  if (nl > 0) {
    // B [K][N] -> this rank's columns K-major, with their sums
    const uint8_t* b = static_cast<const uint8_t*>(B);
    std::vector<uint8_t> t((size_t)(nl * w.kpitch), 0);
    std::vector<int32_t> cs((size_t)nl, 0), zp;
    for (int64_t k = 0; k < K; k++) {
      const uint8_t* row = b + k * N + w.n0;
      for (int64_t c = 0; c < nl; c++) {
        t[(size_t)(c * w.kpitch + k)] = row[c];
        cs[(size_t)c] += b_signed ? (int32_t)(int8_t)row[c] : (int32_t)row[c];
      }
    }
    if (b_zp) {
      const uint8_t* z = static_cast<const uint8_t*>(b_zp);
      zp.resize((size_t)nl);
      for (int64_t c = 0; c < nl; c++) {
        const uint8_t v = z[b_zp_len == 1 ? 0 : w.n0 + c];
        zp[(size_t)c] = b_signed ? (int32_t)(int8_t)v : (int32_t)v;
      }
    }
    cudaError_t e = cudaMalloc(&w.Wi8, t.size());
    if (e == cudaSuccess) e = cudaMemcpy(w.Wi8, t.data(), t.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&w.colsum, cs.size() * 4);
    if (e == cudaSuccess) e = cudaMemcpy(w.colsum, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && b_zp) e = cudaMalloc(&w.bzp, zp.size() * 4);
    if (e == cudaSuccess && b_zp)
      e = cudaMemcpy(w.bzp, zp.data(), zp.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "MatMulInteger weight upload"));
    const int rc = prepare_int8_tc(w);
    if (rc) return cleanup(rc);
  }
  auto it = s->weights.find(name);
  if (it != s->weights.end()) {
    free_weight(it->second);
    s->weights.erase(it);
  }
  s->weights.emplace(name, w);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_upload_dense(ort_cuda_session* s, const char* name, const float* B,
                                       int64_t rows, int64_t cols, int trans_b) {
  ORTC_CHECK(s && name && B, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(rows > 0 && cols > 0 && rows < (1ll << 31) && cols < (1ll << 31),
             ORT_CUDA_ERR_INVALID_ARG, "dense weight: bad shape");
  DeviceGuard g(s->device);
  Weight w;
  w.kind = W_DENSE;
  w.K = trans_b ? cols : rows;
  w.N = trans_b ? rows : cols;
  shard_cols(w.N, s->rank, s->world, &w.n0, &w.nl, &w.ns);
  auto cleanup = [&](int rc) {
    free_weight(w);
    return rc;
  };
  cudaError_t e;
  if (w.nl > 0) {
    e = cudaMalloc(&w.W, (size_t)(w.K * w.nl * 4));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(W)"));
    if (trans_b) {
      // B [N, K]: this rank's rows [n0, n0+nl) are contiguous; transpose
      // them on the device into [K, nl] (the prepack of
      // onnx_graph.dart:1159-1161, once per session).
      float* tmp = nullptr;
      e = cudaMalloc(&tmp, (size_t)(w.nl * w.K * 4));
      if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(tmp)"));
      e = cudaMemcpyAsync(tmp, B + w.n0 * w.K, (size_t)(w.nl * w.K * 4), cudaMemcpyHostToDevice,
                          s->stream);
      int rc = e == cudaSuccess ? launch_transpose(tmp, w.W, w.nl, w.K, s->stream, &s->launches)
                                : cuda_fail(e, "copy B");
      cudaStreamSynchronize(s->stream);
      cudaFree(tmp);
      if (rc) return cleanup(rc);
    } else {
      e = cudaMemcpy2DAsync(w.W, (size_t)(w.nl * 4), B + w.n0, (size_t)(w.N * 4),
                            (size_t)(w.nl * 4), (size_t)w.K, cudaMemcpyHostToDevice, s->stream);
      if (e != cudaSuccess) return cleanup(cuda_fail(e, "copy B"));
    }
    e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "upload sync"));
  }
  auto it = s->weights.find(name);
  if (it != s->weights.end()) {
    free_weight(it->second);
    s->weights.erase(it);
  }
  s->weights.emplace(name, w);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_drop_weight(ort_cuda_session* s, const char* name) {
  ORTC_CHECK(s && name, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  DeviceGuard g(s->device);
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  cudaStreamSynchronize(s->stream);
  free_weight(it->second);
  s->weights.erase(it);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_gemv_plan_get(ort_cuda_session* s, const char* name, int M, int* plan) {
  ORTC_CHECK(s && name && plan, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 1 && M <= 8, ORT_CUDA_ERR_INVALID_ARG, "M must be in 1..8");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  *plan = it->second.gemv_plan[M];
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_gemv_plan_set(ort_cuda_session* s, const char* name, int M, int plan) {
  ORTC_CHECK(s && name, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 1 && M <= 8, ORT_CUDA_ERR_INVALID_ARG, "M must be in 1..8");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  Weight& w = it->second;
  ORTC_CHECK(w.kind == W_NBITS && tc_gemv_ok(w, M), ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + name + "' has no decode-GEMV plans for this M");
  DeviceGuard g(s->device);
  const int n = tc_gemv_plan_count(w, M, s->sm_count);
  ORTC_CHECK(plan >= -1 && plan < n, ORT_CUDA_ERR_INVALID_ARG,
             "plan " + std::to_string(plan) + " outside [-1, " + std::to_string(n) + ")");
  w.gemv_plan[M] = (int8_t)plan;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_weight_shape(ort_cuda_session* s, const char* name, int64_t* K,
                                       int64_t* N) {
  ORTC_CHECK(s && name, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  if (K) *K = it->second.K;
  if (N) *N = it->second.N;
  return ORT_CUDA_OK;
}

// ---- device tensors ----------------------------------------------------------

ORT_CUDA_API int ort_cuda_alloc(ort_cuda_session* s, int64_t bytes, void** dptr) {
  ORTC_CHECK(s && dptr, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(bytes >= 0, ORT_CUDA_ERR_INVALID_ARG, "negative size");
  DeviceGuard g(s->device);
  void* p = nullptr;
  ORTC_CUDA(cudaMalloc(&p, bytes > 0 ? (size_t)bytes : 16));
  s->allocs.insert(p);
  *dptr = p;
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_free(ort_cuda_session* s, void* dptr) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  if (!dptr) return ORT_CUDA_OK;
  DeviceGuard g(s->device);
  auto it = s->allocs.find(dptr);
  ORTC_CHECK(it != s->allocs.end(), ORT_CUDA_ERR_INVALID_ARG,
             "pointer was not allocated by this session");
  cudaStreamSynchronize(s->stream);
  ORTC_CUDA(cudaFree(dptr));
  s->allocs.erase(it);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_h2d(ort_cuda_session* s, void* dst, const void* src, int64_t bytes) {
  ORTC_CHECK(s && dst && src && bytes >= 0, ORT_CUDA_ERR_INVALID_ARG, "bad argument");
  DeviceGuard g(s->device);
  ORTC_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyHostToDevice, s->stream));
  return bounded_sync(s);
}

ORT_CUDA_API int ort_cuda_d2h(ort_cuda_session* s, void* dst, const void* src, int64_t bytes) {
  ORTC_CHECK(s && dst && src && bytes >= 0, ORT_CUDA_ERR_INVALID_ARG, "bad argument");
  DeviceGuard g(s->device);
  ORTC_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToHost, s->stream));
  return bounded_sync(s);
}

ORT_CUDA_API int ort_cuda_argmax(ort_cuda_session* s, const float* X, int64_t rows,
                                 int64_t cols, int64_t ldx, int64_t* out, int flags) {
  ORTC_CHECK(s && X && out, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(rows >= 0 && cols >= 1 && ldx >= cols, ORT_CUDA_ERR_INVALID_ARG,
             "ArgMax: need rows >= 0 and 1 <= cols <= ldx");
  if (rows == 0) return ORT_CUDA_OK;
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  DeviceGuard g(s->device);
  OpTimer timer(s, "ArgMax");
  const int64_t ncand = argminmax_candidates(rows, cols);
  if (ncand > 0 && (rows > s->arg_rows_cap || ncand > s->arg_cand_cap)) {
    ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
               "a buffer would grow while a CUDA graph is being captured; run every "
               "operation of the graph once before capturing it");
    if (s->argscratch) {
      ORTC_CUDA(cudaStreamSynchronize(s->stream));
      ORTC_CUDA(cudaFree(s->argscratch));
      s->argscratch = nullptr;
      s->arg_rows_cap = s->arg_cand_cap = 0;
    }
    const int64_t rcap = std::max<int64_t>(rows, 64), ccap = std::max<int64_t>(ncand, 512);
    const size_t bytes = ((size_t)rcap * 4 + 255) / 256 * 256 + (size_t)ccap * argminmax_candidate_bytes();
    ORTC_CUDA(cudaMalloc(&s->argscratch, bytes));
    ORTC_CUDA(cudaMemsetAsync(s->argscratch, 0, bytes, s->stream));
    s->arg_rows_cap = rcap;
    s->arg_cand_cap = ccap;
  }
  unsigned* tickets = static_cast<unsigned*>(s->argscratch);
  void* cands = s->argscratch
                    ? static_cast<char*>(s->argscratch) + ((size_t)s->arg_rows_cap * 4 + 255) / 256 * 256
                    : nullptr;
  const bool is_min = (flags & ORT_CUDA_ARG_MIN) != 0;
  const bool last = (flags & ORT_CUDA_ARG_SELECT_LAST) != 0;
  if (!host)
    return launch_argminmax(X, rows, cols, ldx, is_min, last, out, tickets, cands, s->stream,
                            &s->launches);
  // host buffers: the rows in, the indices back, synchronously
  const size_t xbytes = (size_t)(rows * cols) * 4, obytes = (size_t)rows * 8;
  int rc = ensure_ws(s, xbytes + obytes + 256);
  if (rc) return rc;
  float* dx = static_cast<float*>(s->ws);
  int64_t* dout = reinterpret_cast<int64_t*>(static_cast<char*>(s->ws) + ((xbytes + 255) & ~(size_t)255));
  ORTC_CUDA(cudaMemcpy2DAsync(dx, (size_t)cols * 4, X, (size_t)ldx * 4, (size_t)cols * 4,
                              (size_t)rows, cudaMemcpyHostToDevice, s->stream));
  rc = launch_argminmax(dx, rows, cols, cols, is_min, last, dout, tickets, cands, s->stream,
                        &s->launches);
  if (rc) return rc;
  ORTC_CUDA(cudaMemcpyAsync(out, dout, obytes, cudaMemcpyDeviceToHost, s->stream));
  return bounded_sync(s);
}

ORT_CUDA_API int ort_cuda_dynamic_quantize_linear(ort_cuda_session* s, const float* X, int64_t n,
                                                  uint8_t* Y, float* scale, uint8_t* zp,
                                                  int flags) {
  ORTC_CHECK(s && X && Y && scale && zp && n >= 0, ORT_CUDA_ERR_INVALID_ARG, "bad argument");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  DeviceGuard g(s->device);
  OpTimer timer(s, "DynamicQuantizeLinear");
  if (!s->dqscratch) {
    ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
               "a buffer would grow while a CUDA graph is being captured; run every "
               "operation of the graph once before capturing it");
    const size_t bytes = dynamic_quant_scratch_bytes(s->sm_count);
    ORTC_CUDA(cudaMalloc(&s->dqscratch, bytes));
    ORTC_CUDA(cudaMemsetAsync(s->dqscratch, 0, bytes, s->stream));
  }
  if (!host)
    return launch_dynamic_quant(X, n, Y, scale, zp, s->dqscratch, s->sm_count, s->stream,
                                &s->launches);
  const size_t xb = (size_t)n * 4, off_y = (xb + 255) & ~(size_t)255;
  const size_t off_s = (off_y + (size_t)n + 255) & ~(size_t)255;
  int rc = ensure_ws(s, off_s + 256);
  if (rc) return rc;
  char* ws = static_cast<char*>(s->ws);
  ORTC_CUDA(cudaMemcpyAsync(ws, X, xb, cudaMemcpyHostToDevice, s->stream));
  rc = launch_dynamic_quant(reinterpret_cast<float*>(ws), n, reinterpret_cast<uint8_t*>(ws + off_y),
                            reinterpret_cast<float*>(ws + off_s),
                            reinterpret_cast<uint8_t*>(ws + off_s + 16), s->dqscratch,
                            s->sm_count, s->stream, &s->launches);
  if (rc) return rc;
  ORTC_CUDA(cudaMemcpyAsync(Y, ws + off_y, (size_t)n, cudaMemcpyDeviceToHost, s->stream));
  ORTC_CUDA(cudaMemcpyAsync(scale, ws + off_s, 4, cudaMemcpyDeviceToHost, s->stream));
  ORTC_CUDA(cudaMemcpyAsync(zp, ws + off_s + 16, 1, cudaMemcpyDeviceToHost, s->stream));
  return bounded_sync(s);
}

ORT_CUDA_API int ort_cuda_topk(ort_cuda_session* s, const float* X, int64_t rows, int64_t cols,
                               int64_t ldx, int64_t k, float* values, int64_t* indices,
                               int flags) {
  ORTC_CHECK(s && X && values && indices, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(rows >= 0 && cols >= 0 && ldx >= cols && k >= 0, ORT_CUDA_ERR_INVALID_ARG,
             "TopK: need rows, cols, k >= 0 and ldx >= cols");
  ORTC_CHECK(k <= cols, ORT_CUDA_ERR_INVALID_ARG, "TopK: k exceeds the axis length");
  ORTC_CHECK(k <= 1024, ORT_CUDA_ERR_UNSUPPORTED, "TopK: k above 1024 is not supported");
  if (rows == 0 || k == 0) return ORT_CUDA_OK;
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  DeviceGuard g(s->device);
  OpTimer timer(s, "TopK");
  const bool largest = (flags & ORT_CUDA_TOPK_SMALLEST) == 0;
  const size_t sb = topk_scratch_bytes(rows, cols, k);
  if (sb) {
    int rc0 = ensure_kscratch(s, sb);
    if (rc0) return rc0;
  }
  if (!host)
    return launch_topk(X, rows, cols, ldx, k, largest, values, indices, s->kscratch, s->stream,
                       &s->launches);
  const size_t xb = (size_t)(rows * cols) * 4, vb = (size_t)(rows * k) * 4,
               ib = (size_t)(rows * k) * 8;
  const size_t ov = (xb + 255) & ~(size_t)255, oi = (ov + vb + 255) & ~(size_t)255;
  int rc = ensure_ws(s, oi + ib + 256);
  if (rc) return rc;
  char* ws = static_cast<char*>(s->ws);
  ORTC_CUDA(cudaMemcpy2DAsync(ws, (size_t)cols * 4, X, (size_t)ldx * 4, (size_t)cols * 4,
                              (size_t)rows, cudaMemcpyHostToDevice, s->stream));
  rc = launch_topk(reinterpret_cast<float*>(ws), rows, cols, cols, k, largest,
                   reinterpret_cast<float*>(ws + ov), reinterpret_cast<int64_t*>(ws + oi),
                   s->kscratch, s->stream, &s->launches);
  if (rc) return rc;
  ORTC_CUDA(cudaMemcpyAsync(values, ws + ov, vb, cudaMemcpyDeviceToHost, s->stream));
  ORTC_CUDA(cudaMemcpyAsync(indices, ws + oi, ib, cudaMemcpyDeviceToHost, s->stream));
  return bounded_sync(s);
}

ORT_CUDA_API int ort_cuda_slice_last_seq(ort_cuda_session* s, const float* X, int64_t outer,
                                         int64_t seq, int64_t inner, float* Y, int flags) {
  ORTC_CHECK(s && X && Y, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(outer >= 0 && seq >= 1 && inner >= 0, ORT_CUDA_ERR_INVALID_ARG,
             "slice_last_seq: need outer, inner >= 0 and seq >= 1");
  ORTC_CHECK((flags & ORT_CUDA_HOST_IO) == 0, ORT_CUDA_ERR_INVALID_ARG,
             "slice_last_seq takes device tensors (on the host it is the caller's copy)");
  if (outer == 0 || inner == 0) return ORT_CUDA_OK;
  DeviceGuard g(s->device);
  OpTimer timer(s, "SliceLastSeq");
  ORTC_CUDA(cudaMemcpy2DAsync(Y, (size_t)inner * 4, X + (seq - 1) * inner, (size_t)(seq * inner) * 4,
                              (size_t)inner * 4, (size_t)outer, cudaMemcpyDeviceToDevice,
                              s->stream));
  return ORT_CUDA_OK;
}

// ---- attention of a decoder step -------------------------------------------

}  // extern "C"

namespace {

// Copies for an ORT_CUDA_HOST_IO call: each host input gets a 256-aligned
// slot in the session workspace, each output a slot copied back afterwards.
struct HostStage {
  struct In {
    const void* src;
    size_t bytes, off;
  };
  struct Out {
    void* dst;
    size_t bytes, off;
  };
  std::vector<In> ins;
  std::vector<Out> outs;
  size_t total = 0;
  bool enabled;  // device-pointer calls stage nothing
  explicit HostStage(bool host) : enabled(host) {}
  size_t slot(size_t bytes) {
    const size_t off = total;
    total += (bytes + 255) & ~(size_t)255;
    return off;
  }
  size_t in(const void* src, size_t bytes) {
    if (!enabled) return 0;
    const size_t off = slot(bytes);
    if (src && bytes) ins.push_back({src, bytes, off});
    return off;
  }
  size_t out(void* dst, size_t bytes) {
    if (!enabled) return 0;
    const size_t off = slot(bytes);
    if (dst && bytes) outs.push_back({dst, bytes, off});
    return off;
  }
};

template <typename T>
T* ws_at(ort_cuda_session* s, size_t off, const void* host) {
  return host ? reinterpret_cast<T*>(static_cast<char*>(s->ws) + off) : nullptr;
}

int host_stage_in(ort_cuda_session* s, const HostStage& st) {
  int rc = ensure_ws(s, st.total + 256);
  if (rc) return rc;
  for (const auto& i : st.ins)
    ORTC_CUDA(cudaMemcpyAsync(static_cast<char*>(s->ws) + i.off, i.src, i.bytes,
                              cudaMemcpyHostToDevice, s->stream));
  return ORT_CUDA_OK;
}

int host_stage_out(ort_cuda_session* s, const HostStage& st) {
  for (const auto& o : st.outs)
    ORTC_CUDA(cudaMemcpyAsync(o.dst, static_cast<char*>(s->ws) + o.off, o.bytes,
                              cudaMemcpyDeviceToHost, s->stream));
  return bounded_sync(s);
}

// Split-key scratch for launch_attention; tickets zero when allocated.
int run_attention(ort_cuda_session* s, ortc::AttnArgs& a) {
  const size_t need = ortc::attention_scratch_bytes(a, s->sm_count);
  if (need > s->attn_bytes) {
    ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
               "a buffer would grow while a CUDA graph is being captured; run every "
               "operation of the graph once before capturing it");
    if (s->attnscratch) {
      ORTC_CUDA(cudaStreamSynchronize(s->stream));
      ORTC_CUDA(cudaFree(s->attnscratch));
      s->attnscratch = nullptr;
      s->attn_bytes = 0;
    }
    const size_t want = std::max<size_t>(need, 1 << 20);
    ORTC_CUDA(cudaMalloc(&s->attnscratch, want));
    ORTC_CUDA(cudaMemsetAsync(s->attnscratch, 0, want, s->stream));
    s->attn_bytes = want;
  }
  a.err = s->err_dev;
  return ortc::launch_attention(a, s->attnscratch, s->sm_count, s->stream, &s->launches);
}

}  // namespace

extern "C" {

ORT_CUDA_API int ort_cuda_group_query_attention(
    ort_cuda_session* s, const float* Q, const float* K, const float* V, const float* past_key,
    const float* past_value, int64_t batch, int64_t seq, int64_t past_len, int num_heads,
    int kv_num_heads, int64_t head_size, double scale, const float* cos_cache,
    const float* sin_cache, int64_t rotary_half, int64_t max_pos, const float* bias,
    int64_t bias_batch, int64_t bias_heads, int64_t kv_capacity, float* out, float* present_key,
    float* present_value, int flags) {
  ORTC_CHECK(s && Q && K && V && out, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(batch >= 0 && seq >= 0 && past_len >= 0 && num_heads >= 1 && kv_num_heads >= 1 &&
                 num_heads % kv_num_heads == 0 && head_size >= 1,
             ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: need num_heads a multiple of kv_num_heads, sizes >= 0");
  ORTC_CHECK(head_size <= 128, ORT_CUDA_ERR_UNSUPPORTED,
             "GroupQueryAttention: head sizes above 128 are not supported");
  ORTC_CHECK(past_len == 0 || (past_key && past_value), ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: past_len > 0 needs past_key and past_value");
  ORTC_CHECK((present_key == nullptr) == (present_value == nullptr), ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: give both present outputs or neither");
  const int64_t T = past_len + seq;
  ORTC_CHECK(kv_capacity == 0 || kv_capacity >= T, ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: kv_capacity below past_len + seq");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  ORTC_CHECK(!(host && kv_capacity), ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: kv_capacity needs device buffers");
  const bool rotary = (flags & ORT_CUDA_ROTARY) != 0;
  ORTC_CHECK(!rotary || (cos_cache && sin_cache && rotary_half >= 1 &&
                         2 * rotary_half <= head_size && max_pos >= T),
             ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: rotary needs cos/sin caches of max_pos >= past_len + seq "
             "rows of rotary_half <= head_size / 2 values");
  ORTC_CHECK(!bias || ((bias_batch == 1 || bias_batch == batch) && bias_heads >= 1),
             ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: attention bias must be [1 or batch, heads, seq, total]");
  const int64_t H = num_heads, Hkv = kv_num_heads, D = head_size;
  ORTC_CHECK(batch * seq * H <= INT_MAX && T <= INT_MAX && batch * Hkv <= INT_MAX,
             ORT_CUDA_ERR_INVALID_ARG, "GroupQueryAttention: sizes too large");
  if (batch == 0 || T == 0) return ORT_CUDA_OK;
  DeviceGuard guard(s->device);
  OpTimer timer(s, "GroupQueryAttention");
  const int64_t pcap = kv_capacity ? kv_capacity : past_len;
  const int64_t rcap = kv_capacity ? kv_capacity : T;

  HostStage st(host);
  const size_t o_q = st.in(Q, sizeof(float) * batch * seq * H * D);
  const size_t o_k = st.in(K, sizeof(float) * batch * seq * Hkv * D);
  const size_t o_v = st.in(V, sizeof(float) * batch * seq * Hkv * D);
  const size_t o_pk = st.in(past_len ? past_key : nullptr, sizeof(float) * batch * Hkv * pcap * D);
  const size_t o_pv = st.in(past_len ? past_value : nullptr, sizeof(float) * batch * Hkv * pcap * D);
  const size_t o_c = st.in(rotary ? cos_cache : nullptr, sizeof(float) * max_pos * rotary_half);
  const size_t o_s = st.in(rotary ? sin_cache : nullptr, sizeof(float) * max_pos * rotary_half);
  const size_t o_b = st.in(bias, sizeof(float) * bias_batch * bias_heads * seq * T);
  const size_t o_o = st.out(out, sizeof(float) * batch * seq * H * D);
  const size_t o_rk = st.out(present_key, sizeof(float) * batch * Hkv * rcap * D);
  const size_t o_rv = st.out(present_value, sizeof(float) * batch * Hkv * rcap * D);
  if (host) {
    int rc = host_stage_in(s, st);
    if (rc) return rc;
    Q = ws_at<const float>(s, o_q, Q);
    K = ws_at<const float>(s, o_k, K);
    V = ws_at<const float>(s, o_v, V);
    past_key = ws_at<const float>(s, o_pk, past_len ? past_key : nullptr);
    past_value = ws_at<const float>(s, o_pv, past_len ? past_value : nullptr);
    cos_cache = ws_at<const float>(s, o_c, rotary ? cos_cache : nullptr);
    sin_cache = ws_at<const float>(s, o_s, rotary ? sin_cache : nullptr);
    bias = ws_at<const float>(s, o_b, bias);
    out = ws_at<float>(s, o_o, out);
    present_key = ws_at<float>(s, o_rk, present_key);
    present_value = ws_at<float>(s, o_rv, present_value);
  }
  const bool alias = present_key && present_key == past_key;
  ORTC_CHECK(!alias || (present_value == past_value && pcap == rcap), ORT_CUDA_ERR_INVALID_ARG,
             "GroupQueryAttention: an in-place cache needs present = past for K and V and "
             "kv_capacity");
  if (seq == 0) {  // present = past
    if (present_key && !alias && past_len) {
      ORTC_CUDA(cudaMemcpy2DAsync(present_key, rcap * D * 4, past_key, pcap * D * 4,
                                  past_len * D * 4, batch * Hkv, cudaMemcpyDeviceToDevice,
                                  s->stream));
      ORTC_CUDA(cudaMemcpy2DAsync(present_value, rcap * D * 4, past_value, pcap * D * 4,
                                  past_len * D * 4, batch * Hkv, cudaMemcpyDeviceToDevice,
                                  s->stream));
    }
    return host ? host_stage_out(s, st) : ORT_CUDA_OK;
  }
  ortc::AttnArgs a;
  a.q = Q;
  a.qsb = seq * H * D, a.qsi = H * D, a.qsh = D;
  a.k = K;
  a.ksb = seq * Hkv * D, a.ksh = D, a.ksj = Hkv * D, a.ksd = 1;
  a.v = V;
  a.vsb = seq * Hkv * D, a.vsh = D, a.vsj = Hkv * D;
  a.pk = past_key, a.pv = past_value;
  a.psb = Hkv * pcap * D, a.psh = pcap * D;
  a.prk = present_key, a.prv = present_value;
  a.rsb = Hkv * rcap * D, a.rsh = rcap * D;
  a.write_past = alias ? 0 : 1;
  a.bias = bias;
  if (bias) {
    a.bsb = bias_batch == 1 ? 0 : bias_heads * seq * T;
    a.bsh = seq * T, a.bsi = T, a.bsj = 1, a.bh = (int)bias_heads;
  }
  a.out = out;
  a.osb = seq * H * D, a.osi = H * D, a.osh = D;
  a.batch = (int)batch, a.seq = (int)seq, a.heads_kv = (int)Hkv, a.group = (int)(H / Hkv);
  a.D = a.Dv = (int)D, a.past = (int)past_len, a.T = (int)T, a.causal = 1;
  a.scale = scale > 0 ? scale : 1.0 / std::sqrt((double)D);
  if (rotary) {
    a.rotary = 1, a.cos = cos_cache, a.sin = sin_cache, a.half_rot = (int)rotary_half;
    a.interleaved = (flags & ORT_CUDA_ROTARY_INTERLEAVED) ? 1 : 0;
  }
  int rc = run_attention(s, a);
  if (rc) return rc;
  return host ? host_stage_out(s, st) : ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_multi_head_attention(ort_cuda_session* s, const float* Q,
                                               const float* K, const float* V, int64_t batch,
                                               int64_t seq, int64_t kv_seq, int num_heads,
                                               int64_t hidden, double scale, const float* bias,
                                               int64_t bias_batch, int64_t bias_heads, float* out,
                                               int flags) {
  ORTC_CHECK(s && Q && K && V && out, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(batch >= 0 && seq >= 0 && kv_seq >= 0 && num_heads >= 1 && hidden >= 1 &&
                 hidden % num_heads == 0,
             ORT_CUDA_ERR_INVALID_ARG,
             "MultiHeadAttention: need hidden a multiple of num_heads, sizes >= 0");
  const int64_t H = num_heads, D = hidden / H;
  ORTC_CHECK(D <= 128, ORT_CUDA_ERR_UNSUPPORTED,
             "MultiHeadAttention: head sizes above 128 are not supported");
  ORTC_CHECK(!bias || ((bias_batch == 1 || bias_batch == batch) && bias_heads >= 1),
             ORT_CUDA_ERR_INVALID_ARG,
             "MultiHeadAttention: attention bias must be [1 or batch, heads, seq, kv_seq]");
  ORTC_CHECK(seq == 0 || kv_seq >= 1, ORT_CUDA_ERR_INVALID_ARG, "MultiHeadAttention: no keys");
  ORTC_CHECK(batch * seq * H <= INT_MAX && kv_seq <= INT_MAX && batch * H <= INT_MAX,
             ORT_CUDA_ERR_INVALID_ARG, "MultiHeadAttention: sizes too large");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  if (batch == 0 || seq == 0) return ORT_CUDA_OK;
  DeviceGuard guard(s->device);
  OpTimer timer(s, "MultiHeadAttention");
  HostStage st(host);
  const size_t o_q = st.in(Q, sizeof(float) * batch * seq * hidden);
  const size_t o_k = st.in(K, sizeof(float) * batch * kv_seq * hidden);
  const size_t o_v = st.in(V, sizeof(float) * batch * kv_seq * hidden);
  const size_t o_b = st.in(bias, sizeof(float) * bias_batch * bias_heads * seq * kv_seq);
  const size_t o_o = st.out(out, sizeof(float) * batch * seq * hidden);
  if (host) {
    int rc = host_stage_in(s, st);
    if (rc) return rc;
    Q = ws_at<const float>(s, o_q, Q);
    K = ws_at<const float>(s, o_k, K);
    V = ws_at<const float>(s, o_v, V);
    bias = ws_at<const float>(s, o_b, bias);
    out = ws_at<float>(s, o_o, out);
  }
  ortc::AttnArgs a;
  a.q = Q;
  a.qsb = seq * hidden, a.qsi = hidden, a.qsh = D;
  a.k = K;
  a.ksb = kv_seq * hidden, a.ksh = D, a.ksj = hidden, a.ksd = 1;
  a.v = V;
  a.vsb = kv_seq * hidden, a.vsh = D, a.vsj = hidden;
  a.bias = bias;
  if (bias) {
    a.bsb = bias_batch == 1 ? 0 : bias_heads * seq * kv_seq;
    a.bsh = seq * kv_seq, a.bsi = kv_seq, a.bsj = 1, a.bh = (int)bias_heads;
  }
  a.out = out;
  a.osb = seq * hidden, a.osi = hidden, a.osh = D;
  a.batch = (int)batch, a.seq = (int)seq, a.heads_kv = (int)H, a.group = 1;
  a.D = a.Dv = (int)D, a.past = 0, a.T = (int)kv_seq, a.causal = 0;
  a.scale = scale > 0 ? scale : 1.0 / std::sqrt((double)D);
  int rc = run_attention(s, a);
  if (rc) return rc;
  return host ? host_stage_out(s, st) : ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_fused_sdpa(ort_cuda_session* s, const float* A, const float* B,
                                     const float* V, const float* mask,
                                     const int64_t* mask_strides, int64_t n0, int64_t n1,
                                     int64_t seq, int64_t kv_seq, int64_t head_size,
                                     int64_t v_head_size, double scale, float* out, int flags) {
  ORTC_CHECK(s && A && B && V && out && (!mask || mask_strides), ORT_CUDA_ERR_INVALID_ARG,
             "NULL argument");
  ORTC_CHECK(n0 >= 0 && n1 >= 0 && seq >= 0 && kv_seq >= 0 && head_size >= 1 &&
                 v_head_size >= 1,
             ORT_CUDA_ERR_INVALID_ARG, "fused SDPA: sizes must be >= 0");
  ORTC_CHECK(head_size <= 128 && v_head_size <= 128, ORT_CUDA_ERR_UNSUPPORTED,
             "fused SDPA: head sizes above 128 are not supported");
  ORTC_CHECK(seq == 0 || kv_seq >= 1, ORT_CUDA_ERR_INVALID_ARG, "fused SDPA: no keys");
  int64_t mask_elems = 0;
  if (mask) {
    const int64_t dims[4] = {n0, n1, seq, kv_seq};
    mask_elems = 1;
    for (int i = 0; i < 4; i++) {
      ORTC_CHECK(mask_strides[i] >= 0, ORT_CUDA_ERR_INVALID_ARG,
                 "fused SDPA: mask strides must be >= 0 (0 broadcasts)");
      if (dims[i] > 0) mask_elems += (dims[i] - 1) * mask_strides[i];
    }
  }
  ORTC_CHECK(n0 * n1 <= INT_MAX && seq <= INT_MAX && kv_seq <= INT_MAX, ORT_CUDA_ERR_INVALID_ARG,
             "fused SDPA: sizes too large");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  if (n0 == 0 || n1 == 0 || seq == 0) return ORT_CUDA_OK;
  DeviceGuard guard(s->device);
  OpTimer timer(s, "FusedSDPA");
  const int64_t D = head_size, Dv = v_head_size;
  HostStage st(host);
  const size_t o_a = st.in(A, sizeof(float) * n0 * n1 * seq * D);
  const size_t o_b = st.in(B, sizeof(float) * n0 * n1 * D * kv_seq);
  const size_t o_v = st.in(V, sizeof(float) * n0 * n1 * kv_seq * Dv);
  const size_t o_m = st.in(mask, sizeof(float) * mask_elems);
  const size_t o_o = st.out(out, sizeof(float) * n0 * n1 * seq * Dv);
  if (host) {
    int rc = host_stage_in(s, st);
    if (rc) return rc;
    A = ws_at<const float>(s, o_a, A);
    B = ws_at<const float>(s, o_b, B);
    V = ws_at<const float>(s, o_v, V);
    mask = ws_at<const float>(s, o_m, mask);
    out = ws_at<float>(s, o_o, out);
  }
  ortc::AttnArgs a;  // (n0, n1) as (batch, head); B is K transposed: [D][kv_seq]
  a.q = A;
  a.qsb = n1 * seq * D, a.qsh = seq * D, a.qsi = D;
  a.k = B;
  a.ksb = n1 * D * kv_seq, a.ksh = D * kv_seq, a.ksj = 1, a.ksd = kv_seq;
  a.v = V;
  a.vsb = n1 * kv_seq * Dv, a.vsh = kv_seq * Dv, a.vsj = Dv;
  a.bias = mask;
  if (mask) {
    a.bsb = mask_strides[0], a.bsh = mask_strides[1], a.bsi = mask_strides[2];
    a.bsj = mask_strides[3], a.bh = (int)n1;
  }
  a.out = out;
  a.osb = n1 * seq * Dv, a.osh = seq * Dv, a.osi = Dv;
  a.batch = (int)n0, a.seq = (int)seq, a.heads_kv = (int)n1, a.group = 1;
  a.D = (int)D, a.Dv = (int)Dv, a.past = 0, a.T = (int)kv_seq, a.causal = 0;
  a.scale = scale;
  int rc = run_attention(s, a);
  if (rc) return rc;
  return host ? host_stage_out(s, st) : ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_rotary_embedding(ort_cuda_session* s, const float* X,
                                           const int64_t* position_ids, int pos_per_batch,
                                           const float* cos_cache, const float* sin_cache,
                                           int64_t max_pos, int64_t rotary_half, int64_t batch,
                                           int64_t seq, int64_t heads, int64_t head_size,
                                           int64_t rotary_dim, float* Y, int flags) {
  ORTC_CHECK(s && X && position_ids && cos_cache && sin_cache && Y, ORT_CUDA_ERR_INVALID_ARG,
             "NULL argument");
  const int64_t rdim = rotary_dim > 0 ? rotary_dim : 2 * rotary_half;
  ORTC_CHECK(batch >= 0 && seq >= 0 && heads >= 0 && head_size >= 1 && rotary_half >= 1 &&
                 max_pos >= 1 && rdim % 2 == 0 && rdim <= head_size && rdim / 2 <= rotary_half,
             ORT_CUDA_ERR_INVALID_ARG,
             "RotaryEmbedding: need an even rotary_dim <= head_size with rotary_dim / 2 <= the "
             "cache row length");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls cannot be recorded into a CUDA graph");
  const int64_t n = batch * seq * heads * head_size;
  if (n == 0) return ORT_CUDA_OK;
  DeviceGuard guard(s->device);
  OpTimer timer(s, "RotaryEmbedding");
  HostStage st(host);
  const size_t o_x = st.in(X, sizeof(float) * n);
  const size_t o_p = st.in(position_ids, sizeof(int64_t) * (pos_per_batch ? batch : 1) * seq);
  const size_t o_c = st.in(cos_cache, sizeof(float) * max_pos * rotary_half);
  const size_t o_s = st.in(sin_cache, sizeof(float) * max_pos * rotary_half);
  const size_t o_y = st.out(Y, sizeof(float) * n);
  if (host) {
    int rc = host_stage_in(s, st);
    if (rc) return rc;
    X = ws_at<const float>(s, o_x, X);
    position_ids = ws_at<const int64_t>(s, o_p, position_ids);
    cos_cache = ws_at<const float>(s, o_c, cos_cache);
    sin_cache = ws_at<const float>(s, o_s, sin_cache);
    Y = ws_at<float>(s, o_y, Y);
  }
  int rc = ortc::launch_rotary(X, Y, position_ids, pos_per_batch ? 1 : 0, cos_cache, sin_cache,
                               max_pos, (int)rotary_half, (int)rdim, batch, seq, heads, head_size,
                               (flags & ORT_CUDA_ROTARY_BHSD) ? 1 : 0,
                               (flags & ORT_CUDA_ROTARY_INTERLEAVED) ? 1 : 0, s->stream,
                               &s->launches);
  if (rc) return rc;
  return host ? host_stage_out(s, st) : ORT_CUDA_OK;
}

// ---- the hot ops --------------------------------------------------------------

}  // extern "C"

namespace {

size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// N-sharded MatMulNBits in a tensor-core mode whose output is too large for
// the peer exchange buffers (prefill).  With the fp16 fused GEMM and mapped
// peers the GEMM pushes its output to the peers itself (below).  Otherwise
// the rows are cut into chunks, and while the session stream runs the GEMM
// of chunk c + 1, the exchange stream all-gathers chunk c (NCCL) and
// re-lays it into Y, so the NVLink transfer overlaps the tensor-core work.
// yloc is [M, Ns], gath [G, M, Ns] (chunk c's gather lands at rows r0.. of
// every rank's part, contiguous per chunk), Y [M, N].
int nbits_prefill_chunked(ort_cuda_session* s, Weight& w, const float* A, int64_t M,
                          float* yloc, float* gath, float* Y, int mode) {
  const int64_t N = w.N, ns = w.ns, G = s->world;
  // Chunks of whole 128-row tile rows, each at least two waves of the GEMM's
  // 128 x 256 tiles on this GPU (a chunk of fewer tiles leaves SMs idle and
  // costs more than its overlap saves); at most 8 chunks.
  const int64_t col_tiles = (ns + 255) / 256;
  int64_t rows_for_waves = (2 * s->sm_count + col_tiles - 1) / col_tiles * 128;
  int64_t mc = std::max<int64_t>(rows_for_waves, ((M + 7) / 8 + 127) / 128 * 128);
  if (mc > M) mc = M;
  const int64_t nch = (M + mc - 1) / mc;
  ORTC_CHECK(nch <= 16, ORT_CUDA_ERR_INVALID_ARG, "too many prefill chunks");
  if (!s->comm_stream)
    ORTC_CUDA(cudaStreamCreateWithFlags(&s->comm_stream, cudaStreamNonBlocking));
  for (int i = 0; i <= 16; i++)
    if (!s->chunk_ev[i])
      ORTC_CUDA(cudaEventCreateWithFlags(&s->chunk_ev[i], cudaEventDisableTiming));
  // Push mode (fp16 fused GEMM, peers mapped): the whole GEMM at once, its
  // epilogue storing each row slice into every peer's big buffer as well as
  // into this rank's columns of Y; a landing kernel then copies the peers'
  // blocks into Y (local memory only).  Every rank decides alike: the
  // conditions depend on shapes and on the mapping all ranks agreed on.
  if (mode == ORT_CUDA_MODE_MMA_F16 && nbits_gemm_f16_layout_ok(w)) {
    bool big = false;
    int rc = p2p_big_ensure(s, (size_t)(G * M * ns), &big);
    if (rc) return rc;
    if (big) {
      const unsigned long long e = ++s->bepoch;
      PrefillPush push;
      rc = p2p_push_prepare(s, e, M, ns, &push);
      if (rc) return rc;
      rc = w.nl > 0 ? launch_mma_nbits(s, w, A, M, Y + w.n0, N, mode, s->stream, 0, &push)
                    : p2p_push_post(s, push);
      if (rc) return rc;
      return p2p_push_land(s, e, M, ns, N, Y);
    }
  }
  // the exchange stream starts after everything queued before this call
  ORTC_CUDA(cudaEventRecord(s->chunk_ev[16], s->stream));
  ORTC_CUDA(cudaStreamWaitEvent(s->comm_stream, s->chunk_ev[16], 0));
  for (int64_t c = 0; c < nch; c++) {
    const int64_t r0 = c * mc, m = std::min(mc, M - r0);
    int rc = launch_mma_nbits(s, w, A + r0 * w.K, m, yloc + r0 * ns, ns, mode, s->stream);
    if (rc) return rc;
    ORTC_CUDA(cudaEventRecord(s->chunk_ev[c], s->stream));
    ORTC_CUDA(cudaStreamWaitEvent(s->comm_stream, s->chunk_ev[c], 0));
    float* g = gath + r0 * ns * G;
    ncclResult_t r = nccl()->AllGather(yloc + r0 * ns, g, (size_t)(m * ns), ncclFloat,
                                       (ncclComm_t)s->nccl, s->comm_stream);
    if (r != ncclSuccess && r != ncclInProgress)
      return fail(ORT_CUDA_ERR_NCCL, std::string("ncclAllGather: ") + nccl()->GetErrorString(r));
    if (r == ncclInProgress) {
      rc = nccl_wait_ready((ncclComm_t)s->nccl, s->timeout_ms);
      if (rc) {
        nccl()->CommAbort((ncclComm_t)s->nccl);
        s->nccl = nullptr;
        return rc;
      }
    }
    rc = launch_unshard(g, Y + r0 * N, G, m, ns, N, s->comm_stream, &s->launches);
    if (rc) return rc;
  }
  // the session stream continues once every chunk has landed in Y
  ORTC_CUDA(cudaEventRecord(s->chunk_ev[16], s->comm_stream));
  ORTC_CUDA(cudaStreamWaitEvent(s->stream, s->chunk_ev[16], 0));
  return ORT_CUDA_OK;
}

// Workspace layout for one op call (byte offsets into s->ws, 256-aligned).
struct WsLayout {
  size_t a = 0, c = 0, yloc = 0, gath = 0, y = 0, total = 0;
};

// Runs one matmul-family op: stages host IO, computes this rank's columns,
// all-gathers across ranks, writes back.  `compute` gets device A, C, the
// local output pointer and its leading dimension.  y_direct: every kernel of
// `compute` writes Y with plain stores only, so with host buffers on an
// unsharded op the kernels store straight into the pinned host Y (its
// device mapping) and no device-to-host copy follows.
template <typename F>
int run_op(ort_cuda_session* s, const Weight& w, const void* A, size_t a_bytes, const void* C,
           size_t c_bytes, float* Y, int64_t M, int flags, F&& compute, bool y_direct = false) {
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls synchronise and cannot be captured in a CUDA graph");
  const int64_t N = w.N;
  const bool sharded = s->world > 1 && !w.replicated;
  WsLayout L;
  size_t off = 0;
  if (host) {
    L.a = off;
    off += al256(a_bytes);
    L.c = off;
    off += al256(c_bytes);
    L.y = off;
    off += al256((size_t)(M * N) * 4);
  }
  if (sharded) {
    L.yloc = off;
    off += al256((size_t)(M * w.ns) * 4);
    L.gath = off;
    off += al256((size_t)(M * w.ns * s->world) * 4);
  }
  L.total = off;
  int rc = ensure_ws(s, L.total);
  if (rc) return rc;
  char* ws = (char*)s->ws;
  const float* dA = static_cast<const float*>(A);
  const float* dC = static_cast<const float*>(C);
  float* dY = Y;
  bool y_pinned = false, y_mapped = false;
  if (host) {
    size_t pin_need = a_bytes + c_bytes + (size_t)(M * N) * 4 + 768;
    rc = ensure_pinned(s, pin_need);
    if (rc) return rc;
    rc = stage_in(s, ws + L.a, A, a_bytes, 0);
    if (rc) return rc;
    dA = (const float*)(ws + L.a);
    if (C && c_bytes) {
      rc = stage_in(s, ws + L.c, C, c_bytes, al256(a_bytes));
      if (rc) return rc;
      dC = (const float*)(ws + L.c);
    }
    dY = (float*)(ws + L.y);
    y_pinned = is_pinned_host(Y);
    if (y_direct && !sharded) {
      // the caller's pinned Y, or the session's pinned staging of Y
      float* hy = y_pinned ? Y : (float*)((char*)s->pinned + al256(al256(a_bytes) + c_bytes + 256));
      void* dp = nullptr;
      if (cudaHostGetDevicePointer(&dp, hy, 0) == cudaSuccess) {
        dY = static_cast<float*>(dp);
        y_mapped = true;
      } else {
        cudaGetLastError();
      }
    }
  }
  float* yloc = sharded ? (float*)(ws + L.yloc) : dY;
  const int64_t ldy = sharded ? w.ns : N;
  // peer loads when the slices fit the exchange buffers (a producer that can
  // writes its slice there itself), else NCCL
  const bool p2p = sharded && p2p_fits(s, M * w.ns);
  s->xsel_offer = p2p;
  s->xsel_taken = false;
  // a producer that can push its outputs to the peers (decode GEMV) writes
  // straight into the gathered Y and p2p_land completes the exchange
  s->push_y = (sharded && p2p_push_fits(s, M, N)) ? dY : nullptr;
  s->push_taken = false;
  const bool nccl_path = sharded && !p2p;
  s->chunk_y = nccl_path ? dY : nullptr;
  s->chunk_gath = nccl_path ? (float*)(ws + L.gath) : nullptr;
  s->gathered = false;
  rc = compute(dA, dC, yloc, ldy);
  const bool pushed = s->push_taken, gathered = s->gathered;
  s->xsel_offer = false;
  s->push_y = nullptr;
  s->push_taken = false;
  s->chunk_y = s->chunk_gath = nullptr;
  s->gathered = false;
  if (rc) return rc;
  if (sharded && !gathered) {
    if (pushed)
      rc = p2p_land(s, M, N, w.n0, w.nl, dY);
    else
      rc = p2p ? p2p_gather(s, s->xsel_taken ? nullptr : yloc, M, w.ns, N, dY)
               : gather_y(s, yloc, (float*)(ws + L.gath), dY, M, w.ns, N);
    if (rc) return rc;
  }
  if (host) {
    const size_t yb = (size_t)(M * N) * 4;
    if (y_mapped) {  // the kernels wrote the host Y (or its staging) already
      rc = bounded_sync(s);
      if (rc) return rc;
      if (!y_pinned)
        std::memcpy(Y, (char*)s->pinned + al256(al256(a_bytes) + c_bytes + 256), yb);
      return ORT_CUDA_OK;
    }
    if (y_pinned) {
      ORTC_CUDA(cudaMemcpyAsync(Y, dY, yb, cudaMemcpyDeviceToHost, s->stream));
      return bounded_sync(s);
    }
    const size_t pin_y = al256(al256(a_bytes) + c_bytes + 256);
    ORTC_CUDA(cudaMemcpyAsync((char*)s->pinned + pin_y, dY, yb, cudaMemcpyDeviceToHost,
                              s->stream));
    rc = bounded_sync(s);
    if (rc) return rc;
    std::memcpy(Y, (char*)s->pinned + pin_y, yb);
  }
  return ORT_CUDA_OK;
}

// Tensor-core GEMV over m <= 8 rows: timed plan choice on the first eager
// call for (w, m), then the launch.
int gemv_call(ort_cuda_session* s, Weight& w, const float* a, int64_t m, float* y, int64_t ly,
              const YSel* ysp) {
  if (w.nl == 0) return ORT_CUDA_OK;  // a rank without columns
  int rc;
  if (w.gemv_plan[m] < 0 && !s->capturing && gemv_tuning_enabled()) {
    rc = ensure_kscratch(s, tc_gemv_partial_floats(w, m, s->sm_count, -1) * 4);
    if (rc) return rc;
    rc = tune_tc_gemv(w, a, m, y, ly, (float*)s->kscratch, s->err_dev, s->sm_count, s->stream,
                      ysp);
    if (rc) return rc;
  }
  const int plan = tc_gemv_plan(w, m, s->sm_count);
  rc = ensure_kscratch(s, tc_gemv_partial_floats(w, m, s->sm_count, plan) * 4);
  if (rc) return rc;
  return launch_tc_gemv(w, plan, a, m, y, ly, (float*)s->kscratch, s->err_dev, s->sm_count,
                        s->stream, &s->launches, ysp);
}

}  // namespace

extern "C" {

ORT_CUDA_API int ort_cuda_matmul_nbits(ort_cuda_session* s, const char* name, const float* A,
                                       int64_t M, float* Y, int flags) {
  ORTC_CHECK(s && name, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 0, ORT_CUDA_ERR_INVALID_ARG, "M must be >= 0");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  Weight& w = it->second;
  ORTC_CHECK(w.kind == W_NBITS, ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + name + "' is not a MatMulNBits weight");
  if (M == 0) return ORT_CUDA_OK;
  ORTC_CHECK(A && Y, ORT_CUDA_ERR_INVALID_ARG, "NULL A or Y");
  const int mode = mode_of(s, flags);
  ORTC_CHECK(valid_mode(mode), ORT_CUDA_ERR_INVALID_ARG, "unknown mode");
  DeviceGuard g(s->device);
  OpTimer timer(s, "MatMulNBits");
  return run_op(s, w, A, (size_t)(M * w.K) * 4, nullptr, 0, Y, M, flags,
                [&](const float* dA, const float*, float* yl, int64_t ldy) -> int {
                  if (mode == ORT_CUDA_MODE_STRICT)
                    return launch_simt_gemm(w, dA, M, false, yl, ldy, true, 1.0f, 1.0f, nullptr,
                                            0, 0, 0, s->stream, &s->launches);
                  auto gemv_rows = [&](const float* a, int64_t m, float* y, int64_t ly,
                                       const YSel* ysp) -> int {
                    return gemv_call(s, w, a, m, y, ly, ysp);
                  };
                  // every rank takes the same path (the exchange that follows
                  // depends on it), also a rank that holds no columns
                  auto gemv_ok = [&](int64_t m) {
                    return w.nl == 0 ? tc_gemv_shape_ok(w, m) : tc_gemv_ok(w, m);
                  };
                  if (gemv_ok(M)) {
                    if (s->push_y) {  // N-sharded: outputs pushed to the peers
                      YSel ys = p2p_ysel_push(s, w.n0, w.N, 0);
                      s->push_taken = true;
                      return gemv_rows(dA, M, s->push_y + w.n0, w.N, &ys);
                    }
                    YSel ys;
                    if (s->xsel_offer) {
                      ys = p2p_ysel(s);
                      s->xsel_taken = true;
                    }
                    return gemv_rows(dA, M, yl, ldy, s->xsel_offer ? &ys : nullptr);
                  }
                  // Up to 8 passes of the GEMV over row chunks (each streams the
                  // weight again) still beat the CUDA-core GEMM at decode-sized
                  // M, and every row keeps the exact arithmetic.
                  int cmax = 0;
                  for (int m = 8; m >= 1 && !cmax; m--)
                    if (gemv_ok(m)) cmax = m;
                  if (cmax > 0 && M > cmax && M <= 8 * cmax) {
                    const bool push = s->push_y != nullptr;
                    for (int64_t r = 0; r < M; r += cmax) {
                      const int64_t m = std::min<int64_t>(cmax, M - r);
                      int rc;
                      if (push) {
                        YSel ys = p2p_ysel_push(s, w.n0, w.N, (int)r);
                        s->push_taken = true;
                        rc = gemv_rows(dA + r * w.K, m, s->push_y + r * w.N + w.n0, w.N, &ys);
                      } else {
                        rc = gemv_rows(dA + r * w.K, m, yl + r * ldy, ldy, nullptr);
                      }
                      if (rc) return rc;
                    }
                    return ORT_CUDA_OK;
                  }
                  if ((mode == ORT_CUDA_MODE_MMA_F16 || mode == ORT_CUDA_MODE_MMA_BF16) &&
                      mma_supported_shape(M, w.K)) {
                    // the same decision on every rank: it depends on shapes only
                    if (s->chunk_gath && M >= 256 && !s->capturing && s->nccl) {
                      s->gathered = true;
                      return nbits_prefill_chunked(s, w, dA, M, yl, s->chunk_gath, s->chunk_y,
                                                   mode);
                    }
                    return launch_mma_nbits(s, w, dA, M, yl, ldy, mode, s->stream);
                  }
                  return launch_simt_gemm(w, dA, M, false, yl, ldy, false, 1.0f, 1.0f, nullptr, 0,
                                          0, 0, s->stream, &s->launches);
                },
                // decode sizes in the exact and strict modes: the GEMV and the
                // CUDA-core GEMM, plain stores of Y
                (mode == ORT_CUDA_MODE_EXACT || mode == ORT_CUDA_MODE_STRICT) && M <= 64);
}

}  // extern "C"

namespace {

int ensure_aux(ort_cuda_session* s, size_t bytes) {
  if (bytes <= s->aux_bytes) return ORT_CUDA_OK;
  ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
             "a buffer would grow while a CUDA graph is being captured; run every "
             "operation of the graph once before capturing it");
  const size_t want = bytes + bytes / 4 + (1 << 20);
  if (s->aux) {
    ORTC_CUDA(cudaStreamSynchronize(s->stream));
    ORTC_CUDA(cudaFree(s->aux));
    s->aux = nullptr;
    s->aux_bytes = 0;
  }
  ORTC_CUDA(cudaMalloc(&s->aux, want));
  s->aux_bytes = want;
  return ORT_CUDA_OK;
}

constexpr int64_t kAmaxRows = 64;  // rows of the fused path's keys (8 GEMV passes of 8)

// MatMulNBits then ArgMax/ArgMin over each row of Y, device pointers.
int nbits_argmax_dev(ort_cuda_session* s, Weight& w, const char* name, const float* dA,
                     int64_t M, int64_t* dI, float* dY, int flags) {
  const int mode = mode_of(s, flags);
  const int arg_flags = flags & (ORT_CUDA_ARG_MIN | ORT_CUDA_ARG_SELECT_LAST);
  int cmax = 0;
  for (int m = 8; m >= 1 && !cmax; m--)
    if (tc_gemv_ok(w, m)) cmax = m;
  const bool fused = (s->world == 1 || w.replicated) && mode != ORT_CUDA_MODE_STRICT && cmax > 0 &&
                     M <= 8 * cmax && M <= kAmaxRows && w.N < (int64_t)UINT32_MAX;
  if (!fused) {
    // the same result from the two separate operations
    const int mflags = flags & (ORT_CUDA_MODE_OVERRIDE | 0xF000);
    int rc = ort_cuda_matmul_nbits(s, name, dA, M, dY, mflags);
    if (rc) return rc;
    return ort_cuda_argmax(s, dY, M, w.N, w.N, dI, arg_flags);
  }
  if (!s->amaxbuf) {
    ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
               "the first fused MatMulNBits + ArgMax call of a session sets it up; make one "
               "before capturing a CUDA graph");
    const size_t bytes = (size_t)kAmaxRows * 12 + 256;
    ORTC_CUDA(cudaMalloc(&s->amaxbuf, bytes));
    ORTC_CUDA(cudaMemsetAsync(s->amaxbuf, 0, bytes, s->stream));
  }
  for (int64_t r = 0; r < M; r += cmax) {
    const int64_t m = std::min<int64_t>(cmax, M - r);
    YSel ys;
    ys.amax = static_cast<unsigned long long*>(s->amaxbuf);
    ys.amax_out = dI;
    ys.amax_rows = (int)M;
    ys.amax_min = (arg_flags & ORT_CUDA_ARG_MIN) ? 1 : 0;
    ys.amax_last = (arg_flags & ORT_CUDA_ARG_SELECT_LAST) ? 1 : 0;
    ys.row0 = (int)r;
    int rc = gemv_call(s, w, dA + r * w.K, m, dY + r * w.N, w.N, &ys);
    if (rc) return rc;
  }
  return ORT_CUDA_OK;
}

}  // namespace

extern "C" {

ORT_CUDA_API int ort_cuda_matmul_nbits_argmax(ort_cuda_session* s, const char* name,
                                              const float* A, int64_t M, int64_t* indices,
                                              float* Y, int flags) {
  ORTC_CHECK(s && name && A && indices, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 0, ORT_CUDA_ERR_INVALID_ARG, "M must be >= 0");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  Weight& w = it->second;
  ORTC_CHECK(w.kind == W_NBITS, ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + name + "' is not a MatMulNBits weight");
  if (M == 0) return ORT_CUDA_OK;
  ORTC_CHECK(valid_mode(mode_of(s, flags)), ORT_CUDA_ERR_INVALID_ARG, "unknown mode");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls synchronise and cannot be captured in a CUDA graph");
  DeviceGuard g(s->device);
  OpTimer timer(s, "MatMulNBits+ArgMax");
  // device views: A and the indices staged when host, Y in session scratch
  // when the caller wants no logits (or has them on the host)
  const size_t ab = (size_t)(M * w.K) * 4, yb = (size_t)(M * w.N) * 4, ib = (size_t)M * 8;
  size_t off = 0;
  const size_t a_off = off;
  if (host) off += al256(ab);
  const size_t y_off = off;
  if (host || !Y) off += al256(yb);
  const size_t i_off = off;
  if (host) off += al256(ib);
  int rc = off ? ensure_aux(s, off) : ORT_CUDA_OK;
  if (rc) return rc;
  char* aux = static_cast<char*>(s->aux);
  const float* dA = A;
  if (host) {
    ORTC_CUDA(cudaMemcpyAsync(aux + a_off, A, ab, cudaMemcpyHostToDevice, s->stream));
    dA = reinterpret_cast<const float*>(aux + a_off);
  }
  float* dY = (host || !Y) ? reinterpret_cast<float*>(aux + y_off) : Y;
  int64_t* dI = host ? reinterpret_cast<int64_t*>(aux + i_off) : indices;
  rc = nbits_argmax_dev(s, w, name, dA, M, dI, dY, flags & ~ORT_CUDA_HOST_IO);
  if (rc || !host) return rc;
  ORTC_CUDA(cudaMemcpyAsync(indices, dI, ib, cudaMemcpyDeviceToHost, s->stream));
  if (Y) ORTC_CUDA(cudaMemcpyAsync(Y, dY, yb, cudaMemcpyDeviceToHost, s->stream));
  return bounded_sync(s);
}

}  // extern "C"

ORT_CUDA_API int ort_cuda_fuse_nbits(ort_cuda_session* s, const char* fused,
                                     const char* const* names, int n, int flags) {
  ORTC_CHECK(s && fused && names, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(n >= 2 && n <= kMaxSegs, ORT_CUDA_ERR_INVALID_ARG,
             "a fused group holds 2 .. " + std::to_string(kMaxSegs) + " weights");
  std::vector<Weight*> parts;
  for (int i = 0; i < n; i++) {
    ORTC_CHECK(names[i] && std::strcmp(names[i], fused) != 0, ORT_CUDA_ERR_INVALID_ARG,
               "the fused name must differ from its parts");
    auto it = s->weights.find(names[i]);
    ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
               std::string("no weight named '") + names[i] + "'");
    ORTC_CHECK(it->second.kind == W_NBITS && it->second.nparts == 0, ORT_CUDA_ERR_INVALID_ARG,
               std::string("weight '") + names[i] + "' is not a plain MatMulNBits weight");
    parts.push_back(&it->second);
  }
  const Weight& p0 = *parts[0];
  for (Weight* p : parts)
    ORTC_CHECK(p->K == p0.K && p->bs == p0.bs && p->has_zp == p0.has_zp &&
                   (p->scales16 != nullptr) == (p0.scales16 != nullptr),
               ORT_CUDA_ERR_INVALID_ARG,
               "fused weights need the same K, block size, zero points and scale type");
  DeviceGuard g(s->device);
  Weight w;
  w.kind = W_NBITS;
  w.K = p0.K;
  w.bs = p0.bs;
  w.nb = p0.nb;
  w.has_zp = p0.has_zp;
  w.nparts = n;
  int64_t N = 0;
  for (int i = 0; i < n; i++) {
    w.part_name[i] = names[i];
    w.part_col[i] = N;
    N += parts[i]->N;
  }
  w.part_col[n] = N;
  w.N = N;
  bool all_replicated = true;
  for (Weight* p : parts) all_replicated = all_replicated && p->replicated;
  w.replicated = s->world > 1 && all_replicated;
  if (s->world > 1 && !all_replicated) {
    // sharded: each part keeps its own shards and exchange; the group call
    // runs them in turn
    w.kind = W_GROUP;
    w.group_only = true;
    auto it = s->weights.find(fused);
    if (it != s->weights.end()) {
      free_weight(it->second);
      s->weights.erase(it);
    }
    s->weights.emplace(fused, w);
    return ORT_CUDA_OK;
  }
  w.n0 = 0;
  w.nl = w.ns = N;
  const int64_t col_bytes = (int64_t)w.nb * w.bs / 2, nb = w.nb, zrows = (nb + 1) / 2;
  w.s_pitch = (N + 3) / 4 * 4;
  auto cleanup = [&](int rc) {
    free_weight(w);
    return rc;
  };
  cudaError_t e = cudaMalloc(&w.B, (size_t)(N * col_bytes));
  if (e == cudaSuccess) e = cudaMalloc(&w.scales, (size_t)(nb * w.s_pitch * 4));
  if (e == cudaSuccess) e = cudaMemsetAsync(w.scales, 0, (size_t)(nb * w.s_pitch * 4), s->stream);
  if (e == cudaSuccess && p0.scales16) {
    w.s16_pitch = (N + 7) / 8 * 8;
    e = cudaMalloc(&w.scales16, (size_t)(nb * w.s16_pitch * 2));
    if (e == cudaSuccess)
      e = cudaMemsetAsync(w.scales16, 0, (size_t)(nb * w.s16_pitch * 2), s->stream);
  }
  if (e == cudaSuccess && w.has_zp) {
    w.z_pitch = (N + 15) / 16 * 16;
    e = cudaMalloc(&w.zp, (size_t)(zrows * w.z_pitch));
    if (e == cudaSuccess) e = cudaMemsetAsync(w.zp, 0, (size_t)(zrows * w.z_pitch), s->stream);
  }
  for (int i = 0; i < n && e == cudaSuccess; i++) {
    const Weight& p = *parts[i];
    const int64_t c0 = w.part_col[i];
    e = cudaMemcpyAsync(w.B + c0 * col_bytes, p.B, (size_t)(p.nl * col_bytes),
                        cudaMemcpyDeviceToDevice, s->stream);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(w.scales + c0, (size_t)(w.s_pitch * 4), p.scales,
                            (size_t)(p.s_pitch * 4), (size_t)(p.nl * 4), (size_t)nb,
                            cudaMemcpyDeviceToDevice, s->stream);
    if (e == cudaSuccess && w.scales16)
      e = cudaMemcpy2DAsync(w.scales16 + c0, (size_t)(w.s16_pitch * 2), p.scales16,
                            (size_t)(p.s16_pitch * 2), (size_t)(p.nl * 2), (size_t)nb,
                            cudaMemcpyDeviceToDevice, s->stream);
    if (e == cudaSuccess && w.zp)
      e = cudaMemcpy2DAsync(w.zp + c0, (size_t)w.z_pitch, p.zp, (size_t)p.z_pitch, (size_t)p.nl,
                            (size_t)zrows, cudaMemcpyDeviceToDevice, s->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  if (e != cudaSuccess) return cleanup(cuda_fail(e, "fuse MatMulNBits weights"));
  int rc = prepare_nbits_tc(w);
  if (rc) return cleanup(rc);
  if (flags & ORT_CUDA_FUSE_DROP_PARTS)
    for (int i = 0; i < n; i++) {
      auto it = s->weights.find(names[i]);
      free_weight(it->second);
      s->weights.erase(it);
    }
  auto it = s->weights.find(fused);
  if (it != s->weights.end()) {
    free_weight(it->second);
    s->weights.erase(it);
  }
  s->weights.emplace(fused, w);
  return ORT_CUDA_OK;
}

ORT_CUDA_API int ort_cuda_matmul_nbits_group(ort_cuda_session* s, const char* fused,
                                             const float* A, int64_t M, float* const* Ys,
                                             int flags) {
  ORTC_CHECK(s && fused && A && Ys, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 0, ORT_CUDA_ERR_INVALID_ARG, "M must be >= 0");
  auto it = s->weights.find(fused);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + fused + "'");
  Weight& w = it->second;
  ORTC_CHECK(w.nparts >= 2, ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + fused + "' is not a fused group");
  for (int i = 0; i < w.nparts; i++)
    ORTC_CHECK(Ys[i], ORT_CUDA_ERR_INVALID_ARG, "NULL output of part " + std::to_string(i));
  if (M == 0) return ORT_CUDA_OK;
  if (w.group_only) {  // N-sharded session: the parts in turn, each exchanged
    for (int i = 0; i < w.nparts; i++) {
      const int rc = ort_cuda_matmul_nbits(s, w.part_name[i].c_str(), A, M, Ys[i], flags);
      if (rc) return rc;
    }
    return ORT_CUDA_OK;
  }
  const int mode = mode_of(s, flags);
  ORTC_CHECK(valid_mode(mode), ORT_CUDA_ERR_INVALID_ARG, "unknown mode");
  const bool host = (flags & ORT_CUDA_HOST_IO) != 0;
  ORTC_CHECK(!(host && s->capturing), ORT_CUDA_ERR_INVALID_ARG,
             "ORT_CUDA_HOST_IO calls synchronise and cannot be captured in a CUDA graph");
  DeviceGuard g(s->device);
  OpTimer timer(s, "MatMulNBits");
  int cmax = 0;
  for (int m = 8; m >= 1 && !cmax; m--)
    if (tc_gemv_ok(w, m)) cmax = m;
  const bool gemv = mode != ORT_CUDA_MODE_STRICT && cmax > 0 && M <= 8 * cmax;
  // prefill-sized: the fused fp16 GEMM writes each part's columns into its
  // own buffer when the part boundaries are multiples of 32
  bool seg_ok = !gemv && !host && mode == ORT_CUDA_MODE_MMA_F16 && nbits_gemm_f16_ok(w) &&
                mma_supported_shape(M, w.K);
  for (int i = 1; i < w.nparts; i++) seg_ok = seg_ok && w.part_col[i] % 32 == 0;
  // device views: staged A / outputs for host buffers, one [M, N] scratch
  // when the op runs whole and is split afterwards
  const size_t ab = (size_t)(M * w.K) * 4, yb = (size_t)(M * w.N) * 4;
  size_t off = 0;
  const size_t a_off = off;
  if (host) off += al256(ab);
  const size_t y_off = off;
  if (host || (!gemv && !seg_ok)) off += al256(yb);
  int rc = off ? ensure_aux(s, off) : ORT_CUDA_OK;
  if (rc) return rc;
  char* aux = static_cast<char*>(s->aux);
  const float* dA = A;
  if (host) {
    ORTC_CUDA(cudaMemcpyAsync(aux + a_off, A, ab, cudaMemcpyHostToDevice, s->stream));
    dA = reinterpret_cast<const float*>(aux + a_off);
  }
  float* scratch = reinterpret_cast<float*>(aux + y_off);
  // part i of the output: in the caller's buffer, or (host) at column
  // part_col[i] of rows of pitch N in scratch
  auto part_y = [&](int i) -> float* { return host ? nullptr : Ys[i]; };
  if (gemv) {
    for (int64_t r = 0; r < M; r += cmax) {
      const int64_t m = std::min<int64_t>(cmax, M - r);
      YSel ys;
      ys.nseg = w.nparts;
      for (int i = 0; i < w.nparts; i++) {
        const int64_t ni = w.part_col[i + 1] - w.part_col[i];
        ys.seg_start[i] = w.part_col[i];
        ys.seg_y[i] = host ? scratch + r * w.N + w.part_col[i] : part_y(i) + r * ni;
        ys.seg_ld[i] = host ? w.N : ni;
      }
      ys.seg_start[w.nparts] = w.N;
      rc = gemv_call(s, w, dA + r * w.K, m, scratch, w.N, &ys);
      if (rc) return rc;
    }
  } else {
    if (seg_ok) {
      YSel ys;
      ys.nseg = w.nparts;
      for (int i = 0; i < w.nparts; i++) {
        ys.seg_start[i] = w.part_col[i];
        ys.seg_y[i] = Ys[i];
        ys.seg_ld[i] = w.part_col[i + 1] - w.part_col[i];
      }
      ys.seg_start[w.nparts] = w.N;
      return launch_mma_nbits(s, w, dA, M, nullptr, w.N, mode, s->stream, 0, nullptr, &ys);
    }
    const int mflags = flags & (ORT_CUDA_MODE_OVERRIDE | 0xF000);
    rc = ort_cuda_matmul_nbits(s, fused, dA, M, scratch, mflags);
    if (rc) return rc;
  }
  if (!host && gemv) return ORT_CUDA_OK;
  // split the [M, N] rows of scratch into the parts
  for (int i = 0; i < w.nparts; i++) {
    const int64_t ni = w.part_col[i + 1] - w.part_col[i];
    ORTC_CUDA(cudaMemcpy2DAsync(Ys[i], (size_t)(ni * 4), scratch + w.part_col[i],
                                (size_t)(w.N * 4), (size_t)(ni * 4), (size_t)M,
                                host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice,
                                s->stream));
  }
  return host ? bounded_sync(s) : ORT_CUDA_OK;
}

static int matmul_integer_op(ort_cuda_session* s, const char* name, const void* A, int64_t M,
                             int a_signed, const void* a_zp, int64_t a_zp_len, int32_t* Y,
                             int flags) {
  ORTC_CHECK(s && name && A && Y, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 0 && M < (1ll << 30), ORT_CUDA_ERR_INVALID_ARG, "bad M");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  const Weight& w = it->second;
  ORTC_CHECK(w.kind == W_INT8, ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + name + "' is not a MatMulInteger weight");
  ORTC_CHECK(a_zp == nullptr || a_zp_len == 1 || a_zp_len == M, ORT_CUDA_ERR_UNSUPPORTED,
             "MatMulInteger: a_zp must be scalar or per-row [M]");
  if (M == 0) return ORT_CUDA_OK;
  DeviceGuard g(s->device);
  OpTimer timer(s, "MatMulInteger");
  const size_t zbytes = a_zp ? (size_t)a_zp_len : 0;
  return run_op(s, w, A, (size_t)(M * w.K), a_zp, zbytes, reinterpret_cast<float*>(Y), M, flags,
                [&](const float* dA, const float* dC, float* yl, int64_t ldy) -> int {
                  const uint8_t* a8 = reinterpret_cast<const uint8_t*>(dA);
                  int64_t lda = w.K;
                  // A rows 16-byte aligned for TMA, padded copy otherwise;
                  // then the row sums the zero-point correction needs
                  const bool pad = (w.K % 16) != 0 || (reinterpret_cast<uintptr_t>(a8) & 15);
                  const size_t pad_bytes = pad ? (size_t)(M * w.kpitch) : 0;
                  int rc = ensure_kscratch(s, ((pad_bytes + 255) & ~(size_t)255) + (size_t)M * 4);
                  if (rc) return rc;
                  if (pad) {
                    ORTC_CUDA(cudaMemcpy2DAsync(s->kscratch, (size_t)w.kpitch, a8, (size_t)w.K,
                                                (size_t)w.K, (size_t)M, cudaMemcpyDeviceToDevice,
                                                s->stream));
                    a8 = static_cast<const uint8_t*>(s->kscratch);
                    lda = w.kpitch;
                  }
                  int32_t* rowsum = reinterpret_cast<int32_t*>(
                      static_cast<char*>(s->kscratch) + ((pad_bytes + 255) & ~(size_t)255));
                  return launch_matmul_i8(w, a8, lda, M, a_signed ? 1 : 0,
                                          reinterpret_cast<const uint8_t*>(dC), a_zp_len,
                                          reinterpret_cast<int32_t*>(yl), ldy, rowsum,
                                          s->err_dev, s->sm_count, s->stream, &s->launches);
                });
}

extern "C" {

ORT_CUDA_API int ort_cuda_matmul_integer(ort_cuda_session* s, const char* name, const void* A,
                                         int64_t M, int a_signed, const void* a_zp,
                                         int64_t a_zp_len, int32_t* Y, int flags) {
  return matmul_integer_op(s, name, A, M, a_signed, a_zp, a_zp_len, Y, flags);
}

static int dense_op(ort_cuda_session* s, const char* op_type, const char* name,
                    const float* A, int64_t M, const float* C, int64_t c_rows, int64_t c_cols,
                    float alpha, float beta, float* Y, int flags) {
  ORTC_CHECK(s && name, ORT_CUDA_ERR_INVALID_ARG, "NULL argument");
  ORTC_CHECK(M >= 0, ORT_CUDA_ERR_INVALID_ARG, "M must be >= 0");
  auto it = s->weights.find(name);
  ORTC_CHECK(it != s->weights.end(), ORT_CUDA_ERR_NOT_FOUND,
             std::string("no weight named '") + name + "'");
  Weight& w = it->second;
  ORTC_CHECK(w.kind == W_DENSE, ORT_CUDA_ERR_INVALID_ARG,
             std::string("weight '") + name + "' is not a dense MatMul/Gemm weight");
  if (C) {
    ORTC_CHECK((c_rows == 1 || c_rows == M) && (c_cols == 1 || c_cols == w.N),
               ORT_CUDA_ERR_INVALID_ARG,
               "Gemm: C [" + std::to_string(c_rows) + "," + std::to_string(c_cols) +
                   "] does not broadcast to [" + std::to_string(M) + "," +
                   std::to_string(w.N) + "]");
  }
  if (M == 0) return ORT_CUDA_OK;
  ORTC_CHECK(A && Y, ORT_CUDA_ERR_INVALID_ARG, "NULL A or Y");
  const int mode = mode_of(s, flags);
  ORTC_CHECK(valid_mode(mode), ORT_CUDA_ERR_INVALID_ARG, "unknown mode");
  const bool transA = (flags & ORT_CUDA_TRANS_A) != 0;
  DeviceGuard g(s->device);
  OpTimer timer(s, op_type);
  return run_op(s, w, A, (size_t)(M * w.K) * 4, C, C ? (size_t)(c_rows * c_cols) * 4 : 0, Y, M,
                flags,
                [&](const float* dA, const float* dC, float* yl, int64_t ldy) -> int {
                  const bool mma = mode == ORT_CUDA_MODE_MMA_F16 || mode == ORT_CUDA_MODE_MMA_BF16;
                  if (mma && mma_supported_shape(M, w.K))
                    return launch_mma_dense(s, w, dA, M, transA, yl, ldy, mode, alpha, beta, dC,
                                            c_rows, c_cols, w.n0, s->stream);
                  return launch_simt_gemm(w, dA, M, transA, yl, ldy, mode == ORT_CUDA_MODE_STRICT,
                                          alpha, beta, dC, c_rows, c_cols, w.n0, s->stream,
                                          &s->launches);
                });
}

ORT_CUDA_API int ort_cuda_matmul(ort_cuda_session* s, const char* name, const float* A,
                                 int64_t M, float* Y, int flags) {
  return dense_op(s, "MatMul", name, A, M, nullptr, 0, 0, 1.0f, 1.0f, Y,
                  flags & ~ORT_CUDA_TRANS_A);
}

ORT_CUDA_API int ort_cuda_gemm(ort_cuda_session* s, const char* name, const float* A, int64_t M,
                               const float* C, int64_t c_rows, int64_t c_cols, float alpha,
                               float beta, float* Y, int flags) {
  return dense_op(s, "Gemm", name, A, M, C, c_rows, c_cols, alpha, beta, Y, flags);
}

ORT_CUDA_API int ort_cuda_matmul_batched(ort_cuda_session* s, const float* A, const float* B,
                                         int64_t batch, int64_t m, int64_t k, int64_t n,
                                         int64_t b_batch_stride, float* Y, int flags) {
  ORTC_CHECK(s, ORT_CUDA_ERR_INVALID_ARG, "session is NULL");
  ORTC_CHECK(batch >= 0 && m >= 0 && k >= 0 && n >= 0, ORT_CUDA_ERR_INVALID_ARG,
             "negative dimension");
  ORTC_CHECK(b_batch_stride == 0 || b_batch_stride == k * n, ORT_CUDA_ERR_INVALID_ARG,
             "b_batch_stride must be 0 or k*n");
  if (batch * m * n == 0) return ORT_CUDA_OK;
  ORTC_CHECK(A && B && Y, ORT_CUDA_ERR_INVALID_ARG, "NULL pointer");
  const int mode = mode_of(s, flags);
  DeviceGuard g(s->device);
  OpTimer timer(s, "MatMul");
  const bool strict = mode == ORT_CUDA_MODE_STRICT;
  if (!(flags & ORT_CUDA_HOST_IO))
    return launch_simt_batched(A, B, batch, m, k, n, b_batch_stride, Y, strict, s->stream,
                               &s->launches);
  const int64_t bB = b_batch_stride ? batch * k * n : k * n;
  const size_t oa = 0, ob = al256((size_t)(batch * m * k) * 4),
               oy = ob + al256((size_t)bB * 4), tot = oy + al256((size_t)(batch * m * n) * 4);
  int rc = ensure_ws(s, tot);
  if (rc) return rc;
  char* ws = (char*)s->ws;
  ORTC_CUDA(cudaMemcpyAsync(ws + oa, A, (size_t)(batch * m * k) * 4, cudaMemcpyHostToDevice, s->stream));
  ORTC_CUDA(cudaMemcpyAsync(ws + ob, B, (size_t)bB * 4, cudaMemcpyHostToDevice, s->stream));
  rc = launch_simt_batched((const float*)(ws + oa), (const float*)(ws + ob), batch, m, k, n,
                           b_batch_stride, (float*)(ws + oy), strict, s->stream, &s->launches);
  if (rc) return rc;
  ORTC_CUDA(cudaMemcpyAsync(Y, ws + oy, (size_t)(batch * m * n) * 4, cudaMemcpyDeviceToHost, s->stream));
  ORTC_CUDA(cudaStreamSynchronize(s->stream));
  return ORT_CUDA_OK;
}

}  // extern "C"
