// Internal declarations shared by the ort_cuda translation units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <unordered_map>
#include <unordered_set>

#include "../../include/ort_cuda.h"

namespace ortc {

// ---- error plumbing ------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define ORTC_CUDA(call)                                  \
  do {                                                   \
    cudaError_t _e = (call);                             \
    if (_e != cudaSuccess) return ::ortc::cuda_fail(_e, #call); \
  } while (0)

#define ORTC_CHECK(cond, code, msg)                      \
  do {                                                   \
    if (!(cond)) return ::ortc::fail((code), (msg));     \
  } while (0)

// ---- weights -------------------------------------------------------------
enum WeightKind { W_NBITS = 1, W_DENSE = 2, W_INT8 = 3, W_GROUP = 4 };
constexpr int kMaxSegs = 4;  // weights in one fused group (ort_cuda_fuse_nbits)

// One uploaded initializer, resident for the session.  For an N-sharded
// session only this rank's columns [n0, n0 + nl) are stored.
struct Weight {
  WeightKind kind = W_NBITS;
  int64_t K = 0, N = 0;   // logical shape [K, N] of the full weight
  int64_t n0 = 0, nl = 0; // this rank's column range
  int64_t ns = 0;         // padded per-rank column count (all-gather unit)
  // MatMulNBits, in the device layout every kernel reads (see nbits_*):
  int bs = 0, nb = 0;
  bool has_zp = false;
  uint8_t* B = nullptr;      // [nl][nb*bs/2] packed uint4, nibbles of each 32-bit
                             // word reordered (nbits_nibble below)
  float* scales = nullptr;   // [nb][s_pitch] fp32 (transposed: block-major)
  int64_t s_pitch = 0;       // >= nl, multiple of 4
  uint16_t* scales16 = nullptr;  // the same as fp16 when uploaded as fp16 (the
  int64_t s16_pitch = 0;         // decode GEMV streams these); pitch % 8 == 0
  uint8_t* zp = nullptr;     // [ceil(nb/2)][z_pitch] bytes: byte (b/2, n) holds
                             // blocks 2j (low nibble) and 2j+1 of column n
  int64_t z_pitch = 0;       // >= nl, multiple of 16
  // TMA views for the tensor-core GEMV (valid when tc_ok)
  CUtensorMap tmB, tmS, tmZ;
  bool tc_ok = false;
  // dense fp32 MatMul / Gemm operand, effective [K][nl] row-major
  float* W = nullptr;
  // Lazily built MMA operand: 16-bit [nl_pad][K_pad] K-major plus the
  // per-column power-of-two exponent that was factored out (F16 only).
  void* W16 = nullptr;
  int w16_mode = -1;
  int64_t w16_rows = 0, w16_k = 0;
  int* col_exp = nullptr;   // [nl_pad] (F16 mode), else nullptr
  uint32_t* sz16 = nullptr;  // nbits f16 MMA: per-(blk,col) {1024 + z, scale * 2^-col_exp} as fp16
  // the fused prefill GEMM's TMA views of the packed weight and of sz16,
  // encoded on its first call (they depend on the weight only)
  CUtensorMap tmQp, tmSZp;
  bool prefill_maps = false;
  // MatMulInteger weight (W_INT8): this rank's columns K-major [nl][kpitch]
  // (kpitch = K rounded up to 16), their column sums and zero points (int32)
  uint8_t* Wi8 = nullptr;
  int64_t kpitch = 0;
  int i8_signed = 0;
  int32_t* colsum = nullptr;
  int32_t* bzp = nullptr;  // [nl], or null without zero points
  CUtensorMap tmW8;
  // decode GEMV: the plan (candidate index) timing chose for each M in 1..8
  int8_t gemv_plan[9] = {-1, -1, -1, -1, -1, -1, -1, -1, -1};
  // N-sharded session, size-based placement: the whole weight on every rank
  // (n0 = 0, nl = ns = N), computed locally with no exchange
  bool replicated = false;
  // a fused group (ort_cuda_fuse_nbits): the parts' names and first columns
  // (part_col[i] .. part_col[i + 1]); on an N-sharded session only the names
  // are kept (no fused copy) and the group call runs the parts in turn
  int nparts = 0;
  std::string part_name[kMaxSegs];
  int64_t part_col[kMaxSegs + 1] = {};
  bool group_only = false;
};

// ---- device layout of a MatMulNBits weight ---------------------------------
// Within each 32-bit word of a column's packed bytes the 8 nibbles (k offsets
// 0..7 of that word) are stored at bit positions 0,8,16,24,4,12,20,28: k0..k3
// sit in the low nibbles of bytes 0..3 and k4..k7 in the high nibbles, so
// (w & 0x0F0F0F0F) and ((w >> 4) & 0x0F0F0F0F) are the int8 values of
// k0..k3 and k4..k7 in order — the tensor-core GEMV's A operand.
__host__ __device__ __forceinline__ int nbits_nibble_pos(int i) {
  return (i & 3) * 8 + (i >> 2) * 4;
}
__host__ __device__ __forceinline__ uint32_t nbits_permute_word(uint32_t o) {
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) w |= ((o >> (4 * i)) & 0xFu) << nbits_nibble_pos(i);
  return w;
}
// q of k offset i (0..7) within a permuted word
__host__ __device__ __forceinline__ uint32_t nbits_q(uint32_t w, int i) {
  return (w >> nbits_nibble_pos(i)) & 0xFu;
}
// zero point of column n, block b in the transposed nibble table
__host__ __device__ __forceinline__ uint32_t nbits_zp(const uint8_t* zp, int64_t z_pitch,
                                                      int64_t n, int64_t b) {
  return (zp[(b >> 1) * z_pitch + n] >> ((b & 1) * 4)) & 0xFu;
}

}  // namespace ortc

struct ort_cuda_profile;  // per-op-type device times (csrc/profile.cu)

struct ort_cuda_session {
  int device = 0;
  int mode = ORT_CUDA_MODE_EXACT;
  int rank = 0, world = 1;
  int timeout_ms = 60000;
  int sm_count = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  void* nccl = nullptr;  // ncclComm_t when world > 1
  std::unordered_map<std::string, ortc::Weight> weights;
  std::unordered_set<void*> allocs;
  // grow-only device scratch (A staging, per-rank Y before the gather ...)
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // grow-only pinned host staging for ORT_CUDA_HOST_IO calls
  void* pinned = nullptr;
  size_t pinned_bytes = 0;
  // grow-only kernel scratch for split-K partials (no initial value needed)
  void* kscratch = nullptr;
  size_t kscratch_bytes = 0;
  // grow-only ArgMax scratch: per-row tickets (arg_rows_cap, first) then
  // segment candidates (arg_cand_cap); zeroed when allocated, and every call
  // returns the tickets it used to zero
  void* argscratch = nullptr;
  int64_t arg_rows_cap = 0, arg_cand_cap = 0;
  // DynamicQuantizeLinear scratch (ticket, scale and zero point, per-CTA
  // ranges); zeroed once, every call returns the ticket to zero
  void* dqscratch = nullptr;
  // attention split-key scratch: tickets (zeroed when allocated, returned
  // to zero by every call) then partials
  void* attnscratch = nullptr;
  size_t attn_bytes = 0;
  // N-sharded sessions: peer-memory exchange of Y (csrc/p2p.cu).  xbuf holds
  // a 256-byte flag area (8 peer flags, epoch counter, CTA counter) then two
  // halves of xcap floats; xpeer[r] is rank r's xbuf mapped into this
  // process (xpeer[rank] = xbuf).
  void* xbuf = nullptr;
  void* xpeer[8] = {};
  size_t xcap = 0;
  bool p2p_ok = false;
  bool xsel_offer = false;  // run_op offers the exchange half to the producer
  bool xsel_taken = false;  // the producer wrote its slice there
  size_t llcap = 0;          // 64-bit words per half of the tagged (push) area
  float* push_y = nullptr;   // run_op offers push mode: the gathered Y [M, N]
  bool push_taken = false;   // the producer pushed (p2p_land completes the op)
  // run_op offers the NCCL exchange to the producer, which may run it in
  // row chunks overlapped with its own compute (prefill): the gathered Y,
  // the [G, M, Ns] landing area; `gathered` says the producer did it
  float* chunk_y = nullptr;
  float* chunk_gath = nullptr;
  bool gathered = false;
  cudaStream_t comm_stream = nullptr;  // the chunks' all-gathers and re-layouts
  // fused MatMulNBits + ArgMax: staging of host A / indices and unwanted
  // logits (grow-only), and the rows' keys (zero between calls)
  void* aux = nullptr;
  size_t aux_bytes = 0;
  void* amaxbuf = nullptr;
  cudaEvent_t chunk_ev[17] = {};       // chunk c computed; [16]: exchange done
  // big exchange buffer for prefill-sized outputs (csrc/p2p.cu): a flag
  // header then two halves of bcap floats, each [source rank][M][Ns];
  // bpeer[r] is rank r's, mapped here; epochs are counted on the host
  // (bepoch, the same on every rank)
  void* bbuf = nullptr;
  void* bpeer[8] = {};
  size_t bcap = 0;
  unsigned long long bepoch = 0;
  // bound of every wait for a peer GPU's flag or data (ms)
  int peer_wait_ms = 1000;
  // MatMulNBits weights of at most this many bytes are replicated on every
  // rank of an N-sharded session (-1: the default, 10 MB)
  int64_t replicate_bytes = -1;
  // CUDA graphs captured from the session stream (ort_cuda_graph_*)
  struct Graph {
    cudaGraphExec_t exec;
    int64_t launches;  // this library's kernels in the graph
  };
  std::map<int, Graph> graphs;
  int next_graph = 1;
  bool capturing = false;
  int64_t capture_launch0 = 0;
  // ort_cuda_profile_*: event pairs around each call while profiling
  ort_cuda_profile* prof = nullptr;
  bool profiling = false;
  // event bounded_sync records and polls (created on first use)
  cudaEvent_t sync_ev = nullptr;
  // host-mapped error word kernels write when a bounded wait gives up
  int* err_host = nullptr;
  int* err_dev = nullptr;
  int64_t launches = 0;
};

namespace ortc {

// Records a CUDA event pair on the session stream around one call of an
// entry point while the session profiles (ort_cuda_profile_enable); does
// nothing otherwise or while a graph is being captured.
class OpTimer {
 public:
  OpTimer(ort_cuda_session* s, const char* op);
  ~OpTimer();
  OpTimer(const OpTimer&) = delete;
  OpTimer& operator=(const OpTimer&) = delete;

 private:
  ort_cuda_session* s_ = nullptr;
  const char* op_ = nullptr;
  cudaEvent_t e0_ = nullptr;
};
void profile_free(ort_cuda_session* s);

// Scratch helpers (session-owned, stream-ordered reuse).
int ensure_ws(ort_cuda_session* s, size_t bytes);
int ensure_pinned(ort_cuda_session* s, size_t bytes);
// Where an N-sharded producer puts its outputs (inactive when ctr is null).
// The device-resident epoch counter ctr gives this operation's epoch
// e = ctr + 1.
//  - pull mode: the outputs go to half (e & 1) of this rank's exchange
//    buffer (half0, cap floats a half); p2p_gather then reads every rank's
//    half over peer memory.
//  - push mode: the outputs go to the caller's Y (the gathered [M, N]
//    layout, at this rank's columns) and, each as one 64-bit word
//    (e << 32 | float bits), to half (e & 1) of every peer's tagged
//    exchange area ll[r] (llcap words a half, row pitch N, row row0 + m,
//    column n0 + n); p2p_land on each peer waits for the tags and copies
//    the values into its own Y.  A 64-bit store is single-copy atomic, so
//    a word whose tag reads e holds this epoch's value: no fence and no
//    flag is needed between producer and consumer.
//  - fused ArgMax / ArgMin (amax non-null, independent of the modes above):
//    every stored value also enters the row's running key (amax_key) in the
//    CTA's shared memory; each CTA folds its keys into amax[row] with a
//    global atomic max, and the grid's last CTA writes amax_out[row] and
//    returns amax[] and its flags to zero (see amax_finish).
struct YSel {
  float* half0 = nullptr;
  int64_t cap = 0;
  const unsigned long long* ctr = nullptr;
  bool push = false;
  int rank = 0, world = 0, row0 = 0;
  int64_t n0 = 0, N = 0, llcap = 0;
  unsigned long long* ll[8] = {};
  // amax: [amax_rows] keys, then [amax_rows] u32 flags (column 0 is NaN),
  // then a u32 CTA ticket; zero between calls
  unsigned long long* amax = nullptr;
  int64_t* amax_out = nullptr;
  int amax_rows = 0, amax_min = 0, amax_last = 0;
  // segmented output (nseg > 0, a fused group of weights on one GPU):
  // column n in [seg_start[j], seg_start[j + 1]) goes to
  // seg_y[j][m * seg_ld[j] + n - seg_start[j]]
  int nseg = 0;
  int64_t seg_start[kMaxSegs + 1] = {};
  float* seg_y[kMaxSegs] = {};
  int64_t seg_ld[kMaxSegs] = {};
};

// ArgMax order of the reference's scan (opArgMinMax, onnx_ops.dart:2198-2237):
// the best non-NaN element under "larger value, then smaller index" (the
// larger index with select_last_index; ArgMin ranks -v), -0.0 equal to 0.0,
// as one unsigned key whose maximum is the answer; 0 for NaN (which wins
// only as element 0: handled by the column-0 flag).
__device__ __forceinline__ unsigned long long amax_key(float v, int64_t col, int is_min,
                                                       int last) {
  if (v != v) return 0ull;
  unsigned u = __float_as_uint(is_min ? -v : v);
  if ((u << 1) == 0u) u = 0u;  // -0.0 -> +0.0
  const unsigned o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  const unsigned ix = last ? (unsigned)col : 0xFFFFFFFFu - (unsigned)col;
  return ((unsigned long long)o << 32) | ix;
}
// Enters value v of local row m, local column n into the CTA's keys.
__device__ __forceinline__ void amax_add(const YSel& s, unsigned long long* s_keys,
                                         unsigned* s_nan0, int m, int n, float v) {
  const int64_t col = s.n0 + n;
  if (col == 0 && v != v) atomicOr(s_nan0, 1u << m);
  const unsigned long long k = amax_key(v, col, s.amax_min, s.amax_last);
  if (k) atomicMax(s_keys + m, k);
}
// Called by every thread of the CTA once its stores are done (after a
// CTA-wide barrier): folds the CTA's keys of rows row0 .. row0 + M - 1 into
// the grid's, and the last CTA decodes and resets them.
__device__ __forceinline__ void amax_finish(const YSel& s, const unsigned long long* s_keys,
                                            const unsigned* s_nan0, unsigned* s_last, int M) {
  unsigned long long* keys = s.amax;
  unsigned* nan0 = reinterpret_cast<unsigned*>(keys + s.amax_rows);
  unsigned* ticket = nan0 + s.amax_rows;
  if ((int)threadIdx.x < M) {
    const int row = s.row0 + (int)threadIdx.x;
    if (s_keys[threadIdx.x]) atomicMax(keys + row, s_keys[threadIdx.x]);
    if ((*s_nan0 >> threadIdx.x) & 1u) atomicOr(nan0 + row, 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    *s_last = atomicAdd(ticket, 1u) == gridDim.x * gridDim.y * gridDim.z - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (*s_last) {
    __threadfence();
    if ((int)threadIdx.x < M) {
      const int row = s.row0 + (int)threadIdx.x;
      const unsigned long long k = *reinterpret_cast<volatile unsigned long long*>(keys + row);
      const unsigned nf = *reinterpret_cast<volatile unsigned*>(nan0 + row);
      const unsigned lo = (unsigned)k;
      s.amax_out[row] = (nf || k == 0ull) ? 0 : (int64_t)(s.amax_last ? lo : 0xFFFFFFFFu - lo);
      keys[row] = 0ull;
      nan0[row] = 0u;
    }
    if (threadIdx.x == 0) *ticket = 0u;
  }
}
__device__ __forceinline__ unsigned long long ysel_epoch(const YSel& s) {
  return s.ctr ? *reinterpret_cast<const volatile unsigned long long*>(s.ctr) + 1 : 0ull;
}
__device__ __forceinline__ float* ysel_base(float* Y, const YSel& s) {
  if (!s.ctr || s.push) return Y;
  return s.half0 + (int64_t)(ysel_epoch(s) & 1) * s.cap;
}
// Yb[m * ldy + n] = v (Yb from ysel_base) and, in push mode, the tagged
// copy of v for every peer; e = ysel_epoch(s), read after the grid's
// dependency wait.
__device__ __forceinline__ void ysel_store(float* Yb, int64_t ldy, const YSel& s,
                                           unsigned long long e, int m, int n, float v) {
  if (s.nseg) {
    float* y = s.seg_y[0];
    int64_t ld = s.seg_ld[0], st = 0;
#pragma unroll
    for (int t = 1; t < kMaxSegs; t++)  // constant indices: no local copy
      if (t < s.nseg && n >= s.seg_start[t]) {
        y = s.seg_y[t];
        ld = s.seg_ld[t];
        st = s.seg_start[t];
      }
    y[m * ld + (n - st)] = v;
    return;
  }
  Yb[m * ldy + n] = v;
  if (s.push) {
    const unsigned long long word = (e << 32) | (unsigned long long)__float_as_uint(v);
    const int64_t off = (int64_t)(e & 1) * s.llcap + (int64_t)(s.row0 + m) * s.N + s.n0 + n;
#pragma unroll
    for (int r = 0; r < 8; r++)
      if (r < s.world && r != s.rank)
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(s.ll[r] + off), "l"(word)
                     : "memory");
  }
}

int ensure_kscratch(ort_cuda_session* s, size_t bytes);
// Reads and clears the kernels' error word (session.cu).
int check_kernel_error(ort_cuda_session* s);
// Waits for the session stream; with a communicator, bounded by the
// session timeout (the communicator is aborted on expiry).
int bounded_sync(ort_cuda_session* s);
struct PrefillPush;  // push mode of the sharded prefill GEMM (defined below)
// Peer-memory all-gather of Y for N-sharded sessions (p2p.cu).
int p2p_setup(ort_cuda_session* s);
void p2p_teardown(ort_cuda_session* s);
bool p2p_fits(ort_cuda_session* s, int64_t floats);
YSel p2p_ysel(ort_cuda_session* s);
// Push mode for a producer of rows [row0, row0 + m) of an [M, N] output
// whose local column 0 is global column n0 (see YSel).
bool p2p_push_fits(ort_cuda_session* s, int64_t M, int64_t N);
YSel p2p_ysel_push(ort_cuda_session* s, int64_t n0, int64_t N, int row0);
// Completes a push-mode operation: waits (bounded) for every peer's tagged
// words of this epoch and copies them into Y [M, N] (row pitch N); this
// rank's columns [n0, n0 + nl) are already there.  Advances the epoch.
int p2p_land(ort_cuda_session* s, int64_t M, int64_t N, int64_t n0, int64_t nl, float* Y);
// Big exchange buffer of two halves of at least half_floats floats on
// every rank (a collective: every rank calls it with the same size); *ok
// false when a peer could not be mapped (every rank then sees false).
int p2p_big_ensure(ort_cuda_session* s, size_t half_floats, bool* ok);
// Push-mode prefill (see PrefillPush): before the GEMM, waits (bounded)
// until every peer has consumed epoch - 2 from the half this epoch reuses;
// after it, lands the peers' blocks of `epoch` into Y [M, N] and tells
// each peer that its block was consumed.  The big buffer holds two halves
// of at least M * N floats.
int p2p_push_prepare(ort_cuda_session* s, unsigned long long epoch, int64_t M, int64_t ns,
                     PrefillPush* push);
int p2p_push_land(ort_cuda_session* s, unsigned long long epoch, int64_t M, int64_t ns,
                  int64_t N, float* Y);
// A rank without columns posts its empty block of the epoch ready.
int p2p_push_post(ort_cuda_session* s, const PrefillPush& push);

// `local` null: the producer already wrote the slice with p2p_ysel().
int p2p_gather(ort_cuda_session* s, const float* local, int64_t M, int64_t Ns, int64_t N,
               float* Y);

// cuTensorMapEncodeTiled through the runtime's driver entry point: a 2-D
// row-major tensor [d1][d0] with row pitch stride1 bytes, box b0 x b1.
int encode_tma_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0,
                  uint64_t d1, uint64_t stride1, uint32_t b0, uint32_t b1,
                  CUtensorMapSwizzle swz);

// ---- kernel launchers (each returns an ORT status) -----------------------
// All pointers are device pointers; launches go to `st`.

// Decode GEMV on tensor cores, exact mode: Y[M, ldy] (columns [0, nl)) =
// A[M, K] . dequant(W) for M <= 8 (tc_gemv_ok).  `partials` holds
// tc_gemv_partial_floats(.., plan) floats (no initial value needed).
int prepare_nbits_tc(Weight& w);
bool tc_gemv_ok(const Weight& w, int64_t M);
// tc_gemv_ok without the rank's own column count: the same answer on every
// rank of an N-sharded group (a rank holding no columns launches nothing).
bool tc_gemv_shape_ok(const Weight& w, int64_t M);
// The work plan a call uses: the one tune_tc_gemv chose for (w, M) when its
// partial sums fit in max_partial_floats, else the heuristic's choice among
// the candidates that fit; -1 if none fits.
int tc_gemv_plan(const Weight& w, int64_t M, int sm_count,
                 size_t max_partial_floats = (size_t)-1);
// Number of candidate plans for (w, M) on this device.
int tc_gemv_plan_count(const Weight& w, int64_t M, int sm_count);
// Partial-sum floats of plan `plan` (-1: the most any candidate needs).
size_t tc_gemv_partial_floats(const Weight& w, int64_t M, int sm_count, int plan);
int launch_tc_gemv(const Weight& w, int plan, const float* A, int64_t M, float* Y, int64_t ldy,
                   float* partials, int* err, int sm_count, cudaStream_t st, int64_t* launches,
                   const YSel* ysel = nullptr);
// Times every candidate plan on this call's operands and records the
// fastest in w.gemv_plan[M] (launches not counted; `partials` holds
// tc_gemv_partial_floats(w, M, sm, -1) floats).  Not while capturing.
int tune_tc_gemv(Weight& w, const float* A, int64_t M, float* Y, int64_t ldy, float* partials,
                 int* err, int sm_count, cudaStream_t st, const YSel* ysel);
// General CUDA-core tiled GEMM over an nbits or dense weight (any M).
// strict=true reproduces the reference's rounding bit for bit.
int launch_simt_gemm(const Weight& w, const float* A, int64_t M, bool transA, float* Y,
                     int64_t ldy, bool strict, float alpha, float beta, const float* C,
                     int64_t c_rows, int64_t c_cols, int64_t c_col0, cudaStream_t st,
                     int64_t* launches);
int launch_simt_batched(const float* A, const float* B, int64_t batch, int64_t m, int64_t k,
                        int64_t n, int64_t b_batch_stride, float* Y, bool strict,
                        cudaStream_t st, int64_t* launches);
// Upload-time device prepack helpers.
// ArgMax / ArgMin over the last axis of X[rows][ldx] (first `cols` columns)
// into out[rows] (device), the reference's tie and NaN rules.  Rows of more
// than one 16K-column segment use argminmax_candidates(rows, cols) slots of
// argminmax_candidate_bytes() in `candidates` and rows tickets, which must
// be zero on entry and are zero again when the kernel ends.
int64_t argminmax_candidates(int64_t rows, int64_t cols);
size_t argminmax_candidate_bytes();
int launch_argminmax(const float* X, int64_t rows, int64_t cols, int64_t ldx, bool is_min,
                     bool last, int64_t* out, unsigned* tickets, void* candidates,
                     cudaStream_t st, int64_t* launches);
// MatMulInteger (int32 Y[M][ldy] over this rank's columns) on tensor cores;
// A rows 16-byte aligned with lda % 16 == 0; rowsum holds M int32 when the
// weight has zero points.
// TopK over the last axis of X [rows][ldx]: vals/idx [rows][k], k <= 1024
size_t topk_scratch_bytes(int64_t rows, int64_t cols, int64_t k);
int launch_topk(const float* X, int64_t rows, int64_t cols, int64_t ldx, int64_t k, bool largest,
                float* vals, int64_t* idx, void* scratch, cudaStream_t st, int64_t* launches);
// DynamicQuantizeLinear of X[n] into Y[n] (uint8), *scale, *zp (device)
size_t dynamic_quant_scratch_bytes(int sm_count);
int launch_dynamic_quant(const float* X, int64_t n, uint8_t* Y, float* scale, uint8_t* zp,
                         void* scratch, int sm_count, cudaStream_t st, int64_t* launches);
// Attention over one (batch, KV head) sequence per CTA group, in fp32
// (csrc/attn.cu): the body of GroupQueryAttention, MultiHeadAttention and
// the fused SDPA pattern.  Element (b, i, h, d) of Q is
// q[b*qsb + i*qsi + h*qsh + d]; key j of KV head g is a past row
// (j < past: pk/pv[b*psb + g*psh + j*D + d]) or a row of this call
// (k[b*ksb + g*ksh + (j-past)*ksj + d*ksd], v[b*vsb + g*vsh + (j-past)*vsj + d]);
// query head h reads KV head h / group.
struct AttnArgs {
  const float* q = nullptr;
  int64_t qsb = 0, qsi = 0, qsh = 0;
  const float* k = nullptr;
  int64_t ksb = 0, ksh = 0, ksj = 0, ksd = 1;
  const float* v = nullptr;
  int64_t vsb = 0, vsh = 0, vsj = 0;
  const float* pk = nullptr;
  const float* pv = nullptr;
  int64_t psb = 0, psh = 0;
  // present K/V (GQA): prk[b*rsb + g*rsh + j*D + d] for j < T; rows j < past
  // are copied only when write_past (present does not alias past)
  float* prk = nullptr;
  float* prv = nullptr;
  int64_t rsb = 0, rsh = 0;
  int write_past = 0;
  // additive bias: bias[b*bsb + (h % bh)*bsh + i*bsi + j*bsj]
  const float* bias = nullptr;
  int64_t bsb = 0, bsh = 0, bsi = 0, bsj = 0;
  int bh = 1;
  float* out = nullptr;
  int64_t osb = 0, osi = 0, osh = 0;
  int batch = 0, seq = 0, heads_kv = 0, group = 1, D = 0, Dv = 0, past = 0, T = 0;
  // keys j < cached come from pk/pv (normally the past; all keys once a
  // pre-pass has written this call's rows to the present cache); query
  // token i is at position past + i either way
  int cached = -1;
  int causal = 0;
  double scale = 1.0;
  // RoPE of Q (position past+i) and of this call's K rows (position j)
  const float* cos = nullptr;
  const float* sin = nullptr;
  int half_rot = 0, interleaved = 0, rotary = 0;
  // filled by launch_attention
  int rows_total = 0, nqt = 0, nsplit = 1, vec = 0;
  float* part = nullptr;
  unsigned* tickets = nullptr;
  int* err = nullptr;  // host-mapped error word for a bounded wait that expired
};
// Scratch the launch needs (0 when no split of the keys is used); the
// tickets at its start must be zero on entry and are zero again at exit.
size_t attention_scratch_bytes(const AttnArgs& a, int sm_count);
int launch_attention(AttnArgs a, void* scratch, int sm_count, cudaStream_t st, int64_t* launches);
// RotaryEmbedding of X laid out [batch][seq][heads][head] (x_bhsd = 0) or
// [batch][heads][seq][head] (1); positions pos[(pos_per_batch ? b : 0)*seq + s]
int launch_rotary(const float* X, float* Y, const int64_t* pos, int pos_per_batch,
                  const float* cos, const float* sin, int64_t max_pos, int half_rot, int rdim,
                  int64_t batch, int64_t seq, int64_t heads, int64_t head, int x_bhsd,
                  int interleaved, cudaStream_t st, int64_t* launches);
int prepare_int8_tc(Weight& w);
int launch_matmul_i8(const Weight& w, const uint8_t* A, int64_t lda, int64_t M, int a_signed,
                     const uint8_t* azp, int64_t az_len, int32_t* Y, int64_t ldy,
                     int32_t* rowsum, int* err, int sm_count, cudaStream_t st,
                     int64_t* launches);
int launch_permute_nibbles(const uint32_t* in, uint32_t* out, int64_t nwords, cudaStream_t st,
                           int64_t* launches);
int launch_half_to_float(const uint16_t* h, float* out, int64_t n, cudaStream_t st,
                         int64_t* launches);
int launch_transpose(const float* in, float* out, int64_t rows, int64_t cols, cudaStream_t st,
                     int64_t* launches);
// [G, M, Ns] (gathered shards) -> Y[M, N]
int launch_unshard(const float* g, float* Y, int64_t world, int64_t M, int64_t Ns, int64_t N,
                   cudaStream_t st, int64_t* launches);

// tcgen05 MMA path (16-bit operands, fp32 accumulation in TMEM).
int mma_supported_shape(int64_t M, int64_t K);
// Fused int4 prefill GEMM (fp16 MMA mode), csrc/gemm_nbits_tc.cu.
bool nbits_gemm_f16_ok(const Weight& w);
// nbits_gemm_f16_ok without the rank's own column count (the same on every rank)
bool nbits_gemm_f16_layout_ok(const Weight& w);
int prepare_nbits_sz16(const Weight& w, const int* col_exp, uint32_t* out, cudaStream_t st,
                       int64_t* launches);
int launch_nbits_gemm_f16(Weight& w, const uint16_t* A16, const int* row_exp, int64_t M,
                          const uint32_t* sz16, const int* col_exp, float* Y, int64_t ldy,
                          int* err, int sm_count, cudaStream_t st, int64_t* launches,
                          int reserve_sms = 0, const PrefillPush* push = nullptr,
                          const YSel* seg = nullptr);
// N-sharded prefill, push mode of the fused fp16 GEMM: besides its own
// columns in Y, every output row slice [row][0, nl) is stored into each
// peer's landing area land[r] (this rank's block of it, [M][Ns] floats);
// when every CTA has finished (each storing thread fences at system scope),
// the last CTA posts `epoch` into flag[r] of every peer.
struct PrefillPush {
  float* land[8] = {};
  unsigned long long* flag[8] = {};
  unsigned* ticket = nullptr;  // this rank's CTA ticket, zero between calls
  unsigned long long epoch = 0;
  int64_t ns = 0;
  int rank = 0, world = 0;
};
// reserve_sms: SMs the fused fp16 GEMM leaves free for a kernel beside it
// seg: the segmented output of a fused group (YSel's seg_* fields; the
// fused fp16 GEMM only, boundaries multiples of 32)
int launch_mma_nbits(ort_cuda_session* s, Weight& w, const float* A, int64_t M, float* Y,
                     int64_t ldy, int mode, cudaStream_t st, int reserve_sms = 0,
                     const PrefillPush* push = nullptr, const YSel* seg = nullptr);

int launch_mma_dense(ort_cuda_session* s, Weight& w, const float* A, int64_t M, bool transA,
                     float* Y, int64_t ldy, int mode, float alpha, float beta, const float* C,
                     int64_t c_rows, int64_t c_cols, int64_t c_col0, cudaStream_t st);

}  // namespace ortc
