/*
 * ort_cuda.h — C ABI of the B200 matmul hot path for onnx_runtime_dart.
 *
 * The reference (CrispStrobe/onnx_runtime_dart 0.10.3, pure Dart) computes
 * MatMulNBits, MatMul and Gemm inside OnnxGraphExecutor._dispatch
 * (lib/src/onnx_graph.dart:961).  This library replaces the bodies of those
 * three cases: a dart:ffi binding calls the functions below, which launch
 * hand-written sm_100a CUDA kernels.  No Python, no PyTorch and no CPU
 * compute sits behind these entry points.
 *
 * Conventions
 *  - Every function returns an int status (ORT_CUDA_OK == 0).  On failure
 *    ort_cuda_last_error() returns a thread-local message.  The Dart side
 *    maps ORT_CUDA_ERR_UNSUPPORTED to UnsupportedError (as
 *    lib/src/onnx_qlinear_ops.dart:117-119 and onnx_graph.dart:1585-1588
 *    throw) and every other code to StateError (onnx_graph.dart:789-795).
 *  - All matrices are row-major fp32 unless stated, like the reference's
 *    Float32List tensors (lib/src/tensor.dart:14-59).
 *  - Weights are uploaded once per session and addressed by initializer
 *    name, as the reference caches prepacked Gemm B by name
 *    (onnx_graph.dart:53-56, :1160).
 *  - A/C/Y pointers are device pointers (stream-ordered, asynchronous on
 *    the session stream) unless ORT_CUDA_HOST_IO is set, in which case they
 *    are host pointers and the call returns after Y has been written.
 */
#ifndef ORT_CUDA_H_
#define ORT_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORT_CUDA_API __attribute__((visibility("default")))

/* ---- status codes ---------------------------------------------------- */
#define ORT_CUDA_OK 0
#define ORT_CUDA_ERR_INVALID_ARG 1 /* bad shape / size / pointer      */
#define ORT_CUDA_ERR_UNSUPPORTED 2 /* bits != 4, g_idx/bias, ...      */
#define ORT_CUDA_ERR_CUDA 3        /* CUDA runtime or launch failure  */
#define ORT_CUDA_ERR_NCCL 4        /* NCCL failure                    */
#define ORT_CUDA_ERR_TIMEOUT 5     /* collective / device wait timed out */
#define ORT_CUDA_ERR_NOT_FOUND 6   /* no weight uploaded under name   */
#define ORT_CUDA_ERR_OOM 7         /* device allocation failed        */

/* ---- arithmetic modes ------------------------------------------------ */
/* fp32 inputs, fp32 dequantisation, fp32 FFMA accumulation.  Within 1e-5
 * max-relative error (max|dY| / max|Y_ref|) of the reference. */
#define ORT_CUDA_MODE_EXACT 0
/* The reference's own rounding sequence (k-ascending, separate fp32
 * multiply and add, double-accumulated tail columns of
 * gemm_kernel_simd.dart:299-307): bitwise equal to the Dart VM result.
 * Slow; meant for parity checks. */
#define ORT_CUDA_MODE_STRICT 1
/* tcgen05 tensor-core MMA on 16-bit operands with fp32 accumulation in
 * TMEM.  F16 operands use per-row / per-column power-of-two range
 * normalisation; BF16 operands are split into two bf16 terms (hi and lo)
 * and every product formed from three MMAs (A_hi.W_hi + A_lo.W_hi +
 * A_hi.W_lo), keeping about 16 significant bits of each operand at three
 * times the tensor work.  Both meet 2e-3 max-relative error with cosine
 * >= 0.99999 (the bf16 mode stays near 1e-5). */
#define ORT_CUDA_MODE_MMA_F16 2
#define ORT_CUDA_MODE_MMA_BF16 3

/* ---- call flags ------------------------------------------------------ */
#define ORT_CUDA_HOST_IO 0x1 /* A, C, Y are host pointers; synchronous   */
#define ORT_CUDA_MODE_OVERRIDE 0x100 /* bits 12..15 carry a mode for this call */
#define ORT_CUDA_FLAGS_MODE(m) (ORT_CUDA_MODE_OVERRIDE | (((m)&0xF) << 12))
#define ORT_CUDA_TRANS_A 0x2 /* Gemm transA=1: A is [K x M]              */

/* ---- upload flags ---------------------------------------------------- */
#define ORT_CUDA_SCALES_F32 0
#define ORT_CUDA_SCALES_F16 1 /* fp16 bit patterns, widened bit-exactly on
                                 the device like
                                 onnx_proto_loader.dart:29-47 */
/* Zero points indexed flat, nibble (n*nb + blk) — the reference's layout
 * (onnx_qlinear_ops.dart:133-138).  Default. */
#define ORT_CUDA_ZP_FLAT 0x0
/* Zero points per column, ceil(nb/2) bytes per column (the ORT
 * com.microsoft spec).  Differs from the reference only when nb is odd. */
#define ORT_CUDA_ZP_PER_COLUMN 0x10
/* ort_cuda_argmax: ArgMin instead of ArgMax; ties to the last index
 * (ONNX select_last_index=1) instead of the first */
#define ORT_CUDA_ARG_MIN 0x20
#define ORT_CUDA_ARG_SELECT_LAST 0x40

typedef struct ort_cuda_session ort_cuda_session;

/* Thread-local text of the last failure on this thread ("" if none). */
ORT_CUDA_API const char* ort_cuda_last_error(void);

/* Library version string. */
ORT_CUDA_API const char* ort_cuda_version(void);

/* Number of visible CUDA devices. */
ORT_CUDA_API int ort_cuda_device_count(int* count);

/* ---- sessions -------------------------------------------------------- */
/* Opens a single-GPU session on `device` with default arithmetic `mode`.
 * Replaces the in-process state OnnxGraphExecutor builds at load
 * (onnx_graph.dart:80-98) for the three hot ops. */
ORT_CUDA_API int ort_cuda_open(int device, int mode, ort_cuda_session** out);

/* Writes a 128-byte NCCL unique id (call on one rank, share the bytes). */
ORT_CUDA_API int ort_cuda_nccl_unique_id(void* id128);

/* Opens rank `rank` of a `world`-rank session, one process per GPU.
 * Weights uploaded afterwards are sharded along N (output columns): rank r
 * keeps columns [r*Ns, min(N, (r+1)*Ns)), Ns = ceil(N/world) rounded up
 * to 4, the B200 counterpart of GemmPool's column split
 * (parallel_pool.dart:121-147).  Every matmul then all-gathers Y over
 * NCCL so each rank holds the full [M x N] result, as GemmPool.matmul
 * reassembles column slices (parallel_pool.dart:179-205).
 * `timeout_ms` bounds NCCL initialisation and every collective; on expiry
 * the communicator is aborted and ORT_CUDA_ERR_TIMEOUT returned. */
ORT_CUDA_API int ort_cuda_open_rank(int device, int rank, int world, const void* nccl_id128,
                                    int mode, int timeout_ms, ort_cuda_session** out);

/* Bound, in milliseconds, of every wait of this rank's kernels for a peer
 * GPU (its flag or its data) in the exchange of Y (default 1000).  When a
 * peer does not arrive in time the waiting kernel stops, records the
 * failure and returns; the next synchronising call reports
 * ORT_CUDA_ERR_TIMEOUT (a rank that skipped an operation or stopped is
 * detected this way, without any unbounded wait on the device). */
ORT_CUDA_API int ort_cuda_set_peer_wait(ort_cuda_session* s, int ms);

/* Size-based placement on an N-sharded session.  A MatMulNBits weight
 * uploaded after this call whose packed bytes (B, scales and zero points) are
 * at most `bytes` is kept whole on every rank and computed there without any
 * exchange of Y; larger weights keep their column shard.  Sharding saves
 * (1 - 1/world) of a weight's stream time but adds the exchange of its
 * output and leaves the per-launch fixed cost of a decode op unshrunk.  -1
 * means the default, 10 MB (measured: small decode projections run faster
 * whole, projections above about 10 MB gain little or lose, and large-M
 * prefill prefers its shard); 0 shards every weight.  The environment
 * variable ORT_CUDA_REPLICATE_BYTES sets it at ort_cuda_open_rank.  Every
 * rank must use the same value.  Results are the single-GPU results either
 * way. */
ORT_CUDA_API int ort_cuda_set_replicate_bytes(ort_cuda_session* s, int64_t bytes);

/* The columns [*n0, *n0 + *nl) of weight `name` held and computed by this
 * rank: its shard, or 0 and N for a replicated weight or a single-GPU
 * session. */
ORT_CUDA_API int ort_cuda_weight_columns(ort_cuda_session* s, const char* name, int64_t* n0,
                                         int64_t* nl);

/* Frees every device buffer of the session (OnnxModel.dispose,
 * lib/onnx_runtime_dart.dart:140). */
ORT_CUDA_API int ort_cuda_close(ort_cuda_session* s);

/* Changes the session's default mode. */
ORT_CUDA_API int ort_cuda_set_mode(ort_cuda_session* s, int mode);

/* Makes the session launch on an existing cudaStream_t (NULL restores the
 * session's own stream).  For hosts that already own a stream. */
ORT_CUDA_API int ort_cuda_set_stream(ort_cuda_session* s, void* cuda_stream);

/* Blocks until all work queued on the session stream has finished. */
ORT_CUDA_API int ort_cuda_sync(ort_cuda_session* s);

/* Rank / world of the session (1-GPU sessions: 0 / 1). */
ORT_CUDA_API int ort_cuda_rank_info(ort_cuda_session* s, int* rank, int* world);

/* ---- weight residency ---------------------------------------------- */
/* Uploads a MatMulNBits weight once per session (the reference reads it
 * from _initializers every call, onnx_qlinear_ops.dart:120-149).
 *   B       uint8 [N, nb, block_size/2], nb = ceil(K/block_size), packed
 *           low nibble first
 *   scales  [N*nb] fp32, or fp16 bit patterns with ORT_CUDA_SCALES_F16
 *   zp      NULL (implicit 8) or packed uint4 zero points (see ZP flags)
 * bits must be 4 (else ORT_CUDA_ERR_UNSUPPORTED, as
 * onnx_qlinear_ops.dart:117-119); block_size a power of two >= 16.
 * Host pointers; the call is synchronous.  Re-uploading a name replaces
 * the previous weight. */
ORT_CUDA_API int ort_cuda_upload_nbits(ort_cuda_session* s, const char* name, const uint8_t* B,
                                       const void* scales, const uint8_t* zp, int64_t K,
                                       int64_t N, int bits, int block_size, int flags);

/* Uploads a dense fp32 MatMul/Gemm weight.  `B` is [rows x cols]; with
 * trans_b=1 it is stored transposed ([K,N] = B^T), the prepack of
 * onnx_graph.dart:1156-1173 done once at upload instead of at first run.
 * Host pointer, synchronous. */
ORT_CUDA_API int ort_cuda_upload_dense(ort_cuda_session* s, const char* name, const float* B,
                                       int64_t rows, int64_t cols, int trans_b);

/* The same weight read straight from a file of ONNX external data (the
 * companion `.onnx.data` of a model too large to hold in host memory): packed
 * B at byte b_offset (N * ceil(K/bs) * bs/2 bytes), scales at scales_offset
 * (N * ceil(K/bs) fp32, or fp16 with ORT_CUDA_SCALES_F16), zero points at
 * zp_offset (< 0: none; flat or ORT_CUDA_ZP_PER_COLUMN size).  B streams
 * through a small pinned buffer and an N-sharded rank reads only its own
 * columns, so no host copy of the weight is made.  `path` is the resolved
 * companion file (the host keeps the reference's rules for which paths a
 * model may name); a range outside the file or a short read returns
 * ORT_CUDA_ERR_INVALID_ARG (the reference's FormatException).  Replaces, for
 * MatMulNBits initializers, the resolve() of loadOnnxModel
 * (lib/onnx_runtime_dart_io.dart:19-45) feeding _rawBytes
 * (lib/src/onnx_proto_loader.dart:89-112). */
ORT_CUDA_API int ort_cuda_upload_nbits_file(ort_cuda_session* s, const char* name,
                                            const char* path, int64_t b_offset,
                                            int64_t scales_offset, int64_t zp_offset, int64_t K,
                                            int64_t N, int bits, int block_size, int flags);

/* MatMulInteger weight (the int8 dynamic-quantisation path of
 * opMatMulInteger, lib/src/onnx_qlinear_ops.dart:26-79): B [K x N] row-major
 * bytes, int8 when b_signed else uint8; zero points b_zp (same type, host)
 * scalar (b_zp_len 1) or per column (N), or NULL.  Packed once, K-major with
 * per-column sums, like the reference's prepacked Gemm B. */
ORT_CUDA_API int ort_cuda_upload_int8(ort_cuda_session* s, const char* name, const void* B,
                                      int64_t K, int64_t N, int b_signed, const void* b_zp,
                                      int64_t b_zp_len);

/* Releases one weight. */
ORT_CUDA_API int ort_cuda_drop_weight(ort_cuda_session* s, const char* name);

/* Shape of an uploaded weight ([K, N], full unsharded N). */
ORT_CUDA_API int ort_cuda_weight_shape(ort_cuda_session* s, const char* name, int64_t* K,
                                       int64_t* N);

/* ---- device tensors (activations kept resident between ops) --------- */
ORT_CUDA_API int ort_cuda_alloc(ort_cuda_session* s, int64_t bytes, void** dptr);
ORT_CUDA_API int ort_cuda_free(ort_cuda_session* s, void* dptr);
ORT_CUDA_API int ort_cuda_h2d(ort_cuda_session* s, void* dst, const void* src, int64_t bytes);
ORT_CUDA_API int ort_cuda_d2h(ort_cuda_session* s, void* dst, const void* src, int64_t bytes);

/* ---- the hot ops ---------------------------------------------------- */
/* MatMulNBits (com.microsoft), onnx_qlinear_ops.dart:114-156 and its
 * dispatch case onnx_graph.dart:1584-1596:  Y[M,N] = A[M,K] . W[K,N],
 * W[k,n] = (q - zp) * scale.  M = element count of A / K. */
ORT_CUDA_API int ort_cuda_matmul_nbits(ort_cuda_session* s, const char* name, const float* A,
                                       int64_t M, float* Y, int flags);

/* MatMulNBits that allocates no device memory.  No counterpart in the
 * reference (which has no device memory at all).  For hosts that must not
 * allocate once running — a fixed memory budget reserved at start-up,
 * device memory owned by another runtime's allocator, or a latency path
 * where cudaMalloc's implicit device synchronisation is not acceptable.
 * ort_cuda_matmul_nbits may grow session scratch with cudaMalloc; this
 * call runs the same exact-mode decode GEMV with its split-K scratch in a
 * static device array of this library: 4 MiB of partial sums, held by every
 * GPU that loads the library until the process exits.  When the work plan
 * the regular entry point uses would need more scratch than that, the call
 * runs the fastest-estimated plan that fits (the tile-major plan needs
 * none); every plan gives the same bits, so Y equals the regular entry
 * point's Y bit for bit and only the speed can differ.
 *   A, Y   DEVICE pointers ([M,K] and [M,N] fp32); the call is
 *          stream-ordered on the session stream
 *   M      1..4 (else ORT_CUDA_ERR_INVALID_ARG); 32 <= block_size <= 512;
 *          single-GPU sessions whose mode is not STRICT (the call always
 *          runs the exact-mode GEMV; a STRICT session gets
 *          ORT_CUDA_ERR_UNSUPPORTED)
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture
 * (a first call during a capture returns ORT_CUDA_ERR_INVALID_ARG).
 * All calls share the array, so calls that overlap on the GPU (other
 * streams, other sessions on the same device) race. */
ORT_CUDA_API int ort_cuda_matmul_nbits_noalloc(ort_cuda_session* s, const char* name,
                                               const float* A, int64_t M, float* Y);

/* MatMul with an uploaded [K,N] weight, onnx_ops.dart:1375-1431 with the
 * shared-weight batch collapse of :1389-1400 (pass M = batch*m). */
ORT_CUDA_API int ort_cuda_matmul(ort_cuda_session* s, const char* name, const float* A,
                                 int64_t M, float* Y, int flags);

/* Gemm, onnx_ops.dart:1777-1793 on the prepacked B of
 * onnx_graph.dart:1156-1173:  Y = alpha * A' . B + beta * C.
 * C is NULL or [c_rows x c_cols] with c_rows in {1, M}, c_cols in {1, N}
 * (numpy broadcast as opAdd does, onnx_ops.dart:218-250).  With
 * ORT_CUDA_TRANS_A, A is stored [K x M]. */
ORT_CUDA_API int ort_cuda_gemm(ort_cuda_session* s, const char* name, const float* A, int64_t M,
                               const float* C, int64_t c_rows, int64_t c_cols, float alpha,
                               float beta, float* Y, int flags);

/* Batched activation x activation MatMul (no uploaded weight), the
 * per-batch loop of onnx_ops.dart:1402-1429 for equal batch counts:
 * Y[b] = A[b] . B[b], A [batch,m,k], B [batch,k,n] (b_batch_stride = 0
 * broadcasts one B).  Device or host pointers as per flags. */
ORT_CUDA_API int ort_cuda_matmul_batched(ort_cuda_session* s, const float* A, const float* B,
                                         int64_t batch, int64_t m, int64_t k, int64_t n,
                                         int64_t b_batch_stride, float* Y, int flags);

/* CUDA graphs of a sequence of device-pointer calls (the decode step of a
 * model, for instance).  No counterpart in the reference, whose executor
 * interprets the graph op by op on the CPU (onnx_graph.dart:961); here the
 * ops of one step are recorded once and replayed with a single launch, so
 * the host's per-op cost leaves the step.  Between graph_begin and
 * graph_end, matmul / gemm calls on device pointers are recorded, not run;
 * run every recorded op once before capturing (a call that would grow a
 * buffer, use ORT_CUDA_HOST_IO or synchronise is refused with
 * ORT_CUDA_ERR_INVALID_ARG).  Replays read and write the same device
 * buffers as the recorded calls.  The session stream must not be the
 * legacy default stream.  N-sharded sessions replay correctly: the
 * peer-exchange epoch lives on the device. */
ORT_CUDA_API int ort_cuda_graph_begin(ort_cuda_session* s);
ORT_CUDA_API int ort_cuda_graph_end(ort_cuda_session* s, int* graph_id);
ORT_CUDA_API int ort_cuda_graph_launch(ort_cuda_session* s, int graph_id);
ORT_CUDA_API int ort_cuda_graph_drop(ort_cuda_session* s, int graph_id);

/* Decode-GEMV work plan of MatMulNBits weight `name` for M rows (1..8):
 * the candidate decomposition the library timed and chose on the weight's
 * first call with that M, -1 while none is chosen.  Setting a plan (or -1)
 * replaces that choice, e.g. to reuse choices saved from an earlier
 * session of the same shapes on the same device instead of timing again;
 * every plan gives identical results.  ORT_CUDA_ERR_INVALID_ARG for a plan
 * outside [-1, number of candidates).  No counterpart in the reference,
 * whose one CPU kernel has no plans (lib/src/onnx_qlinear_ops.dart:114). */
ORT_CUDA_API int ort_cuda_gemv_plan_get(ort_cuda_session* s, const char* name, int M, int* plan);
ORT_CUDA_API int ort_cuda_gemv_plan_set(ort_cuda_session* s, const char* name, int M, int plan);

/* MatMulInteger: Y[M x N] (int32) = (A - a_zp) . (B - b_zp) over the
 * uploaded weight `name`, as opMatMulInteger (lib/src/onnx_qlinear_ops.dart:
 * 26-79) computes it (the reference keeps int64; int32 holds every result for
 * K <= 33025, ONNX's int32 output type).  A [M x K] bytes, int8 when
 * a_signed else uint8 (the output of DynamicQuantizeLinear); a_zp of A's type,
 * scalar (a_zp_len 1) or per row (M), or NULL.  A, a_zp and Y are device
 * pointers (stream-ordered) unless ORT_CUDA_HOST_IO is set. */
ORT_CUDA_API int ort_cuda_matmul_integer(ort_cuda_session* s, const char* name, const void* A,
                                         int64_t M, int a_signed, const void* a_zp,
                                         int64_t a_zp_len, int32_t* Y, int flags);

/* DynamicQuantizeLinear (opDynamicQuantizeLinear, lib/src/onnx_ops.dart:
 * 2556-2580) of X[n] fp32: Y[n] uint8, *scale fp32, *zp uint8, with the
 * reference's range, float32 rounding and round-half-even steps (defined for
 * finite X; the reference raises on inf or NaN).  The device half of the int8
 * path ahead of ort_cuda_matmul_integer; all pointers device (stream-ordered)
 * unless ORT_CUDA_HOST_IO is set. */
ORT_CUDA_API int ort_cuda_dynamic_quantize_linear(ort_cuda_session* s, const float* X, int64_t n,
                                                  uint8_t* Y, float* scale, uint8_t* zp,
                                                  int flags);

/* ArgMax (or, with ORT_CUDA_ARG_MIN, ArgMin) over the last axis of X, a
 * [rows x cols] fp32 matrix with row stride ldx: out[r] is the int64 index
 * the reference's opArgMinMax (lib/src/onnx_ops.dart:2198-2237) gives for
 * row r — ties to the first index (the last with ORT_CUDA_ARG_SELECT_LAST),
 * a NaN selected only when it is the row's first element.  Replaces the
 * body of an `ArgMax` node whose input is on the device (the lm_head logits
 * of a greedy decode step), so a step reads back rows x 8 bytes instead of
 * the logits.  X and out are device pointers (stream-ordered) unless
 * ORT_CUDA_HOST_IO is set.  Other axes: move the axis last first. */
ORT_CUDA_API int ort_cuda_argmax(ort_cuda_session* s, const float* X, int64_t rows, int64_t cols,
                                 int64_t ldx, int64_t* out, int flags);

/* ---- attention of a decoder step --------------------------------------
 * fp32 on the device (exact mode's rounding: fp32 dot products, expf, the
 * reference's double scale step); the device counterparts of the
 * reference's GroupQueryAttention, MultiHeadAttention, fused SDPA and
 * RotaryEmbedding cases of OnnxGraphExecutor._dispatch
 * (lib/src/onnx_graph.dart:978-1005, :1029-1033).  Head sizes up to 128.
 * All pointers are device pointers (stream-ordered) unless ORT_CUDA_HOST_IO
 * is set.  `scale` <= 0 selects 1/sqrt(head_size) (GQA and MHA). */
#define ORT_CUDA_ROTARY 0x80              /* GQA do_rotary=1                   */
#define ORT_CUDA_ROTARY_INTERLEAVED 0x200 /* rotary_interleaved / interleaved=1 */
#define ORT_CUDA_ROTARY_BHSD 0x400        /* RotaryEmbedding X is [b, h, s, d]  */

/* GroupQueryAttention (opGroupQueryAttention, lib/src/onnx_ops.dart:
 * 1507-1650): Q [batch, seq, num_heads*head], K/V [batch, seq,
 * kv_num_heads*head], past K/V [batch, kv_num_heads, past_len, head] (NULL
 * when past_len is 0); with ORT_CUDA_ROTARY, RoPE from cos/sin caches
 * [max_pos, rotary_half] at positions past_len..past_len+seq-1 (GPT-J pairs
 * with ORT_CUDA_ROTARY_INTERLEAVED); query token i attends to keys
 * 0..past_len+i, plus bias [bias_batch (1 or batch), bias_heads, seq,
 * past_len+seq] (head h reads bias head h % bias_heads) or NULL.  Writes out
 * [batch, seq, num_heads*head] and, unless both are NULL, present K/V
 * [batch, kv_num_heads, past_len+seq, head] = past then this step's (roped)
 * K and V.  kv_capacity > 0 (device buffers): past and present rows are
 * kv_capacity apart, and present may be the past buffer itself (only this
 * step's rows are then written: an in-place KV cache).  softcap and
 * local_window_size are not supported (the reference raises too). */
ORT_CUDA_API int ort_cuda_group_query_attention(
    ort_cuda_session* s, const float* Q, const float* K, const float* V, const float* past_key,
    const float* past_value, int64_t batch, int64_t seq, int64_t past_len, int num_heads,
    int kv_num_heads, int64_t head_size, double scale, const float* cos_cache,
    const float* sin_cache, int64_t rotary_half, int64_t max_pos, const float* bias,
    int64_t bias_batch, int64_t bias_heads, int64_t kv_capacity, float* out, float* present_key,
    float* present_value, int flags);

/* MultiHeadAttention (opMultiHeadAttention, lib/src/onnx_ops.dart:
 * 1656-1725): Q [batch, seq, hidden], K/V [batch, kv_seq, hidden], no causal
 * mask, optional bias [bias_batch, bias_heads, seq, kv_seq]; out [batch,
 * seq, hidden]. */
ORT_CUDA_API int ort_cuda_multi_head_attention(ort_cuda_session* s, const float* Q,
                                               const float* K, const float* V, int64_t batch,
                                               int64_t seq, int64_t kv_seq, int num_heads,
                                               int64_t hidden, double scale, const float* bias,
                                               int64_t bias_batch, int64_t bias_heads, float* out,
                                               int flags);

/* _FusedSDPA (opFusedSDPA, lib/src/onnx_ops.dart:1733-1774; the
 * MatMul -> Div/Mul -> Add -> Softmax -> MatMul pattern that
 * onnx_graph.dart:332-386 fuses): out = softmax(A.B * scale + mask) . V with
 * A [n0, n1, seq, head], B [n0, n1, head, kv_seq] (K already transposed),
 * V [n0, n1, kv_seq, v_head]; mask element (i0, i1, r, c) at
 * mask[i0*ms[0] + i1*ms[1] + r*ms[2] + c*ms[3]] (stride 0 broadcasts; the
 * host array mask_strides holds ms), or mask NULL. */
ORT_CUDA_API int ort_cuda_fused_sdpa(ort_cuda_session* s, const float* A, const float* B,
                                     const float* V, const float* mask,
                                     const int64_t* mask_strides, int64_t n0, int64_t n1,
                                     int64_t seq, int64_t kv_seq, int64_t head_size,
                                     int64_t v_head_size, double scale, float* out, int flags);

/* RotaryEmbedding (opRotaryEmbedding, lib/src/onnx_ops.dart:2121-2172): X
 * [batch, seq, heads*head] (or [batch, heads, seq, head] with
 * ORT_CUDA_ROTARY_BHSD), int64 position_ids [batch, seq] (pos_per_batch 1)
 * or [seq] shared, cos/sin [max_pos, rotary_half]; the first rotary_dim
 * features of each head (0: 2*rotary_half) are rotated, the rest copied.
 * A position outside [0, max_pos) yields NaN for that row (the reference
 * raises). */
ORT_CUDA_API int ort_cuda_rotary_embedding(ort_cuda_session* s, const float* X,
                                           const int64_t* position_ids, int pos_per_batch,
                                           const float* cos_cache, const float* sin_cache,
                                           int64_t max_pos, int64_t rotary_half, int64_t batch,
                                           int64_t seq, int64_t heads, int64_t head_size,
                                           int64_t rotary_dim, float* Y, int flags);

/* TopK (opTopK, lib/src/onnx_ops.dart:2261-2303) over the last axis of X,
 * a [rows x cols] fp32 matrix with row stride ldx: values[r][0..k) and
 * indices[r][0..k) (int64) in the reference's order -- value descending
 * (ascending with ORT_CUDA_TOPK_SMALLEST), ties to the smaller index, NaN
 * ranked above every number, -0.0 equal to 0.0.  1 <= k <= min(cols, 1024);
 * rows above 40960 columns are split into segments of at most 40960
 * columns, at most floor(4096 / k) of them, so such rows also need
 * cols <= 40960 * floor(4096 / k) (a 128256-column vocabulary takes every
 * k <= 1024, a 256000-column one k <= 585); beyond that the call returns
 * ORT_CUDA_ERR_UNSUPPORTED.  Among equal NaNs the smaller index comes first
 * (the reference's sort leaves that order unspecified).
 * The candidates of top-k sampling after lm_head stay on the device.  All
 * pointers device (stream-ordered) unless ORT_CUDA_HOST_IO is set. */
#define ORT_CUDA_TOPK_SMALLEST 0x800
ORT_CUDA_API int ort_cuda_topk(ort_cuda_session* s, const float* X, int64_t rows, int64_t cols,
                               int64_t ldx, int64_t k, float* values, int64_t* indices, int flags);

/* MatMulNBits followed by ArgMax (ArgMin with ORT_CUDA_ARG_MIN; ties to
 * the last index with ORT_CUDA_ARG_SELECT_LAST) over the last axis of its
 * output: the greedy step after lm_head, fused.  The reference runs the two
 * nodes one after the other (opMatMulNBits, onnx_qlinear_ops.dart:114-156,
 * then opArgMinMax, onnx_ops.dart:2198-2237, on the last-token logits of
 * the lastTokenLogits rewrite, onnx_graph.dart:407-470); here, on one GPU
 * and in the non-STRICT modes for M <= 64, every value the decode GEMV
 * stores also enters a per-row (value, index) key, CTAs fold their keys
 * with atomics and the last CTA writes the indices, so no separate pass
 * re-reads the logits.  Otherwise (N-sharded sessions, STRICT, larger M)
 * the call runs the two operations in turn; the indices are the same
 * either way: those of ort_cuda_argmax on this call's logits.
 *   indices  [M] int64 (device, or host with ORT_CUDA_HOST_IO)
 *   Y        the [M x N] logits, or NULL when the caller does not want them
 * flags: ORT_CUDA_HOST_IO, ORT_CUDA_FLAGS_MODE(m), ORT_CUDA_ARG_MIN,
 * ORT_CUDA_ARG_SELECT_LAST.  The first fused call of a session sets up a
 * small key buffer; make it before capturing a CUDA graph. */
ORT_CUDA_API int ort_cuda_matmul_nbits_argmax(ort_cuda_session* s, const char* name,
                                              const float* A, int64_t M, int64_t* indices,
                                              float* Y, int flags);

/* Sibling MatMulNBits nodes that read the same input (q, k, v of an
 * attention block; gate and up of a SwiGLU MLP) are separate nodes in the
 * reference's graph (opMatMulNBits per node, onnx_graph.dart:1584-1596).
 * ort_cuda_fuse_nbits makes one weight `fused` whose output columns are
 * the parts' columns side by side (2 .. 4 parts with the same K, block
 * size, zero-point presence and scale type, already uploaded); with
 * ORT_CUDA_FUSE_DROP_PARTS the parts are freed, else they stay usable
 * alone (their memory is then held twice).  On an N-sharded session the
 * group is only recorded (the parts stay, ORT_CUDA_FUSE_DROP_PARTS has no
 * effect): the group call then runs the parts in turn.
 * ort_cuda_matmul_nbits_group runs the whole group as one operation and
 * writes part i's [M x N_i] output to Ys[i]: on one GPU at decode sizes one
 * GEMV launch streams every part's weights, so the fixed cost of a launch
 * (dependency release, activation build, first MMA, sums) is paid once for
 * the group.  Each part's result is bit for bit the one
 * ort_cuda_matmul_nbits gives for that part.  Ys[] holds DEVICE pointers,
 * or host pointers with ORT_CUDA_HOST_IO (then A is a host pointer too);
 * ort_cuda_matmul_nbits(s, fused, ...) gives the side-by-side [M x N]. */
#define ORT_CUDA_FUSE_DROP_PARTS 0x1
ORT_CUDA_API int ort_cuda_fuse_nbits(ort_cuda_session* s, const char* fused,
                                     const char* const* names, int n, int flags);
ORT_CUDA_API int ort_cuda_matmul_nbits_group(ort_cuda_session* s, const char* fused,
                                             const float* A, int64_t M, float* const* Ys,
                                             int flags);

/* _SliceLastSeq (onnx_graph.dart:456-473, inserted before the vocab
 * projection by the lastTokenLogits rewrite, :398-451): Y[o][i] =
 * X[o][seq-1][i] for X [outer][seq][inner], device pointers (a strided copy
 * on the session stream), so that lm_head runs on the last position of a
 * device-resident prefill. */
ORT_CUDA_API int ort_cuda_slice_last_seq(ort_cuda_session* s, const float* X, int64_t outer,
                                         int64_t seq, int64_t inner, float* Y, int flags);

/* Kernel launches issued by this session since it was opened (all of
 * them this library's own kernels; a graph launch counts the kernels it
 * holds). */
ORT_CUDA_API int ort_cuda_launch_count(ort_cuda_session* s, int64_t* count);

/* ---- per-op-type profile --------------------------------------------- */
/* The device-side counterpart of ExecutionProfile (onnx_graph.dart:22-47):
 * while enabled, every call of an op entry point records a CUDA event pair
 * on the session stream around its work, under its ONNX op type
 * ("MatMulNBits", "Gemm", "MatMul", "MatMulInteger", "GroupQueryAttention",
 * "TopK", ...).  Events between kernels end their programmatic overlap, so
 * a profiled sequence runs somewhat slower; calls captured into a CUDA
 * graph are not recorded.  Enabling keeps earlier totals; reset clears
 * them (both synchronise the session stream). */
ORT_CUDA_API int ort_cuda_profile_enable(ort_cuda_session* s, int on);
ORT_CUDA_API int ort_cuda_profile_reset(ort_cuda_session* s);
/* Entry `index` of the report, sorted by cumulative device time, longest
 * first (ExecutionProfile.report's order): op type (NUL-terminated,
 * truncated to op_type_cap), call count and device microseconds.
 * Synchronises the session stream; ORT_CUDA_ERR_NOT_FOUND past the end. */
ORT_CUDA_API int ort_cuda_profile_read(ort_cuda_session* s, int index, char* op_type,
                                       int op_type_cap, int64_t* calls, double* device_us);

/* ---- diagnostics ------------------------------------------------------ */
/* Measured fp32 FFMA throughput (TFLOP/s) of the session's GPU, the
 * CUDA-core roofline of the exact and strict modes' dense Gemm/MatMul.  No
 * counterpart in the reference.  Runs one probe kernel for a few ms. */
ORT_CUDA_API int ort_cuda_probe_ffma(ort_cuda_session* s, double* tflops);

#ifdef __cplusplus
}
#endif
#endif /* ORT_CUDA_H_ */
