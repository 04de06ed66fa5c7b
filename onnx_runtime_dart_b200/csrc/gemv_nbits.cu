// int4 block-quantised GEMV for decode (M <= 4), exact fp32 (FFMA) mode.
//
// Replaces, for small M, the reference's per-call dequantisation of all of
// B into an fp32 [K x N] buffer followed by matmulKernel's _gemv
// (onnx_qlinear_ops.dart:127-154, gemm_kernel_simd.dart:183-246).  B stays
// packed in HBM and is streamed exactly once.
//
// Structure: a persistent, warp-specialised kernel, one CTA per SM.
//   * Work item = 32 output columns x 1024 k (16 KB of packed B).  Items are
//     dealt round-robin to the CTAs; a column tile's items sit next to each
//     other so its k-chunks run concurrently.
//   * One producer thread streams each item's B tile (TMA 2-D box, 32 rows
//     of 512 bytes) and the matching 1024-k chunk of each A row (TMA, 128-byte
//     swizzle) into a ring of shared-memory stages guarded by mbarriers.
//   * Eight consumer warps each own 4 of the 32 columns.  Lane l owns the 32
//     k values [32l, 32l+32) of the chunk: one 16-byte shared load per column,
//     eight conflict-free 16-byte loads of A per row (the swizzle spreads the
//     lanes' 128-byte strided rows over all banks).
//   * Reduction order is fixed and depends on K only: 32 lanes by butterfly
//     shuffle, then the K/1024 chunk partials in chunk order by the last CTA
//     to finish a column tile (a self-resetting arrival counter).  A column's
//     rounding therefore never depends on N or on which columns a GPU owns:
//     N-sharded results equal 1-GPU results bit for bit.
//
// Arithmetic per weight.  A nibble q at bit p of a 32-bit word (p in
// {0,4,8,12,16}) becomes the fp32 value 2^(23-p) + q with one LOP3 (mask,
// OR the exponent of 2^(23-p)); subtracting 2^(23-p) + zp is exact (same
// binade) and gives q - zp.  Nibbles at bits 20..28 are shifted down by 12
// first.  Packed add.rn.f32x2 forms the differences, packed fma.rn.f32x2
// accumulates them against pairs of A, and each lane's 32-k partial is
// scaled once:  y += scale[n, blk] * sum_k a_k * (q_k - zp).  This differs
// from the reference's per-element fl((q-zp)*scale) only by fp32
// reassociation, well inside the 1e-5 max-relative budget.
#include "common.cuh"
#include "ptx.cuh"

namespace ortc {
namespace {

__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1,%2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ float lo2(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi2(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// 2^(23-p) + q for the nibble at bit p (p <= 16).
template <int P>
__device__ __forceinline__ float nib(uint32_t w) {
  return __uint_as_float((w & (0xFu << P)) | ((150u - P) << 23));
}

// Packed subtrahends of one word: nibble i -> 2^(23-p_i) + zp, p = 0,4,8,
// 12,16 for nibbles 0..4 and 8,12,16 for nibbles 5..7.
struct Sub4 {
  uint64_t s01, s23, s45, s67;
};
__device__ __forceinline__ Sub4 make_sub(float z) {
  const uint64_t zz = pk2(-z, -z);
  Sub4 r;
  r.s01 = fadd2(pk2(-8388608.0f, -524288.0f), zz);
  r.s23 = fadd2(pk2(-32768.0f, -2048.0f), zz);
  r.s45 = fadd2(pk2(-128.0f, -32768.0f), zz);
  r.s67 = fadd2(pk2(-2048.0f, -128.0f), zz);
  return r;
}

// acc[m] += a[m][0..7] . (q - zp)[0..7] for one packed word.
template <int MR>
__device__ __forceinline__ void word_fma(uint32_t w, const Sub4& sub, const float4 (&a)[MR][2],
                                         uint64_t (&acc)[MR]) {
  const uint32_t w2 = w >> 12;
  const uint64_t x01 = fadd2(pk2(nib<0>(w), nib<4>(w)), sub.s01);
  const uint64_t x23 = fadd2(pk2(nib<8>(w), nib<12>(w)), sub.s23);
  const uint64_t x45 = fadd2(pk2(nib<16>(w), nib<8>(w2)), sub.s45);
  const uint64_t x67 = fadd2(pk2(nib<12>(w2), nib<16>(w2)), sub.s67);
#pragma unroll
  for (int m = 0; m < MR; m++) {
    acc[m] = ffma2(pk2(a[m][0].x, a[m][0].y), x01, acc[m]);
    acc[m] = ffma2(pk2(a[m][0].z, a[m][0].w), x23, acc[m]);
    acc[m] = ffma2(pk2(a[m][1].x, a[m][1].y), x45, acc[m]);
    acc[m] = ffma2(pk2(a[m][1].z, a[m][1].w), x67, acc[m]);
  }
}

__device__ __forceinline__ float zp_at(const uint8_t* __restrict__ Z, int64_t zi) {
  const uint32_t byte = __ldg(Z + (zi >> 1));
  return (float)((byte >> ((zi & 1) * 4)) & 0xFu);
}

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileCols = 32;       // columns per work item
constexpr int kCols = kTileCols / kConsumerWarps;  // columns per consumer warp
constexpr int kChunk = 1024;        // k per work item
constexpr uint32_t kBBytes = kTileCols * kChunk / 2;  // 16 KB
constexpr uint32_t kARowBytes = kChunk * 4;           // 4 KB per A row

struct GemvParams {
  const float* S;
  const uint8_t* Z;
  float* Y;
  float* part;      // [nch][MR][tiles*32] chunk partials (nch > 1)
  unsigned* cnt;    // [tiles * kConsumerWarps] arrival counters (nch > 1)
  int* err;
  int64_t ldy;
  int N, K, nb, bs_log2, stages;
};

template <int MR, bool HAS_ZP, bool BS16>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmA, const GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Stage layout: [A rows: MR x 4 KB][B: 16 KB]; 1024-aligned for the swizzle.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr uint32_t kStageBytes = MR * kARowBytes + kBBytes;
  const int stages = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * kStageBytes);
  uint64_t* empty = full + stages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.N + kTileCols - 1) / kTileCols;
  const int nch = (p.K + kChunk - 1) / kChunk;
  const int total = tiles * nch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbarrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmB);
      prefetch_tensormap(&tmA);
      const uint64_t pol = policy_evict_first();
      const int rows_per_m = p.K / 32;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int armed[8];  // parity each stage was last armed with (-1: never)
      for (int s = 0; s < 8; s++) armed[s] = -1;
      for (int it = blockIdx.x; it < total; it += gridDim.x) {
        const int tile = it / nch, ch = it - tile * nch;
        if (!mbar_wait(&empty[stage], phase ^ 1)) {
          record_error(p.err, KERR_WAIT_EMPTY);
          ok = false;
          break;
        }
        uint8_t* st = smem + stage * kStageBytes;
        armed[stage] = (int)phase;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
#pragma unroll
        for (int m = 0; m < MR; m++)
          tma_load_2d(st + m * kARowBytes, &tmA, &full[stage], 0, m * rows_per_m + ch * 32);
        tma_load_2d_hint(st + MR * kARowBytes, &tmB, &full[stage], ch * (kChunk / 8),
                         tile * kTileCols, pol);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA exits.
        for (int s = 0; s < stages; s++)
          if (armed[s] >= 0 && !mbar_wait(&full[s], (uint32_t)armed[s]))
            record_error(p.err, KERR_WAIT_DRAIN);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  int stage = 0;
  uint32_t phase = 0;
  const int colw = warp * kCols;  // this warp's first column within a tile
  for (int it = blockIdx.x; it < total; it += gridDim.x) {
    const int tile = it / nch, ch = it - tile * nch;
    if (!mbar_wait(&full[stage], phase)) {
      record_error(p.err, KERR_WAIT_FULL);
      return;
    }
    const uint32_t sA = smem_u32(smem + stage * kStageBytes);
    const uint32_t sB = sA + MR * kARowBytes;
    const int kb = ch * kChunk + lane * 32;
    const int col0 = tile * kTileCols + colw;
    float y[kCols][MR];
#pragma unroll
    for (int c = 0; c < kCols; c++)
#pragma unroll
      for (int m = 0; m < MR; m++) y[c][m] = 0.0f;

    if (kb < p.K) {
      const int blk = kb >> p.bs_log2;
      uint64_t acc[kCols][MR];
#pragma unroll
      for (int c = 0; c < kCols; c++)
#pragma unroll
        for (int m = 0; m < MR; m++) acc[c][m] = 0ull;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        // A[m][kb + 16h .. +16): swizzled 16-byte chunks 4h..4h+3 of row `lane`
        float4 a0[MR][2], a1[MR][2];
#pragma unroll
        for (int m = 0; m < MR; m++) {
          const uint32_t rowA = sA + m * kARowBytes + lane * 128;
          a0[m][0] = lds128f(rowA + (((4 * h + 0) ^ (lane & 7)) << 4));
          a0[m][1] = lds128f(rowA + (((4 * h + 1) ^ (lane & 7)) << 4));
          a1[m][0] = lds128f(rowA + (((4 * h + 2) ^ (lane & 7)) << 4));
          a1[m][1] = lds128f(rowA + (((4 * h + 3) ^ (lane & 7)) << 4));
        }
#pragma unroll
        for (int c = 0; c < kCols; c++) {
          const int col = col0 + c;
          const bool ok = col < p.N;
          const int64_t sb = (int64_t)(ok ? col : 0) * p.nb + blk + (BS16 ? h : 0);
          const Sub4 sub = make_sub(HAS_ZP ? (ok ? zp_at(p.Z, sb) : 0.0f) : 8.0f);
          const uint4 w = lds128(sB + (colw + c) * 512 + lane * 16);
          word_fma<MR>(h == 0 ? w.x : w.z, sub, a0, acc[c]);
          word_fma<MR>(h == 0 ? w.y : w.w, sub, a1, acc[c]);
          if (BS16 || h == 1) {
            const float s = ok ? __ldg(p.S + sb) : 0.0f;
#pragma unroll
            for (int m = 0; m < MR; m++) {
              y[c][m] = fmaf(s, lo2(acc[c][m]) + hi2(acc[c][m]), y[c][m]);
              acc[c][m] = 0ull;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1;
    }

    // Fixed-order lane reduction; lane (c*MR + m) ends up owning y[c][m].
    float mine = 0.0f;
#pragma unroll
    for (int c = 0; c < kCols; c++)
#pragma unroll
      for (int m = 0; m < MR; m++) {
        float v = y[c][m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == c * MR + m) mine = v;
      }
    const int oc = lane / MR, om = lane % MR;
    const int ocol = col0 + oc;
    const bool owner = lane < kCols * MR && ocol < p.N;
    if (nch == 1) {
      if (owner) p.Y[om * p.ldy + ocol] = mine;
      continue;
    }
    const int64_t npad = (int64_t)tiles * kTileCols;
    if (owner) p.part[((int64_t)ch * MR + om) * npad + ocol] = mine;
    __threadfence();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) {
      const unsigned old = atomicAdd(&p.cnt[tile * kConsumerWarps + warp], 1u);
      last = (old == (unsigned)(nch - 1));
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      if (owner) {
        float v = 0.0f;
        for (int c2 = 0; c2 < nch; c2++) v += __ldcg(p.part + ((int64_t)c2 * MR + om) * npad + ocol);
        p.Y[om * p.ldy + ocol] = v;
      }
      if (lane == 0) p.cnt[tile * kConsumerWarps + warp] = 0u;
    }
  }
}

template <int MR, bool ZP, bool B16>
int launch_t(const CUtensorMap& tmB, const CUtensorMap& tmA, const GemvParams& prm, int grid,
             size_t smem, cudaStream_t st) {
  auto kern = gemv_tma_kernel<MR, ZP, B16>;
  static unsigned long long configured = 0;  // one attribute call per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    ORTC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    configured |= 1ull << (dev & 63);
  }
  kern<<<grid, kThreads, smem, st>>>(tmB, tmA, prm);
  ORTC_CUDA(cudaGetLastError());
  return ORT_CUDA_OK;
}

template <int MR>
int launch_mr(const CUtensorMap& tmB, const CUtensorMap& tmA, const GemvParams& prm, bool zp,
              bool b16, int grid, size_t smem, cudaStream_t st) {
  if (zp) return b16 ? launch_t<MR, true, true>(tmB, tmA, prm, grid, smem, st)
                     : launch_t<MR, true, false>(tmB, tmA, prm, grid, smem, st);
  return b16 ? launch_t<MR, false, true>(tmB, tmA, prm, grid, smem, st)
             : launch_t<MR, false, false>(tmB, tmA, prm, grid, smem, st);
}

}  // namespace

size_t gemv_partial_floats(int64_t K, int64_t nl, int64_t M) {
  const int64_t nch = (K + kChunk - 1) / kChunk;
  if (nch <= 1) return 0;
  const int64_t tiles = (nl + kTileCols - 1) / kTileCols;
  return (size_t)(nch * M * tiles * kTileCols);
}

size_t gemv_counter_words(int64_t K, int64_t nl) {
  const int64_t nch = (K + kChunk - 1) / kChunk;
  if (nch <= 1) return 0;
  return (size_t)(((nl + kTileCols - 1) / kTileCols) * kConsumerWarps);
}

// Preconditions (checked by the dispatcher): 1 <= M <= 4, K % 32 == 0,
// A 16-byte aligned with row stride K, block size >= 16.  `partials` holds
// gemv_partial_floats() floats; `counters` gemv_counter_words() words that
// are zero on entry (the kernel leaves them zero again).
int launch_nbits_gemv(const Weight& w, const float* A, int64_t M, float* Y, int64_t ldy,
                      float* partials, unsigned* counters, int* err, int sm_count,
                      cudaStream_t st, int64_t* launches) {
  if (w.nl == 0) return ORT_CUDA_OK;
  CUtensorMap tmA;
  int rc = encode_tma_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, A, 32, (uint64_t)(M * w.K / 32),
                         128, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  GemvParams prm;
  prm.S = w.scales;
  prm.Z = w.zp;
  prm.Y = Y;
  prm.err = err;
  prm.ldy = ldy;
  prm.N = (int)w.nl;
  prm.K = (int)w.K;
  prm.nb = w.nb;
  int bl = 0;
  while ((1 << bl) < w.bs) bl++;
  prm.bs_log2 = bl;
  const int64_t nch = (w.K + kChunk - 1) / kChunk;
  const int64_t tiles = (w.nl + kTileCols - 1) / kTileCols;
  prm.part = nch > 1 ? partials : nullptr;
  prm.cnt = nch > 1 ? counters : nullptr;
  const size_t stage_bytes = (size_t)M * kARowBytes + kBBytes;
  int stages = (int)((200 * 1024) / stage_bytes);
  if (stages > 8) stages = 8;
  prm.stages = stages;
  const size_t smem = 1024 + stages * stage_bytes + 2 * stages * sizeof(uint64_t);
  const int64_t total = tiles * nch;
  const int grid = (int)(total < sm_count ? total : sm_count);
  const bool zp = w.has_zp, b16 = w.bs == 16;
  switch (M) {
    case 1: rc = launch_mr<1>(w.tmB, tmA, prm, zp, b16, grid, smem, st); break;
    case 2: rc = launch_mr<2>(w.tmB, tmA, prm, zp, b16, grid, smem, st); break;
    case 3: rc = launch_mr<3>(w.tmB, tmA, prm, zp, b16, grid, smem, st); break;
    case 4: rc = launch_mr<4>(w.tmB, tmA, prm, zp, b16, grid, smem, st); break;
    default: return fail(ORT_CUDA_ERR_INVALID_ARG, "gemv: M out of range");
  }
  if (rc == ORT_CUDA_OK) (*launches)++;
  return rc;
}

}  // namespace ortc
