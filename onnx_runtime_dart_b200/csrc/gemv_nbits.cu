// int4 block-quantised GEMV for decode (M <= 4), exact fp32 (FFMA) mode.
//
// Replaces, for small M, the reference's per-call dequantisation of all of
// B into an fp32 [K x N] buffer followed by matmulKernel's _gemv
// (onnx_qlinear_ops.dart:127-154, gemm_kernel_simd.dart:183-246).  Here B
// stays packed in HBM and is streamed exactly once.
//
// Work decomposition.  B is stored as the reference receives it:
// [N][K/2] bytes, column n's nibbles contiguous (low nibble = even k).  A
// lane owns 32-k "chunks" (one 16-byte load per column); a warp covers
// 1024 k of CPW columns per step, so each warp-wide load instruction moves
// 512 contiguous bytes of one column.  The WG warps of a column group split
// the 1024-k steps round-robin; WG depends on K only, so a column's
// arithmetic (and its fp32 rounding) never depends on N or on which
// columns a GPU owns — N-sharded results are bitwise equal to 1-GPU ones.
//
// Arithmetic per weight.  A nibble q at bit position p of a 32-bit word
// (p in {0,4,8,12,16}) becomes the fp32 value 2^(23-p) + q with one LOP3
// (mask, then OR the exponent of 2^(23-p)); subtracting 2^(23-p) + zp is
// exact (same binade), giving x = q - zp exactly.  Nibbles at bits 20..28
// are shifted down by 12 first.  Pairs of x are formed with packed
// add.rn.f32x2 and accumulated with packed fma.rn.f32x2 against pairs of
// A, so a weight costs about 1.75 issue slots at M = 1.  The per-block
// scale multiplies the block partial sum once:
//     y += scale[n, blk] * sum_{k in chunk} a_k * (q_k - zp)
// which differs from the reference's fl((q-zp)*scale) per element only by
// fp32 reassociation (well inside the 1e-5 max-relative budget).
#include "common.cuh"

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

// Streaming 16-byte load: read once, keep it out of L1 (A lives there).
__device__ __forceinline__ uint4 ld_stream16(const uint8_t* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

// 2^(23-p) + q for the nibble at bit p (p <= 16).
template <int P>
__device__ __forceinline__ float nib(uint32_t w) {
  return __uint_as_float((w & (0xFu << P)) | ((150u - P) << 23));
}

// The four packed subtrahends of one word: nibble i -> 2^(23-p_i) + zp with
// p = 0,4,8,12,16 for nibbles 0..4 and 8,12,16 for nibbles 5..7.
struct Sub4 {
  uint64_t s01, s23, s45, s67;
};
__device__ __forceinline__ Sub4 make_sub(float z) {
  Sub4 r;
  r.s01 = pk2(-(8388608.0f + z), -(524288.0f + z));
  r.s23 = pk2(-(32768.0f + z), -(2048.0f + z));
  r.s45 = pk2(-(128.0f + z), -(32768.0f + z));
  r.s67 = pk2(-(2048.0f + z), -(128.0f + z));
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

constexpr int kWarps = 8;

template <int MR, int CPW, bool HAS_ZP, bool BS16>
__global__ void __launch_bounds__(kWarps * 32)
    gemv_nbits_kernel(const float* __restrict__ A, int64_t lda, const uint8_t* __restrict__ B,
                      int64_t col_bytes, const float* __restrict__ S, int nb, int bs_log2,
                      const uint8_t* __restrict__ Z, float* __restrict__ Y, int64_t ldy, int N,
                      int K, int WG) {
  __shared__ float red[kWarps][CPW * MR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int CG = kWarps / WG;
  const int g = warp / WG, wi = warp % WG;
  const int col0 = (blockIdx.x * CG + g) * CPW;
  const int nchunks = (K + 1023) >> 10;

  float y[CPW][MR];
#pragma unroll
  for (int c = 0; c < CPW; c++)
#pragma unroll
    for (int m = 0; m < MR; m++) y[c][m] = 0.0f;

  bool colok[CPW];
#pragma unroll
  for (int c = 0; c < CPW; c++) colok[c] = (col0 + c) < N;

  uint4 cur[CPW], nxt[CPW];
  auto load_chunk = [&](int ci, uint4(&dst)[CPW]) {
    const int kb = (ci << 10) + (lane << 5);
#pragma unroll
    for (int c = 0; c < CPW; c++) {
      if (colok[c] && kb < K)
        dst[c] = ld_stream16(B + (int64_t)(col0 + c) * col_bytes + (kb >> 1));
      else
        dst[c] = make_uint4(0, 0, 0, 0);
    }
  };
  if (wi < nchunks) load_chunk(wi, cur);

  for (int ci = wi; ci < nchunks; ci += WG) {
    if (ci + WG < nchunks) load_chunk(ci + WG, nxt);
    const int kb = (ci << 10) + (lane << 5);
    if (kb < K) {
      const int blk = kb >> bs_log2;
      float s[CPW][BS16 ? 2 : 1];
      Sub4 sub[CPW][BS16 ? 2 : 1];
#pragma unroll
      for (int c = 0; c < CPW; c++) {
        const int64_t sb = (int64_t)(colok[c] ? col0 + c : 0) * nb + blk;
#pragma unroll
        for (int h = 0; h < (BS16 ? 2 : 1); h++) {
          s[c][h] = colok[c] ? __ldg(S + sb + h) : 0.0f;
          sub[c][h] = make_sub(HAS_ZP ? (colok[c] ? zp_at(Z, sb + h) : 0.0f) : 8.0f);
        }
      }
      uint64_t acc[CPW][MR];
#pragma unroll
      for (int c = 0; c < CPW; c++)
#pragma unroll
        for (int m = 0; m < MR; m++) acc[c][m] = 0ull;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        // A[m][kb + 16h .. +16): 16 floats per row, through L1.
        float4 a0[MR][2], a1[MR][2];
#pragma unroll
        for (int m = 0; m < MR; m++) {
          const float4* ap = reinterpret_cast<const float4*>(A + m * lda + kb + 16 * h);
          a0[m][0] = __ldg(ap + 0);
          a0[m][1] = __ldg(ap + 1);
          a1[m][0] = __ldg(ap + 2);
          a1[m][1] = __ldg(ap + 3);
        }
#pragma unroll
        for (int c = 0; c < CPW; c++) {
          const uint32_t wa = h == 0 ? cur[c].x : cur[c].z;
          const uint32_t wb = h == 0 ? cur[c].y : cur[c].w;
          const Sub4& sb = sub[c][BS16 ? h : 0];
          word_fma<MR>(wa, sb, a0, acc[c]);
          word_fma<MR>(wb, sb, a1, acc[c]);
          if (BS16) {
#pragma unroll
            for (int m = 0; m < MR; m++) {
              y[c][m] = fmaf(s[c][h], lo2(acc[c][m]) + hi2(acc[c][m]), y[c][m]);
              acc[c][m] = 0ull;
            }
          }
        }
      }
      if (!BS16) {
#pragma unroll
        for (int c = 0; c < CPW; c++)
#pragma unroll
          for (int m = 0; m < MR; m++)
            y[c][m] = fmaf(s[c][0], lo2(acc[c][m]) + hi2(acc[c][m]), y[c][m]);
      }
    }
#pragma unroll
    for (int c = 0; c < CPW; c++) cur[c] = nxt[c];
  }

  // Fixed-order reduction: butterfly over lanes, then warps in index order.
#pragma unroll
  for (int c = 0; c < CPW; c++)
#pragma unroll
    for (int m = 0; m < MR; m++) {
      float v = y[c][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      y[c][m] = v;
    }
  if (WG == 1) {
    if (lane == 0) {
#pragma unroll
      for (int c = 0; c < CPW; c++)
        if (colok[c])
#pragma unroll
          for (int m = 0; m < MR; m++) Y[m * ldy + col0 + c] = y[c][m];
    }
    return;
  }
  if (lane == 0) {
#pragma unroll
    for (int c = 0; c < CPW; c++)
#pragma unroll
      for (int m = 0; m < MR; m++) red[warp][c * MR + m] = y[c][m];
  }
  __syncthreads();
  if (wi == 0 && lane < CPW * MR) {
    const int c = lane / MR, m = lane % MR;
    float v = red[warp][lane];
    for (int j = 1; j < WG; j++) v += red[warp + j][lane];
    if (col0 + c < N) Y[m * ldy + col0 + c] = v;
  }
}

template <int MR, int CPW>
int launch_mr(const Weight& w, const float* A, float* Y, int64_t ldy, cudaStream_t st) {
  const int K = (int)w.K, N = (int)w.nl;
  const int nchunks = (K + 1023) / 1024;
  int WG = 1;
  while (WG * 2 <= kWarps && WG * 2 <= nchunks) WG *= 2;
  const int cols_per_cta = CPW * (kWarps / WG);
  const int grid = (N + cols_per_cta - 1) / cols_per_cta;
  int bs_log2 = 0;
  while ((1 << bs_log2) < w.bs) bs_log2++;
  const int64_t col_bytes = (int64_t)w.nb * w.bs / 2;
  const bool bs16 = w.bs == 16;
#define ORTC_GEMV_LAUNCH(ZP, B16)                                                           \
  gemv_nbits_kernel<MR, CPW, ZP, B16><<<grid, kWarps * 32, 0, st>>>(                      \
      A, (int64_t)K, w.B, col_bytes, w.scales, w.nb, bs_log2, w.zp, Y, ldy, N, K, WG)
  if (w.has_zp) {
    if (bs16) ORTC_GEMV_LAUNCH(true, true);
    else ORTC_GEMV_LAUNCH(true, false);
  } else {
    if (bs16) ORTC_GEMV_LAUNCH(false, true);
    else ORTC_GEMV_LAUNCH(false, false);
  }
#undef ORTC_GEMV_LAUNCH
  ORTC_CUDA(cudaGetLastError());
  return ORT_CUDA_OK;
}

}  // namespace

// Preconditions (checked by the dispatcher): 1 <= M <= 4, K % 32 == 0,
// A 16-byte aligned with row stride K, block size >= 16.
int launch_nbits_gemv(const Weight& w, const float* A, int64_t M, float* Y, int64_t ldy,
                      cudaStream_t st, int64_t* launches) {
  if (w.nl == 0) return ORT_CUDA_OK;
  int rc;
  switch (M) {
    case 1: rc = launch_mr<1, 4>(w, A, Y, ldy, st); break;
    case 2: rc = launch_mr<2, 4>(w, A, Y, ldy, st); break;
    case 3: rc = launch_mr<3, 2>(w, A, Y, ldy, st); break;
    case 4: rc = launch_mr<4, 2>(w, A, Y, ldy, st); break;
    default: return fail(ORT_CUDA_ERR_INVALID_ARG, "gemv: M out of range");
  }
  if (rc == ORT_CUDA_OK) (*launches)++;
  return rc;
}

}  // namespace ortc
