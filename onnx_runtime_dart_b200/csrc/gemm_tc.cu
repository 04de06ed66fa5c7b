// tcgen05 tensor-core GEMM for the MMA modes (prefill-sized M).
//
//   Y[M, N] = 2^(e_m + f_n) * (A16[M, K] . W16[N, K]^T)   (then Gemm's
//   alpha / beta*C epilogue, onnx_ops.dart:1785-1792)
//
// A16 / W16 are 16-bit K-major copies: f16 with a power-of-two range
// normalisation per A row (e_m) and per weight column (f_n) so that the
// largest magnitude of a row/column lands in [2^14, 2^15) — the scaling is
// exact in fp32 and keeps f16's 11-bit precision away from overflow and
// subnormals — or, in the bf16 mode, a two-term bf16 split of each value
// (hi = bf16(v), lo = bf16(v - hi): 16 significant bits together) stored
// as two planes, hi then lo.  The bf16 product is formed from three MMAs,
// A_hi.W_hi + A_lo.W_hi + A_hi.W_lo (the dropped A_lo.W_lo is below 2^-16
// of the product), so its error is about 2^-16 relative per product
// instead of bf16's 2^-9 — inside the mode's 2e-3 bar with a wide margin —
// at three times the tensor-core work.  A is converted per call
// (one warp per row); dense weights are converted once per session and kept;
// int4 weights are dequantised per call, W = (q - zp) * scale, into a 16-bit
// scratch operand.
//
// Kernel: one CTA per 128 x 256 output tile, 6 warps, warp-specialised.
//   warp 0   TMA producer: A and W 64-k slices (128-byte swizzle) into a
//            4-stage ring (48 KB per stage) guarded by mbarriers
//   warp 1   allocates 256 TMEM columns; one thread issues
//            tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) x 4 per
//            stage, fp32 accumulation in TMEM, and tcgen05.commit frees the
//            stage / signals the epilogue
//   warps 2-5 epilogue: tcgen05.ld of their 32-lane quarter, exact 2^e
//            rescaling, alpha / C, fp32 stores
// Every mbarrier wait is bounded (ptx.cuh); on expiry the kernel records an
// error code, drains its copies and returns.
#include <cuda_bf16.h>

#include <atomic>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace ortc {
namespace {

constexpr int TBM = 128, TBN = 256, TBK = 64;
constexpr uint32_t kABytes = TBM * TBK * 2;            // 16 KB
constexpr uint32_t kBBytes = TBN * TBK * 2;            // 32 KB
constexpr uint32_t kTmemCols = 256;
constexpr int kThreads = 192;
// one plane: 4 stages of A + W (48 KB); split: 2 stages of A_hi, A_lo, W_hi, W_lo (96 KB)
template <bool SPLIT>
struct Ring {
  static constexpr int kStages = SPLIT ? 2 : 4;
  static constexpr uint32_t kStageBytes = (SPLIT ? 2 : 1) * (kABytes + kBBytes);
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 256;
};

struct Epilogue {
  float* Y;
  int64_t ldy;
  int M, N;
  const int* row_exp;  // [M] or null
  const int* col_exp;  // [N] or null
  float alpha, beta;
  const float* C;
  int64_t c_rows, c_cols, c_col0;
  int has_c;
  int* err;
};

__device__ __forceinline__ float pow2f(int e) {
  // 2^e for e in [-126, 127] (callers split larger exponents)
  return __uint_as_float((uint32_t)(e + 127) << 23);
}
__device__ __forceinline__ float scale_pow2(float v, int e) {
  while (e > 100) { v *= pow2f(100); e -= 100; }
  while (e < -100) { v *= pow2f(-100); e += 100; }
  return v * pow2f(e);
}

template <bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    mma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmA2,
                    const __grid_constant__ CUtensorMap tmB2, int K, uint32_t idesc, Epilogue ep) {
  constexpr int kStages = Ring<SPLIT>::kStages;
  constexpr uint32_t kStageBytes = Ring<SPLIT>::kStageBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* accum = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // row tiles vary fastest: CTAs resident together share a weight tile (read
  // from DRAM about once) and re-read A, which stays in L2
  const int m0 = blockIdx.x * TBM, n0 = blockIdx.y * TBN;
  const int nk = (K + TBK - 1) / TBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&tmA);
      prefetch_tensormap(&tmB);
      if (SPLIT) {
        prefetch_tensormap(&tmA2);
        prefetch_tensormap(&tmB2);
      }
      bool ok = true;
      int issued = 0;
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          record_error(ep.err, KERR_WAIT_EMPTY);
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(st, &tmA, &full[s], kb * TBK, m0);
        tma_load_2d(st + kABytes, &tmB, &full[s], kb * TBK, n0);
        if (SPLIT) {  // [A_hi][W_hi][A_lo][W_lo]
          tma_load_2d(st + kABytes + kBBytes, &tmA2, &full[s], kb * TBK, m0);
          tma_load_2d(st + 2 * kABytes + kBBytes, &tmB2, &full[s], kb * TBK, n0);
        }
        issued = kb + 1;
      }
      if (!ok) {
        // wait (bounded) for the copies already issued to land
        for (int kb = (issued > kStages ? issued - kStages : 0); kb < issued; kb++)
          if (!mbar_wait(&full[kb % kStages], (kb / kStages) & 1))
            record_error(ep.err, KERR_WAIT_DRAIN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < nk && ok; kb++) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait(&full[s], ph)) {
          record_error(ep.err, KERR_WAIT_FULL);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kStageBytes);
        const uint32_t sb = sa + kABytes;
#pragma unroll
        for (int kk = 0; kk < TBK / 16; kk++) {
          mma_f16_ss(tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sb + kk * 32), idesc,
                     (kb | kk) != 0);
          if (SPLIT) {
            const uint32_t sa2 = sb + kBBytes, sb2 = sa2 + kABytes;
            mma_f16_ss(tmem, smem_desc_sw128(sa2 + kk * 32), smem_desc_sw128(sb + kk * 32),
                       idesc, true);  // A_lo . W_hi
            mma_f16_ss(tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sb2 + kk * 32),
                       idesc, true);  // A_hi . W_lo
          }
        }
        mma_commit(&empty[s]);
      }
      mma_commit(accum);  // arrives once all issued MMAs are complete
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const bool ok = mbar_wait(accum, 0);
    if (!ok) record_error(ep.err, KERR_WAIT_MMA);
    tc_fence_after();
    if (ok) {
      const int re = (ep.row_exp && row < ep.M) ? ep.row_exp[row] : 0;
      for (int c0 = 0; c0 < TBN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c0, r);
        tmem_ld_wait();
        if (row >= ep.M) continue;
        float* yrow = ep.Y + (int64_t)row * ep.ldy;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int n = n0 + c0 + j;
          if (n >= ep.N) break;
          float v = __uint_as_float(r[j]);
          const int ce = ep.col_exp ? ep.col_exp[n] : 0;
          v = scale_pow2(scale_pow2(v, re), ce);
          if (ep.alpha != 1.0f) v = __fmul_rn(v, ep.alpha);
          if (ep.has_c) {
            const int64_t cn = ep.c_col0 + n;
            float c = ep.C[(ep.c_rows == 1 ? 0 : row) * ep.c_cols + (ep.c_cols == 1 ? 0 : cn)];
            if (ep.beta != 1.0f) c = __fmul_rn(c, ep.beta);
            v = __fadd_rn(v, c);
          }
          yrow[n] = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- operand conversion ----------------------------------------------------

__device__ __forceinline__ int norm_exp(float amax) {
  // exponent e with amax * 2^-e in [2^14, 2^15); 0 for an all-zero / non-finite row
  if (!(amax > 0.0f) || !isfinite(amax)) return 0;
  int ex;
  frexpf(amax, &ex);  // amax = f * 2^ex, f in [0.5, 1)
  return ex - 15;
}

template <bool BF16>
__device__ __forceinline__ uint16_t to16(float v) {
  if (BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}
// The low term of the bf16 split: bf16(v - float(bf16(v))).
__device__ __forceinline__ uint16_t bf16_lo(float v, uint16_t hi) {
  const float h = __uint_as_float((uint32_t)hi << 16);
  return __bfloat16_as_ushort(__float2bfloat16_rn(v - h));
}

// A [M, K] (or [K, M] with transA) fp32 -> 16-bit [M, K] (+ row exponent
// for f16).  One warp per row.
template <bool BF16>
__global__ void a16_kernel(const float* __restrict__ A, int M, int K, bool transA,
                           uint16_t* __restrict__ out, int* __restrict__ row_exp) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int m = warp;
  auto at = [&](int k) { return transA ? A[(int64_t)k * M + m] : A[(int64_t)m * K + k]; };
  int e = 0;
  if (!BF16) {
    float mx = 0.0f;
    for (int k = lane; k < K; k += 32) mx = fmaxf(mx, fabsf(at(k)));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    e = norm_exp(mx);
    if (lane == 0) row_exp[m] = e;
  }
  uint16_t* o = out + (int64_t)m * K;
  uint16_t* lo = out + (int64_t)M * K + (int64_t)m * K;  // bf16: the low plane
  for (int k = lane; k < K; k += 32) {
    const float v = at(k);
    const uint16_t h = to16<BF16>(BF16 ? v : scale_pow2(v, -e));
    o[k] = h;
    if (BF16) lo[k] = bf16_lo(v, h);
  }
}

// The same conversion for row-major A with K % 4 == 0 and a 16-byte
// aligned base: 16-byte loads in both passes, 8-byte stores (same bits).
template <bool BF16>
__global__ void a16_vec_kernel(const float* __restrict__ A, int M, int K,
                               uint16_t* __restrict__ out, int* __restrict__ row_exp) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const float4* row = reinterpret_cast<const float4*>(A + (int64_t)warp * K);
  const int k4 = K / 4;
  int e = 0;
  if (!BF16) {
    float mx = 0.0f;
    for (int i = lane; i < k4; i += 32) {
      const float4 v = __ldg(row + i);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    e = norm_exp(mx);
    if (lane == 0) row_exp[warp] = e;
  }
  uint2* o = reinterpret_cast<uint2*>(out + (int64_t)warp * K);
  uint2* lo = reinterpret_cast<uint2*>(out + (int64_t)M * K + (int64_t)warp * K);
  for (int i = lane; i < k4; i += 32) {
    const float4 v = __ldg(row + i);
    const uint32_t a = to16<BF16>(BF16 ? v.x : scale_pow2(v.x, -e));
    const uint32_t b = to16<BF16>(BF16 ? v.y : scale_pow2(v.y, -e));
    const uint32_t c = to16<BF16>(BF16 ? v.z : scale_pow2(v.z, -e));
    const uint32_t d = to16<BF16>(BF16 ? v.w : scale_pow2(v.w, -e));
    o[i] = make_uint2(a | (b << 16), c | (d << 16));
    if (BF16) {
      const uint32_t la = bf16_lo(v.x, (uint16_t)a), lb = bf16_lo(v.y, (uint16_t)b);
      const uint32_t lc = bf16_lo(v.z, (uint16_t)c), ld = bf16_lo(v.w, (uint16_t)d);
      lo[i] = make_uint2(la | (lb << 16), lc | (ld << 16));
    }
  }
}

// Dense weight [K][nl] fp32 -> 16-bit [nl][K] with per-column exponent.
__global__ void wcol_exp_kernel(const float* __restrict__ W, int K, int nl, int* __restrict__ col_exp) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= nl) return;
  float mx = 0.0f;
  for (int k = 0; k < K; k++) mx = fmaxf(mx, fabsf(W[(int64_t)k * nl + n]));
  col_exp[n] = norm_exp(mx);
}

template <bool BF16>
__global__ void w16_dense_kernel(const float* __restrict__ W, int K, int nl,
                                 const int* __restrict__ col_exp, uint16_t* __restrict__ out) {
  __shared__ float t[32][33];
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    t[i][threadIdx.x] = (k < K && n < nl) ? W[(int64_t)k * nl + n] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (n < nl && k < K) {
      const float v = t[threadIdx.x][i];
      const uint16_t h = to16<BF16>(BF16 ? v : scale_pow2(v, -col_exp[n]));
      out[(int64_t)n * K + k] = h;
      if (BF16) out[(int64_t)nl * K + (int64_t)n * K + k] = bf16_lo(v, h);
    }
  }
}

// int4 weight -> 16-bit [nl][K]: W = (q - zp) * scale (fp32, as the
// reference rounds it), then * 2^-f_n and rounded to 16 bits.
__global__ void nbits_col_exp_kernel(const float* __restrict__ S, int64_t s_pitch, int nb, int nl,
                                     int* __restrict__ col_exp) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= nl) return;
  float mx = 0.0f;
  for (int b = 0; b < nb; b++) mx = fmaxf(mx, fabsf(S[(int64_t)b * s_pitch + n]));
  col_exp[n] = norm_exp(15.0f * mx);
}

template <bool BF16>
__global__ void w16_nbits_kernel(const uint8_t* __restrict__ B, const float* __restrict__ S,
                                 int64_t s_pitch, const uint8_t* __restrict__ Z, int64_t z_pitch,
                                 int K, int nb, int bs, int nl, const int* __restrict__ col_exp,
                                 uint16_t* __restrict__ out) {
  const int64_t col_bytes = (int64_t)nb * bs / 2;
  const int64_t wpc = (K + 7) / 8;  // 32-bit words per column that hold k < K
  const int64_t total = (int64_t)nl * wpc;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / wpc;
    const int k0 = (int)(i % wpc) * 8;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(B + n * col_bytes + k0 / 2);
    const int e = BF16 ? 0 : col_exp[n];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int k = k0 + j;
      if (k >= K) break;
      const int blk = k / bs;
      const float z = Z ? (float)nbits_zp(Z, z_pitch, n, blk) : 8.0f;
      const float w = __fmul_rn((float)nbits_q(word, j) - z, S[(int64_t)blk * s_pitch + n]);
      const uint16_t h = to16<BF16>(BF16 ? w : scale_pow2(w, -e));
      out[n * K + k] = h;
      if (BF16) out[(int64_t)nl * K + n * K + k] = bf16_lo(w, h);
    }
  }
}

int launch_gemm(ort_cuda_session* s, const uint16_t* A16, const int* row_exp, int64_t M,
                const uint16_t* W16, const int* col_exp, int64_t nl, int64_t K, bool bf16,
                float* Y, int64_t ldy, float alpha, float beta, const float* C, int64_t c_rows,
                int64_t c_cols, int64_t c_col0, cudaStream_t st) {
  const CUtensorMapDataType dt =
      bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // bf16: two planes each (hi at A16 / W16, lo one plane later)
  CUtensorMap tmA, tmB, tmA2, tmB2;
  int rc = encode_tma_2d(&tmA, dt, A16, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, TBK, TBM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tma_2d(&tmB, dt, W16, (uint64_t)K, (uint64_t)nl, (uint64_t)K * 2, TBK, TBN,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  tmA2 = tmA;
  tmB2 = tmB;
  if (bf16) {
    rc = encode_tma_2d(&tmA2, dt, A16 + M * K, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, TBK,
                       TBM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tma_2d(&tmB2, dt, W16 + nl * K, (uint64_t)K, (uint64_t)nl, (uint64_t)K * 2, TBK,
                       TBN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Epilogue ep{Y, ldy, (int)M, (int)nl, bf16 ? nullptr : row_exp, bf16 ? nullptr : col_exp,
              alpha, beta, C, c_rows, c_cols, c_col0, C != nullptr, s->err_dev};
  static std::atomic<unsigned long long> configured{0};  // per device, both variants
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load() >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(mma_gemm_kernel<false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)Ring<false>::kSmemBytes));
    ORTC_CUDA(cudaFuncSetAttribute(mma_gemm_kernel<true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)Ring<true>::kSmemBytes));
    if (dev < 64) configured.fetch_or(1ull << dev);
  }
  ORTC_CHECK((nl + TBN - 1) / TBN <= 65535, ORT_CUDA_ERR_UNSUPPORTED,
             "tensor-core GEMM: more than 65535 column tiles");
  dim3 grid((unsigned)((M + TBM - 1) / TBM), (unsigned)((nl + TBN - 1) / TBN));
  if (bf16)
    mma_gemm_kernel<true><<<grid, kThreads, Ring<true>::kSmemBytes, st>>>(
        tmA, tmB, tmA2, tmB2, (int)K, idesc_f16(1, TBM, TBN), ep);
  else
    mma_gemm_kernel<false><<<grid, kThreads, Ring<false>::kSmemBytes, st>>>(
        tmA, tmB, tmA2, tmB2, (int)K, idesc_f16(0, TBM, TBN), ep);
  ORTC_CUDA(cudaGetLastError());
  s->launches++;
  return ORT_CUDA_OK;
}

size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Converts A into kscratch: returns pointers to the 16-bit copy and the row
// exponents placed at `off` bytes into the scratch.
int convert_a(ort_cuda_session* s, const float* A, int64_t M, int64_t K, bool transA, bool bf16,
              size_t off, uint16_t** A16, int** row_exp, cudaStream_t st) {
  char* base = (char*)s->kscratch + off;
  *A16 = (uint16_t*)base;
  *row_exp = (int*)(base + al256((size_t)(M * K) * 2 * (bf16 ? 2 : 1)));
  const int64_t threads = M * 32;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  const bool vec = !transA && K % 4 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
  if (vec && bf16)
    a16_vec_kernel<true><<<blocks, 256, 0, st>>>(A, (int)M, (int)K, *A16, *row_exp);
  else if (vec)
    a16_vec_kernel<false><<<blocks, 256, 0, st>>>(A, (int)M, (int)K, *A16, *row_exp);
  else if (bf16)
    a16_kernel<true><<<blocks, 256, 0, st>>>(A, (int)M, (int)K, transA, *A16, *row_exp);
  else
    a16_kernel<false><<<blocks, 256, 0, st>>>(A, (int)M, (int)K, transA, *A16, *row_exp);
  ORTC_CUDA(cudaGetLastError());
  s->launches++;
  return ORT_CUDA_OK;
}

size_t a_scratch_bytes(int64_t M, int64_t K, bool bf16 = false) {
  return al256((size_t)(M * K) * 2 * (bf16 ? 2 : 1)) + al256((size_t)M * 4);
}

}  // namespace

// Shapes the tensor-core path takes: TMA needs 16-byte row strides of the
// 16-bit operands (K % 8 == 0); below M = 64 the decode kernels are used.
int mma_supported_shape(int64_t M, int64_t K) {
  return M >= 64 && K >= 16 && (K % 8) == 0 && M < (int64_t)65535 * 128;
}

int launch_mma_dense(ort_cuda_session* s, Weight& w, const float* A, int64_t M, bool transA,
                     float* Y, int64_t ldy, int mode, float alpha, float beta, const float* C,
                     int64_t c_rows, int64_t c_cols, int64_t c_col0, cudaStream_t st) {
  if (w.nl == 0 || M == 0) return ORT_CUDA_OK;
  const bool bf16 = mode == ORT_CUDA_MODE_MMA_BF16;
  const int64_t K = w.K, nl = w.nl;
  if (w.W16 == nullptr || w.w16_mode != mode) {
    ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
               "the weight's first tensor-core call prepares it; run it once before "
               "capturing a CUDA graph");
    // Prepack once per session (and per MMA mode): 16-bit [nl][K] + column exponents.
    if (w.W16) cudaFree(w.W16);
    if (w.col_exp) cudaFree(w.col_exp);
    w.W16 = nullptr;
    w.col_exp = nullptr;
    ORTC_CUDA(cudaMalloc(&w.W16, (size_t)(nl * K) * 2 * (bf16 ? 2 : 1)));  // bf16: hi, lo
    ORTC_CUDA(cudaMalloc(&w.col_exp, (size_t)nl * 4));
    if (!bf16) {
      wcol_exp_kernel<<<(unsigned)((nl + 255) / 256), 256, 0, st>>>(w.W, (int)K, (int)nl, w.col_exp);
      s->launches++;
    }
    dim3 g((unsigned)((nl + 31) / 32), (unsigned)((K + 31) / 32));
    if (bf16)
      w16_dense_kernel<true><<<g, dim3(32, 8), 0, st>>>(w.W, (int)K, (int)nl, w.col_exp,
                                                        (uint16_t*)w.W16);
    else
      w16_dense_kernel<false><<<g, dim3(32, 8), 0, st>>>(w.W, (int)K, (int)nl, w.col_exp,
                                                         (uint16_t*)w.W16);
    ORTC_CUDA(cudaGetLastError());
    s->launches++;
    w.w16_mode = mode;
  }
  int rc = ensure_kscratch(s, a_scratch_bytes(M, K, bf16));
  if (rc) return rc;
  uint16_t* A16;
  int* rexp;
  rc = convert_a(s, A, M, K, transA, bf16, 0, &A16, &rexp, st);
  if (rc) return rc;
  return launch_gemm(s, A16, rexp, M, (const uint16_t*)w.W16, w.col_exp, nl, K, bf16, Y, ldy,
                     alpha, beta, C, c_rows, c_cols, c_col0, st);
}

int launch_mma_nbits(ort_cuda_session* s, Weight& w, const float* A, int64_t M, float* Y,
                     int64_t ldy, int mode, cudaStream_t st, int reserve_sms,
                     const PrefillPush* push, const YSel* seg) {
  if (w.nl == 0 || M == 0) return ORT_CUDA_OK;
  const bool bf16 = mode == ORT_CUDA_MODE_MMA_BF16;
  const int64_t K = w.K, nl = w.nl;
  if (!bf16 && nbits_gemm_f16_ok(w)) {
    // fp16 mode: dequantisation fused into the GEMM; the per-(block, column)
    // zero-point / scale table and the column exponents are made once per
    // session and kept with the weight.
    if (w.sz16 == nullptr) {
      ORTC_CHECK(!s->capturing, ORT_CUDA_ERR_INVALID_ARG,
                 "the weight's first tensor-core call prepares it; run it once before "
                 "capturing a CUDA graph");
      if (w.col_exp == nullptr) ORTC_CUDA(cudaMalloc(&w.col_exp, (size_t)nl * 4));
      ORTC_CUDA(cudaMalloc(&w.sz16, (size_t)w.nb * w.s_pitch * 4));
      nbits_col_exp_kernel<<<(unsigned)((nl + 255) / 256), 256, 0, st>>>(w.scales, w.s_pitch, w.nb,
                                                                          (int)nl, w.col_exp);
      ORTC_CUDA(cudaGetLastError());
      s->launches++;
      int rc = prepare_nbits_sz16(w, w.col_exp, w.sz16, st, &s->launches);
      if (rc) return rc;
    }
    int rc = ensure_kscratch(s, a_scratch_bytes(M, K));
    if (rc) return rc;
    uint16_t* A16;
    int* rexp;
    rc = convert_a(s, A, M, K, false, false, 0, &A16, &rexp, st);
    if (rc) return rc;
    return launch_nbits_gemm_f16(w, A16, rexp, M, w.sz16, w.col_exp, Y, ldy, s->err_dev,
                                 s->sm_count, st, &s->launches, reserve_sms, push, seg);
  }
  ORTC_CHECK(push == nullptr && (seg == nullptr || seg->nseg == 0), ORT_CUDA_ERR_INVALID_ARG,
             "push mode and segmented output need the fused fp16 GEMM");
  const size_t a_bytes = a_scratch_bytes(M, K, bf16);
  const size_t w_bytes = al256((size_t)(nl * K) * 2 * (bf16 ? 2 : 1));
  const size_t e_bytes = al256((size_t)nl * 4);
  int rc = ensure_kscratch(s, a_bytes + w_bytes + e_bytes);
  if (rc) return rc;
  uint16_t* A16;
  int* rexp;
  rc = convert_a(s, A, M, K, false, bf16, 0, &A16, &rexp, st);
  if (rc) return rc;
  uint16_t* W16 = (uint16_t*)((char*)s->kscratch + a_bytes);
  int* cexp = (int*)((char*)s->kscratch + a_bytes + w_bytes);
  if (!bf16) {
    nbits_col_exp_kernel<<<(unsigned)((nl + 255) / 256), 256, 0, st>>>(w.scales, w.s_pitch, w.nb,
                                                                        (int)nl, cexp);
    s->launches++;
  }
  const int64_t total = nl * ((K + 7) / 8);
  unsigned blocks = (unsigned)((total + 255) / 256);
  if (blocks > (unsigned)s->sm_count * 16) blocks = (unsigned)s->sm_count * 16;
  if (bf16)
    w16_nbits_kernel<true><<<blocks, 256, 0, st>>>(w.B, w.scales, w.s_pitch, w.zp, w.z_pitch, (int)K,
                                                  w.nb, w.bs, (int)nl, cexp, W16);
  else
    w16_nbits_kernel<false><<<blocks, 256, 0, st>>>(w.B, w.scales, w.s_pitch, w.zp, w.z_pitch,
                                                   (int)K, w.nb, w.bs, (int)nl, cexp, W16);
  ORTC_CUDA(cudaGetLastError());
  s->launches++;
  return launch_gemm(s, A16, rexp, M, W16, cexp, nl, K, bf16, Y, ldy, 1.0f, 1.0f, nullptr, 0, 0, 0,
                     st);
}

}  // namespace ortc
