// CUDA-core tiled GEMM for every M, over a packed int4 (MatMulNBits) or a
// dense fp32 (MatMul / Gemm) weight, plus the small helper kernels.
//
// Each output is accumulated by one thread in ascending k from 0, which is
// the order of every path of the reference's matmulKernel
// (gemm_kernel_simd.dart:27-169).  Two arithmetic variants:
//   exact  (ORT_CUDA_MODE_EXACT)  acc = fma(a, w, acc)
//   strict (ORT_CUDA_MODE_STRICT) acc = fl(acc + fl(a * w))  -- the
//          reference's two roundings, so the result is bitwise equal.
// In both, the int4 weight tile is dequantised exactly as
// onnx_qlinear_ops.dart:144-147 does: w = fl((q - zp) * scale).
// The Gemm epilogue follows onnx_ops.dart:1785-1792: multiply by alpha
// (when alpha != 1), add beta * C (beta applied only when != 1), each an
// fp32 rounding of its own.
#include "common.cuh"

namespace ortc {
namespace {

constexpr int BM = 64, BN = 64, BK = 32, TM = 4, TN = 4;  // 256 threads

template <bool STRICT>
__device__ __forceinline__ float mac(float acc, float a, float b) {
  if (STRICT) return __fadd_rn(acc, __fmul_rn(a, b));
  return __fmaf_rn(a, b, acc);
}

struct NbitsSrc {
  const uint8_t* B;   // permuted-nibble packed columns
  const float* S;     // [nb][s_pitch]
  const uint8_t* Z;   // [ceil(nb/2)][z_pitch] or null
  int64_t col_bytes, s_pitch, z_pitch;
  int nb, bs;
};
struct DenseSrc {
  const float* W;  // [K][ldw]
  int64_t ldw;
};

// Fill Ws[BK][BN] with the dequantised weight tile (k0.., n0..).
__device__ __forceinline__ void load_w_tile(float (&Ws)[BK][BN + 4], const NbitsSrc& src,
                                            int k0, int n0, int K, int N) {
  // 64 columns x 32 k = 64 x 4 words of 8 nibbles; one word per thread.
  const int t = threadIdx.x;
  const int c = t >> 2, wd = t & 3;
  const int n = n0 + c;
  const int kw = k0 + wd * 8;
  float v[8];
  if (n < N && kw < K) {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(src.B + (int64_t)n * src.col_bytes + (kw >> 1)));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int kk = kw + i;
      const int blk = kk / src.bs;
      if (kk < K) {
        const float scale = __ldg(src.S + (int64_t)blk * src.s_pitch + n);
        const float z = src.Z ? (float)nbits_zp(src.Z, src.z_pitch, n, blk) : 8.0f;
        const float q = (float)nbits_q(w, i);
        v[i] = __fmul_rn(__fsub_rn(q, z), scale);
      } else {
        v[i] = 0.0f;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = 0.0f;
  }
#pragma unroll
  for (int i = 0; i < 8; i++) Ws[wd * 8 + i][c] = v[i];
}

__device__ __forceinline__ void load_w_tile(float (&Ws)[BK][BN + 4], const DenseSrc& src,
                                            int k0, int n0, int K, int N) {
  for (int i = threadIdx.x; i < BK * BN; i += 256) {
    const int kk = i / BN, c = i % BN;
    const int k = k0 + kk, n = n0 + c;
    Ws[kk][c] = (k < K && n < N) ? __ldg(src.W + (int64_t)k * src.ldw + n) : 0.0f;
  }
}

// Batched activation x activation MatMul: batch b reads B + b * stride.
__device__ __forceinline__ NbitsSrc batch_offset(const NbitsSrc& s, int64_t) { return s; }
__device__ __forceinline__ DenseSrc batch_offset(const DenseSrc& s, int64_t off) {
  return DenseSrc{s.W + off, s.ldw};
}

struct Epi {
  float alpha, beta;
  const float* C;
  int64_t c_rows, c_cols, c_col0;  // C indexed with global column c_col0 + n
  bool has_c;
};

template <bool STRICT, typename Src>
__global__ void __launch_bounds__(256)
    simt_gemm_kernel(const float* __restrict__ A, int64_t M, int K, int N, bool transA, Src src,
                     float* __restrict__ Y, int64_t ldy, Epi epi, int64_t batch_a, int64_t batch_y,
                     int64_t batch_w) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Ws[BK][BN + 4];
  const int bz = blockIdx.z;
  A += bz * batch_a;
  Y += bz * batch_y;
  const int64_t m0 = (int64_t)blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;
  const int tx = threadIdx.x % (BN / TN), ty = threadIdx.x / (BN / TN);
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;

  const Src s2 = batch_offset(src, bz * batch_w);

  for (int k0 = 0; k0 < K; k0 += BK) {
    // A tile: As[k][m] = A[m0+m][k0+k]
    for (int i = threadIdx.x; i < BK * BM; i += 256) {
      int kk, mm;
      if (!transA) {
        mm = i / BK;
        kk = i % BK;
      } else {
        kk = i / BM;
        mm = i % BM;
      }
      const int64_t m = m0 + mm;
      const int k = k0 + kk;
      float v = 0.0f;
      if (m < M && k < K) v = transA ? __ldg(A + (int64_t)k * M + m) : __ldg(A + m * K + k);
      As[kk][mm] = v;
    }
    load_w_tile(Ws, s2, k0, n0, K, N);
    __syncthreads();
    const int kmax = (K - k0) < BK ? (K - k0) : BK;
    for (int kk = 0; kk < kmax; kk++) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; i++) a[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; j++) b[j] = Ws[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = mac<STRICT>(acc[i][j], a[i], b[j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int64_t m = m0 + ty * TM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      const int n = n0 + tx * TN + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (epi.alpha != 1.0f) v = __fmul_rn(v, epi.alpha);
      if (epi.has_c) {
        const int64_t cn = epi.c_col0 + n;
        float c = epi.C[(epi.c_rows == 1 ? 0 : m) * epi.c_cols + (epi.c_cols == 1 ? 0 : cn)];
        if (epi.beta != 1.0f) c = __fmul_rn(c, epi.beta);
        v = __fadd_rn(v, c);
      }
      Y[m * ldy + n] = v;
    }
  }
}

// Strict mode, M == 1, the last N % 4 (global) columns: the reference's
// _gemvScalar tail accumulates in double (gemm_kernel_simd.dart:299-307).
// One thread per column; [col_lo, col_hi) are local column indices.
template <typename Src>
__global__ void strict_tail_kernel(const float* __restrict__ A, int K, Src src, int col_lo,
                                   int col_hi, float* __restrict__ Y, Epi epi);

template <>
__global__ void strict_tail_kernel<NbitsSrc>(const float* __restrict__ A, int K, NbitsSrc src,
                                             int col_lo, int col_hi, float* __restrict__ Y,
                                             Epi epi) {
  const int n = col_lo + threadIdx.x;
  if (n >= col_hi) return;
  double acc = 0.0;
  for (int k = 0; k < K; k++) {
    const int blk = k / src.bs;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(src.B + (int64_t)n * src.col_bytes + ((k >> 3) << 2));
    const float q = (float)nbits_q(word, k & 7);
    const float z = src.Z ? (float)nbits_zp(src.Z, src.z_pitch, n, blk) : 8.0f;
    const float w = __fmul_rn(__fsub_rn(q, z), src.S[(int64_t)blk * src.s_pitch + n]);
    acc = __dadd_rn(acc, __dmul_rn((double)A[k], (double)w));
  }
  Y[n] = (float)acc;
}

template <>
__global__ void strict_tail_kernel<DenseSrc>(const float* __restrict__ A, int K, DenseSrc src,
                                             int col_lo, int col_hi, float* __restrict__ Y,
                                             Epi epi) {
  const int n = col_lo + threadIdx.x;
  if (n >= col_hi) return;
  double acc = 0.0;
  for (int k = 0; k < K; k++)
    acc = __dadd_rn(acc, __dmul_rn((double)A[k], (double)src.W[(int64_t)k * src.ldw + n]));
  float v = (float)acc;
  if (epi.alpha != 1.0f) v = __fmul_rn(v, epi.alpha);
  if (epi.has_c) {
    const int64_t cn = epi.c_col0 + n;
    float c = epi.C[epi.c_cols == 1 ? 0 : cn];
    if (epi.beta != 1.0f) c = __fmul_rn(c, epi.beta);
    v = __fadd_rn(v, c);
  }
  Y[n] = v;
}

__global__ void permute_nibbles_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                       int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = nbits_permute_word(in[i]);
}

__global__ void half_to_float_kernel(const uint16_t* __restrict__ h, float* __restrict__ out,
                                     int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __half2float(__ushort_as_half(h[i]));  // exact widening
}

__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out,
                                 int64_t rows, int64_t cols) {
  __shared__ float t[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = t[threadIdx.x][i];
  }
}

__global__ void unshard_kernel(const float* __restrict__ g, float* __restrict__ Y, int64_t world,
                               int64_t M, int64_t Ns, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i % N;
    const int64_t r = n / Ns, c = n % Ns;
    Y[i] = g[(r * M + m) * Ns + c];
  }
}

// Exact-mode dense GEMM (FFMA), row-major A with K % 4 == 0 and a weight
// of row pitch ldw % 4 == 0, both 16-byte aligned: 64 x 64 tiles, 16-k
// stages double-buffered through registers, one float4 of A and one of W
// per thread and stage; A is stored transposed in shared memory so each
// thread reads its 4 rows and 4 columns with one 16-byte load each per k.
// Every output still accumulates with fma in ascending k from 0, as the
// general kernel does (the exact mode's arithmetic), so the two kernels
// give the same bits.
constexpr int XBM = 64, XBN = 64, XBK = 16;

__global__ void __launch_bounds__(256)
    sgemm_exact_kernel(const float* __restrict__ A, int64_t M, int K, int N,
                       const float* __restrict__ W, int64_t ldw, float* __restrict__ Y,
                       int64_t ldy, Epi epi) {
  __shared__ __align__(16) float As[2][XBK][XBM];
  __shared__ __align__(16) float Bs[2][XBK][XBN];
  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * XBM;
  const int n0 = blockIdx.x * XBN;
  // loader coordinates: A row t / 4, k quad t % 4; W k row t / 16, n quad t % 16
  const int ar = t >> 2, ak = (t & 3) * 4;
  const int bk = t >> 4, bn = (t & 15) * 4;
  const int64_t am = m0 + ar;
  const int gn = n0 + bn;
  auto load = [&](int k0, float4& va, float4& vb) {
    va = make_float4(0.f, 0.f, 0.f, 0.f);
    vb = make_float4(0.f, 0.f, 0.f, 0.f);
    if (am < M && k0 + ak < K)  // K % 4 == 0: the quad is whole
      va = __ldg(reinterpret_cast<const float4*>(A + am * K + k0 + ak));
    const int k = k0 + bk;
    if (k < K) {
      const float* wr = W + (int64_t)k * ldw;
      if (gn + 3 < N) {
        vb = __ldg(reinterpret_cast<const float4*>(wr + gn));
      } else {
        if (gn < N) vb.x = __ldg(wr + gn);
        if (gn + 1 < N) vb.y = __ldg(wr + gn + 1);
        if (gn + 2 < N) vb.z = __ldg(wr + gn + 2);
      }
    }
  };
  auto store = [&](int buf, const float4& va, const float4& vb) {
    As[buf][ak + 0][ar] = va.x;
    As[buf][ak + 1][ar] = va.y;
    As[buf][ak + 2][ar] = va.z;
    As[buf][ak + 3][ar] = va.w;
    *reinterpret_cast<float4*>(&Bs[buf][bk][bn]) = vb;
  };
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
  float4 va, vb;
  load(0, va, vb);
  store(0, va, vb);
  __syncthreads();
  const int nst = (K + XBK - 1) / XBK;
  for (int s = 0; s < nst; s++) {
    const int buf = s & 1;
    if (s + 1 < nst) load((s + 1) * XBK, va, vb);
#pragma unroll
    for (int kk = 0; kk < XBK; kk++) {
      const float4 a = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
    }
    if (s + 1 < nst) {
      store(buf ^ 1, va, vb);
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (epi.alpha != 1.0f) v = __fmul_rn(v, epi.alpha);
      if (epi.has_c) {
        const int64_t cn = epi.c_col0 + n;
        float c = epi.C[(epi.c_rows == 1 ? 0 : m) * epi.c_cols + (epi.c_cols == 1 ? 0 : cn)];
        if (epi.beta != 1.0f) c = __fmul_rn(c, epi.beta);
        v = __fadd_rn(v, c);
      }
      Y[m * ldy + n] = v;
    }
  }
}

template <bool STRICT, typename Src>
int run_simt(const float* A, int64_t M, int K, int N, bool transA, const Src& src, float* Y,
             int64_t ldy, const Epi& epi, int64_t batch, int64_t batch_a, int64_t batch_y,
             int64_t batch_w, cudaStream_t st, int64_t* launches) {
  if (M == 0 || N == 0) return ORT_CUDA_OK;
  const int64_t gy = (M + BM - 1) / BM;
  if (gy > 65535 || batch > 65535) return fail(ORT_CUDA_ERR_INVALID_ARG, "simt gemm: grid too large");
  dim3 grid((N + BN - 1) / BN, (unsigned)gy, (unsigned)batch);
  simt_gemm_kernel<STRICT, Src><<<grid, 256, 0, st>>>(A, M, K, N, transA, src, Y, ldy, epi,
                                                      batch_a, batch_y, batch_w);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

}  // namespace

int launch_simt_gemm(const Weight& w, const float* A, int64_t M, bool transA, float* Y,
                     int64_t ldy, bool strict, float alpha, float beta, const float* C,
                     int64_t c_rows, int64_t c_cols, int64_t c_col0, cudaStream_t st,
                     int64_t* launches) {
  if (w.nl == 0 || M == 0) return ORT_CUDA_OK;
  Epi epi{alpha, beta, C, c_rows, c_cols, c_col0, C != nullptr};
  const int K = (int)w.K, N = (int)w.nl;
  int rc;
  // Strict M == 1: the reference's double-accumulated tail columns are the
  // last N % 4 of the FULL weight (global columns >= N - N % 4).
  int tail_lo = N;
  if (strict && M == 1 && (w.N & 3) != 0) {
    const int64_t g_lo = w.N - (w.N & 3) - w.n0;  // local index of first tail column
    tail_lo = (int)(g_lo < 0 ? 0 : (g_lo > N ? N : g_lo));
  }
  if (w.kind == W_NBITS) {
    NbitsSrc src{w.B, w.scales, w.zp, (int64_t)w.nb * w.bs / 2, w.s_pitch, w.z_pitch, w.nb, w.bs};
    rc = strict ? run_simt<true>(A, M, K, tail_lo, transA, src, Y, ldy, epi, 1, 0, 0, 0, st, launches)
                : run_simt<false>(A, M, K, N, transA, src, Y, ldy, epi, 1, 0, 0, 0, st, launches);
    if (rc == ORT_CUDA_OK && tail_lo < N) {
      strict_tail_kernel<NbitsSrc><<<1, 32, 0, st>>>(A, K, src, tail_lo, N, Y, epi);
      ORTC_CUDA(cudaGetLastError());
      (*launches)++;
    }
  } else {
    DenseSrc src{w.W, w.nl};
    const bool fast = !strict && !transA && K % 4 == 0 && w.nl % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(w.W) & 15) == 0 &&
                      (M + XBM - 1) / XBM <= 65535;
    if (fast) {
      dim3 grid((unsigned)((N + XBN - 1) / XBN), (unsigned)((M + XBM - 1) / XBM));
      sgemm_exact_kernel<<<grid, 256, 0, st>>>(A, M, K, N, w.W, w.nl, Y, ldy, epi);
      ORTC_CUDA(cudaGetLastError());
      (*launches)++;
      return ORT_CUDA_OK;
    }
    rc = strict ? run_simt<true>(A, M, K, tail_lo, transA, src, Y, ldy, epi, 1, 0, 0, 0, st, launches)
                : run_simt<false>(A, M, K, N, transA, src, Y, ldy, epi, 1, 0, 0, 0, st, launches);
    if (rc == ORT_CUDA_OK && tail_lo < N) {
      strict_tail_kernel<DenseSrc><<<1, 32, 0, st>>>(A, K, src, tail_lo, N, Y, epi);
      ORTC_CUDA(cudaGetLastError());
      (*launches)++;
    }
  }
  return rc;
}

int launch_simt_batched(const float* A, const float* B, int64_t batch, int64_t m, int64_t k,
                        int64_t n, int64_t b_batch_stride, float* Y, bool strict,
                        cudaStream_t st, int64_t* launches) {
  if (batch == 0 || m == 0 || n == 0) return ORT_CUDA_OK;
  Epi epi{1.0f, 1.0f, nullptr, 0, 0, 0, false};
  DenseSrc src{B, n};
  int rc;
  // m == 1 per batch runs the reference's _gemv, whose tail columns
  // (n % 4) accumulate in double (gemm_kernel_simd.dart:299-307).
  const int tail_lo = (strict && m == 1) ? (int)(n - (n & 3)) : (int)n;
  if (strict)
    rc = run_simt<true>(A, m, (int)k, tail_lo, false, src, Y, n, epi, batch, m * k, m * n,
                        b_batch_stride, st, launches);
  else
    rc = run_simt<false>(A, m, (int)k, (int)n, false, src, Y, n, epi, batch, m * k, m * n,
                         b_batch_stride, st, launches);
  if (rc == ORT_CUDA_OK && tail_lo < n) {
    for (int64_t b = 0; b < batch; b++) {
      DenseSrc sb{B + b * b_batch_stride, n};
      strict_tail_kernel<DenseSrc><<<1, 32, 0, st>>>(A + b * k, (int)k, sb, tail_lo, (int)n,
                                                     Y + b * n, epi);
      ORTC_CUDA(cudaGetLastError());
      (*launches)++;
    }
  }
  return rc;
}

int launch_permute_nibbles(const uint32_t* in, uint32_t* out, int64_t nwords, cudaStream_t st,
                           int64_t* launches) {
  if (nwords == 0) return ORT_CUDA_OK;
  int64_t blocks = (nwords + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  permute_nibbles_kernel<<<(unsigned)blocks, 256, 0, st>>>(in, out, nwords);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

int launch_half_to_float(const uint16_t* h, float* out, int64_t n, cudaStream_t st,
                         int64_t* launches) {
  if (n == 0) return ORT_CUDA_OK;
  half_to_float_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(h, out, n);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

int launch_transpose(const float* in, float* out, int64_t rows, int64_t cols, cudaStream_t st,
                     int64_t* launches) {
  if (rows == 0 || cols == 0) return ORT_CUDA_OK;
  if ((rows + 31) / 32 > 65535) return fail(ORT_CUDA_ERR_INVALID_ARG, "transpose: too many rows");
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(in, out, rows, cols);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

int launch_unshard(const float* g, float* Y, int64_t world, int64_t M, int64_t Ns, int64_t N,
                   cudaStream_t st, int64_t* launches) {
  if (M * N == 0) return ORT_CUDA_OK;
  int64_t blocks = (M * N + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  unshard_kernel<<<(unsigned)blocks, 256, 0, st>>>(g, Y, world, M, Ns, N);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

}  // namespace ortc
