/*
 * CPU ORACLE — test infrastructure only, never the product path.
 *
 * A plain-C restatement of the reference's MatMulNBits / MatMul / Gemm
 * arithmetic (CrispStrobe/onnx_runtime_dart 0.10.3, pure Dart).  Only the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library; the CUDA path never calls it.
 *
 * Parity is pinned against the reference's own ORT-generated fixtures
 * (test/fixtures/matmulnbits_{basic,zeropoints,partial_block},
 * gemm_transB_bias, matmul_batched) and the hand-computed known answer of
 * test/gemm_prepack_test.dart:147; see tests/test_oracle.py.
 *
 * Rounding model.  The reference computes in Dart doubles and stores into
 * Float32List, or uses Float32x4 lanes.  Every scalar step it takes is one
 * of: fp32*fp32 or fp32+fp32 evaluated in double then narrowed, which is
 * the correctly rounded fp32 result (53 >= 2*24+2), or a Float32x4 lane op,
 * which is IEEE fp32.  This file therefore uses plain fp32 * and + and must
 * be compiled with -ffp-contract=off (no FMA contraction), except where the
 * reference itself accumulates in double (see gemv_tail below).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* onnx_proto_loader.dart:29-47 halfToFloat32Bits: fp16 bit pattern ->
 * fp32 bit pattern, bit-exact (subnormals normalised, inf/nan kept). */
ORC_API uint32_t orc_half_to_float_bits(uint32_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  int32_t exp = (int32_t)((h >> 10) & 0x1Fu);
  uint32_t mant = h & 0x3FFu;
  if (exp == 0) {
    if (mant == 0) return sign;
    int32_t e = -1;
    do {
      mant <<= 1;
      e++;
    } while ((mant & 0x400u) == 0);
    mant &= 0x3FFu;
    return sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
  } else if (exp == 0x1F) {
    return sign | 0x7F800000u | (mant << 13);
  }
  return sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13);
}

ORC_API void orc_half_to_float_array(const uint16_t* h, float* out, int64_t n) {
  for (int64_t i = 0; i < n; i++) {
    uint32_t b = orc_half_to_float_bits(h[i]);
    memcpy(&out[i], &b, 4);
  }
}

/* onnx_qlinear_ops.dart:120-149: dequantise packed uint4 B [N, nb, bs/2]
 * into the transposed fp32 matrix W [K x N] (row-major), column by column:
 *   W[k, n] = (q - zp) * scale[n*nb + blk]
 * q is the low nibble of byte B[n, blk, j>>1] for even j, the high nibble
 * for odd j; zp defaults to 8, else nibble (n*nb+blk) of the flat packed
 * zero-point array (low nibble first, :133-138).  The product of a small
 * integer and an fp32 is exact in double, so narrowing it equals fp32 *.
 * Columns [n0, n1) only, so threads can split the work. */
static void dequant_cols(const uint8_t* B, const float* scales, const uint8_t* zp,
                         int K, int N, int bs, float* W, int n0, int n1) {
  const int nb = (K + bs - 1) / bs;
  const int blob = bs / 2;
  for (int col = n0; col < n1; col++) {
    const int64_t col_base = (int64_t)col * nb * blob;
    for (int blk = 0; blk < nb; blk++) {
      const float scale = scales[(int64_t)col * nb + blk];
      float z = 8.0f;
      if (zp) {
        const int64_t zi = (int64_t)col * nb + blk;
        const uint8_t byte = zp[zi >> 1];
        z = (float)((zi & 1) == 0 ? (byte & 0xF) : (byte >> 4));
      }
      const int64_t blob_base = col_base + (int64_t)blk * blob;
      const int k_base = blk * bs;
      const int k_end = k_base + bs < K ? k_base + bs : K;
      for (int kk = k_base; kk < k_end; kk++) {
        const int j = kk - k_base;
        const uint8_t byte = B[blob_base + (j >> 1)];
        const int q = (j & 1) == 0 ? (byte & 0xF) : (byte >> 4);
        W[(int64_t)kk * N + col] = ((float)q - z) * scale;
      }
    }
  }
}

ORC_API void orc_dequant_nbits(const uint8_t* B, const float* scales, const uint8_t* zp,
                               int K, int N, int bs, float* W) {
  dequant_cols(B, scales, zp, K, N, bs, W, 0, N);
}

/* gemm_kernel_simd.dart:27-309 matmulKernel: out[m x n] = a[m x k] . b[k x n].
 * Every path of the SIMD kernel (4x8 register tiles :82-113, lane and row
 * remainders :115-168, _gemvAligned :196-246, the Float32x4 part of
 * _gemvScalar :251-298) accumulates each output independently, in
 * ascending k, as c = c + a*b with two fp32 roundings, starting from 0.
 * Column panels and tiling only reorder independent outputs.  The one
 * exception is m == 1 with n % 4 != 0: _gemvScalar's scalar tail
 * (:299-307) accumulates the last n % 4 columns in double and narrows once.
 * (B is always a fresh, 16-byte aligned Float32List on the MatMulNBits and
 * Gemm paths, so with n % 4 == 0 the aligned kernel runs; with an
 * unaligned base but n % 4 == 0 _gemvScalar has no tail, same numbers.)
 * Computes columns [n0, n1) of the full-width call. */
static void matmul_cols(const float* a, const float* b, float* out, int64_t m, int k,
                        int n, int n0, int n1) {
  const int tail0 = (m == 1) ? (n - (n & 3)) : n;
  float* acc = (float*)malloc(sizeof(float) * (size_t)(n1 > n0 ? n1 - n0 : 1));
  for (int64_t i = 0; i < m; i++) {
    const float* arow = a + i * (int64_t)k;
    float* orow = out + i * (int64_t)n;
    const int f1 = n1 < tail0 ? n1 : tail0;
    /* fp32 columns: c = fl(c + fl(a*b)), k ascending (vectorises over j). */
    if (f1 > n0) {
      const int w = f1 - n0;
      for (int j = 0; j < w; j++) acc[j] = 0.0f;
      for (int kk = 0; kk < k; kk++) {
        const float av = arow[kk];
        const float* brow = b + (int64_t)kk * n + n0;
        for (int j = 0; j < w; j++) {
          const float p = av * brow[j];
          acc[j] = acc[j] + p;
        }
      }
      for (int j = 0; j < w; j++) orow[n0 + j] = acc[j];
    }
    /* _gemvScalar tail columns (m == 1 only): double accumulation. */
    for (int j = (n0 > tail0 ? n0 : tail0); j < n1; j++) {
      double s = 0.0;
      for (int kk = 0; kk < k; kk++) s += (double)arow[kk] * (double)b[(int64_t)kk * n + j];
      orow[j] = (float)s;
    }
  }
  free(acc);
}

/* gemm_kernel_scalar.dart:10-41 (web kernel): out += v * bv with the
 * product exact in double and one rounding of (out + product) to fp32
 * (Float32List store).  Provided for completeness of the oracle; the
 * native (SIMD) kernel above is the one the parity tests pin. */
ORC_API void orc_matmul_kernel_scalar(const float* a, const float* b, float* out,
                                      int64_t m, int k, int n) {
  for (int64_t i = 0; i < m; i++) {
    for (int j = 0; j < n; j++) out[i * n + j] = 0.0f;
    for (int kk = 0; kk < k; kk++) {
      const double v = a[i * k + kk];
      for (int j = 0; j < n; j++) {
        out[i * n + j] = (float)((double)out[i * n + j] + v * (double)b[(int64_t)kk * n + j]);
      }
    }
  }
}

/* Column split of parallel_pool.dart:124-125: worker w owns
 * base + (w < rem) columns, base = n / W, rem = n % W, in order. */
static void split_cols(int n, int workers, int w, int* c0, int* c1) {
  const int base = n / workers, rem = n % workers;
  int start = 0;
  for (int i = 0; i < w; i++) start += base + (i < rem ? 1 : 0);
  *c0 = start;
  *c1 = start + base + (w < rem ? 1 : 0);
}

typedef struct {
  /* matmul */
  const float* a;
  const float* b;
  float* out;
  int64_t m;
  int k, n;
  /* dequant */
  const uint8_t* B;
  const float* scales;
  const uint8_t* zp;
  int K, N, bs;
  float* W;
  int workers, w;
  int phase; /* 0 = dequant, 1 = matmul */
} job_t;

static void* run_job(void* p) {
  job_t* j = (job_t*)p;
  int c0, c1;
  if (j->phase == 0) {
    split_cols(j->N, j->workers, j->w, &c0, &c1);
    dequant_cols(j->B, j->scales, j->zp, j->K, j->N, j->bs, j->W, c0, c1);
  } else {
    split_cols(j->n, j->workers, j->w, &c0, &c1);
    if (c1 > c0) matmul_cols(j->a, j->b, j->out, j->m, j->k, j->n, c0, c1);
  }
  return NULL;
}

static void run_parallel(job_t* proto, int threads) {
  if (threads < 1) threads = 1;
  if (threads == 1) {
    proto->workers = 1;
    proto->w = 0;
    run_job(proto);
    return;
  }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  job_t* jobs = (job_t*)malloc(sizeof(job_t) * (size_t)threads);
  for (int w = 0; w < threads; w++) {
    jobs[w] = *proto;
    jobs[w].workers = threads;
    jobs[w].w = w;
    pthread_create(&th[w], NULL, run_job, &jobs[w]);
  }
  for (int w = 0; w < threads; w++) pthread_join(th[w], NULL);
  free(th);
  free(jobs);
}

/* matmulKernel over `threads` column slices (parallel_pool.dart:124-125).
 * Each column keeps the full-width call's arithmetic, so the result is
 * bitwise independent of `threads` (the reference's pool invariant,
 * parallel_pool.dart:7-8, test/parallel_pool_test.dart). */
ORC_API void orc_matmul_kernel(const float* a, const float* b, float* out, int64_t m, int k,
                               int n, int threads) {
  job_t j;
  memset(&j, 0, sizeof(j));
  j.a = a;
  j.b = b;
  j.out = out;
  j.m = m;
  j.k = k;
  j.n = n;
  j.phase = 1;
  run_parallel(&j, threads);
}

/* onnx_qlinear_ops.dart:114-156 opMatMulNBits: dequantise all of B into a
 * fresh [K x N] fp32 buffer, then matmulKernel(A, W) with M = len(A)/K.
 * Returns 0, or -1 if bits != 4 (the reference throws UnsupportedError). */
ORC_API int orc_matmul_nbits(const float* A, int64_t M, const uint8_t* B, const float* scales,
                             const uint8_t* zp, int K, int N, int bits, int bs, float* Y,
                             int threads) {
  if (bits != 4) return -1;
  float* W = (float*)malloc(sizeof(float) * (size_t)K * (size_t)N);
  if (!W) return -2;
  job_t j;
  memset(&j, 0, sizeof(j));
  j.B = B;
  j.scales = scales;
  j.zp = zp;
  j.K = K;
  j.N = N;
  j.bs = bs;
  j.W = W;
  j.phase = 0;
  run_parallel(&j, threads);
  orc_matmul_kernel(A, W, Y, M, K, N, threads);
  free(W);
  return 0;
}

/* onnx_ops.dart:629-689 opTranspose for rank 2: out[j, i] = in[i, j]. */
ORC_API void orc_transpose(const float* in, float* out, int rows, int cols) {
  for (int i = 0; i < rows; i++)
    for (int j = 0; j < cols; j++) out[(int64_t)j * rows + i] = in[(int64_t)i * cols + j];
}

/* onnx_ops.dart:1777-1793 opGemm on the prepacked B of
 * onnx_graph.dart:1156-1173 (Bt is the effective [K x N] operand):
 *   mm = matmulKernel(A, Bt)            (opMatMul :1375-1431)
 *   mm = mm * alpha   if alpha != 1     (:1785-1789, fp32 store)
 *   C' = C * beta     if beta  != 1     (:1791, _elementwiseUnary)
 *   Y  = mm + C'  with numpy broadcast  (opAdd / _arithFloatFast :218-250)
 * C is [c_rows x c_cols] with c_rows in {1, M} and c_cols in {1, N}
 * (covers scalar, [N], [1,N], [M,1] and [M,N] bias); C may be NULL. */
ORC_API void orc_gemm(const float* A, const float* Bt, int64_t M, int K, int N, float alpha,
                      float beta, const float* C, int64_t c_rows, int64_t c_cols, float* Y,
                      int threads) {
  orc_matmul_kernel(A, Bt, Y, M, K, N, threads);
  if (alpha != 1.0f) {
    for (int64_t i = 0; i < M * (int64_t)N; i++) Y[i] = Y[i] * alpha;
  }
  if (!C) return;
  for (int64_t i = 0; i < M; i++) {
    for (int j = 0; j < N; j++) {
      float c = C[(c_rows == 1 ? 0 : i) * c_cols + (c_cols == 1 ? 0 : j)];
      if (beta != 1.0f) c = c * beta;
      Y[i * N + j] = Y[i * N + j] + c;
    }
  }
}
