// MatMulInteger on tensor cores (opMatMulInteger, lib/src/onnx_qlinear_ops.
// dart:26-79): Y[M, N] = (A - a_zp) . (B - b_zp) in 32-bit integers, with A
// (activations, typically the uint8 output of DynamicQuantizeLinear) and B
// (an uploaded int8 or uint8 weight) of either signedness, a_zp scalar or per
// row, b_zp scalar or per column.  Expanding the product,
//   Y = A.B - a_zp[m] colsum(B)[n] - b_zp[n] rowsum(A)[m] + K a_zp[m] b_zp[n],
// so tcgen05.mma.kind::i8 takes the raw 8-bit operands straight from shared
// memory (exact s32 accumulation in TMEM) and the zero points become an
// epilogue correction (two's-complement wraparound, as int32 outputs wrap;
// the value is exact whenever it fits 32 bits, which holds for K <= 33025).
//
// Roles are swapped against the 16-bit GEMM: the MMA's M side is 128 weight
// columns (TMEM lanes) and its N side TBA activation rows (16..256, chosen by
// M), so a decode-sized M wastes little MMA work and each epilogue lane owns
// one output column (coalesced stores).  Per tile: a TMA warp streams 128-k
// stages of the weight (128 columns x 128 bytes) and of A (TBA rows x 128
// bytes, 128-byte swizzle) into a 4-stage ring; one thread issues 4 MMAs
// (K = 32) per stage; 4 epilogue warps apply the correction and store.  Grids
// too small for the SMs split K: the slices add into a zeroed Y with int32
// atomics (exact and order-free), the first slice adding the correction.
// Every wait is bounded; on expiry the kernel records an error and returns.
#include <atomic>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace ortc {
namespace {

constexpr int IBW = 128;      // weight columns per tile (MMA M, TMEM lanes)
constexpr int IBK = 128;      // k (bytes) per stage
constexpr int kI8Stages = 4;
constexpr int kI8Threads = 192;

struct I8Params {
  int32_t* Y;
  int64_t ldy;
  int M, N, K;
  int nk, per, ksplit;        // k blocks, k blocks per split, splits
  const int32_t* colsum;      // [N]
  const int32_t* bzp;         // [N] or null
  const int32_t* rowsum;      // [M] (when bzp)
  const uint8_t* azp;         // a zero point bytes (a_signed), null: 0
  int az_len;                 // 1 or M
  int a_signed;
  int* err;
};

template <int TBA>
__global__ void __launch_bounds__(kI8Threads, 1)
    matmul_i8_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                     uint32_t idesc, I8Params p) {
  constexpr uint32_t kWBytes = IBW * IBK, kABytes = TBA * IBK, kStage = kWBytes + kABytes;
  constexpr uint32_t kCols = TBA < 32 ? 32 : TBA;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kI8Stages * kStage);
  uint64_t* empty = full + kI8Stages;
  uint64_t* accum = empty + kI8Stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * IBW, m0 = blockIdx.y * TBA, z = blockIdx.z;
  const int kb0 = z * p.per, kb1 = min(p.nk, kb0 + p.per);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kI8Stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&tmW);
      prefetch_tensormap(&tmA);
      bool ok = true;
      int issued = 0;
      for (int kb = kb0; kb < kb1; kb++) {
        const int i = kb - kb0, s = i % kI8Stages;
        if (!mbar_wait(&empty[s], ((i / kI8Stages) & 1) ^ 1)) {
          record_error(p.err, KERR_WAIT_EMPTY);
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kStage;
        mbar_arrive_expect_tx(&full[s], kStage);
        tma_load_2d(st, &tmW, &full[s], kb * IBK, n0);
        tma_load_2d(st + kWBytes, &tmA, &full[s], kb * IBK, m0);
        issued = i + 1;
      }
      if (!ok)  // the copies already issued land before the CTA exits
        for (int i = (issued > kI8Stages ? issued - kI8Stages : 0); i < issued; i++)
          if (!mbar_wait(&full[i % kI8Stages], (i / kI8Stages) & 1))
            record_error(p.err, KERR_WAIT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int kb = kb0; kb < kb1 && ok; kb++) {
        const int i = kb - kb0, s = i % kI8Stages;
        if (!mbar_wait(&full[s], (i / kI8Stages) & 1)) {
          record_error(p.err, KERR_WAIT_FULL);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sw = smem_u32(smem + s * kStage), sa = sw + kWBytes;
#pragma unroll
        for (int kk = 0; kk < IBK / 32; kk++)
          mma_i8_ss(tmem, smem_desc_sw128(sw + kk * 32), smem_desc_sw128(sa + kk * 32), idesc,
                    (i | kk) != 0);
        mma_commit(&empty[s]);
      }
      mma_commit(accum);  // arrives once every issued MMA has completed
    }
    __syncwarp();
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = weight columns
    const int q = warp & 3;
    const int n = n0 + q * 32 + lane;
    const bool ok = mbar_wait(accum, 0);
    if (!ok) record_error(p.err, KERR_WAIT_MMA);
    tc_fence_after();
    const bool any = kb1 > kb0;  // an empty K slice contributes zero
    if (ok) {
      const uint32_t cs = n < p.N ? (uint32_t)p.colsum[n] : 0u;
      const uint32_t bz = (p.bzp && n < p.N) ? (uint32_t)p.bzp[n] : 0u;
      for (int c0 = 0; c0 < TBA; c0 += (TBA < 32 ? 16 : 32)) {
        uint32_t r[32];
        if constexpr (TBA < 32) {
          uint32_t r16[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + c0, r16);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; j++) r[j] = r16[j];
        } else {
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c0, r);
          tmem_ld_wait();
        }
        if (n >= p.N) continue;
#pragma unroll
        for (int j = 0; j < (TBA < 32 ? 16 : 32); j++) {
          const int m = m0 + c0 + j;
          if (m >= p.M) break;
          uint32_t v = any ? r[j] : 0u;
          if (z == 0) {
            uint32_t az = 0;
            if (p.azp) {
              const uint8_t b = p.azp[p.az_len == 1 ? 0 : m];
              az = p.a_signed ? (uint32_t)(int32_t)(int8_t)b : (uint32_t)b;
            }
            const uint32_t rs = p.bzp ? (uint32_t)p.rowsum[m] : 0u;
            v += (uint32_t)p.K * az * bz - az * cs - bz * rs;  // mod 2^32
          }
          int32_t* y = p.Y + (int64_t)m * p.ldy + n;
          if (p.ksplit > 1)
            atomicAdd(y, (int32_t)v);
          else
            *y = (int32_t)v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// rowsum[m] = sum_k A[m, k] (signed or unsigned bytes), one warp per row
__global__ void i8_rowsum_kernel(const uint8_t* __restrict__ A, int64_t lda, int M, int K,
                                 int a_signed, int32_t* __restrict__ rowsum) {
  const int m = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  const uint8_t* a = A + (int64_t)m * lda;
  int s = 0;
  for (int k = lane; k < K; k += 32) s += a_signed ? (int)(int8_t)a[k] : (int)a[k];
  s = __reduce_add_sync(0xffffffffu, s);
  if (lane == 0) rowsum[m] = s;
}

template <int TBA>
int launch_tba(const CUtensorMap& tmW, const CUtensorMap& tmA, uint32_t idesc, const I8Params& p,
               dim3 grid, cudaStream_t st) {
  constexpr size_t smem = 1024 + kI8Stages * (size_t)(IBW * IBK + TBA * IBK) + 256;
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load() >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(matmul_i8_kernel<TBA>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (dev < 64) configured.fetch_or(1ull << dev);
  }
  matmul_i8_kernel<TBA><<<grid, kI8Threads, smem, st>>>(tmW, tmA, idesc, p);
  ORTC_CUDA(cudaGetLastError());
  return ORT_CUDA_OK;
}

}  // namespace

int prepare_int8_tc(Weight& w) {
  return encode_tma_2d(&w.tmW8, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.Wi8, (uint64_t)w.K,
                       (uint64_t)w.nl, (uint64_t)w.kpitch, IBK, IBW, CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_matmul_i8(const Weight& w, const uint8_t* A, int64_t lda, int64_t M, int a_signed,
                     const uint8_t* azp, int64_t az_len, int32_t* Y, int64_t ldy,
                     int32_t* rowsum, int* err, int sm_count, cudaStream_t st,
                     int64_t* launches) {
  if (M == 0 || w.nl == 0) return ORT_CUDA_OK;
  ORTC_CHECK(lda % 16 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 && M < (1 << 30),
             ORT_CUDA_ERR_INVALID_ARG, "MatMulInteger: A rows must be 16-byte aligned");
  const int tba = M >= 256 ? 256 : (M > 64 ? 128 : (M > 32 ? 64 : (M > 16 ? 32 : 16)));
  CUtensorMap tmA;
  int rc = encode_tma_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, (uint64_t)w.K, (uint64_t)M,
                         (uint64_t)lda, IBK, tba, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  I8Params p;
  p.Y = Y;
  p.ldy = ldy;
  p.M = (int)M;
  p.N = (int)w.nl;
  p.K = (int)w.K;
  p.nk = (int)((w.K + IBK - 1) / IBK);
  const int tiles = (int)((w.nl + IBW - 1) / IBW) * (int)((M + tba - 1) / tba);
  int ksplit = std::max(1, std::min(p.nk, (sm_count + tiles - 1) / tiles));
  p.per = (p.nk + ksplit - 1) / ksplit;
  p.ksplit = (p.nk + p.per - 1) / p.per;
  p.colsum = w.colsum;
  p.bzp = w.bzp;
  p.rowsum = rowsum;
  p.azp = azp;
  p.az_len = (int)az_len;
  p.a_signed = a_signed;
  p.err = err;
  if (p.ksplit > 1)
    ORTC_CUDA(cudaMemset2DAsync(Y, (size_t)ldy * 4, 0, (size_t)w.nl * 4, (size_t)M, st));
  if (w.bzp) {
    i8_rowsum_kernel<<<(unsigned)((M + 7) / 8), 256, 0, st>>>(A, lda, (int)M, (int)w.K,
                                                            a_signed, rowsum);
    ORTC_CUDA(cudaGetLastError());
    (*launches)++;
  }
  const uint32_t idesc = idesc_i8_signs(w.i8_signed, a_signed, IBW, tba);
  const dim3 grid((unsigned)((w.nl + IBW - 1) / IBW), (unsigned)((M + tba - 1) / tba),
                  (unsigned)p.ksplit);
  switch (tba) {
    case 16: rc = launch_tba<16>(w.tmW8, tmA, idesc, p, grid, st); break;
    case 32: rc = launch_tba<32>(w.tmW8, tmA, idesc, p, grid, st); break;
    case 64: rc = launch_tba<64>(w.tmW8, tmA, idesc, p, grid, st); break;
    case 128: rc = launch_tba<128>(w.tmW8, tmA, idesc, p, grid, st); break;
    default: rc = launch_tba<256>(w.tmW8, tmA, idesc, p, grid, st); break;
  }
  if (rc) return rc;
  (*launches)++;
  return ORT_CUDA_OK;
}

}  // namespace ortc
