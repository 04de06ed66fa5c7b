// Prefill MatMulNBits on tcgen05 tensor cores with the int4 dequantisation
// fused into the GEMM main loop (fp16 MMA mode).
//
//   Y[M, N] = 2^(e_m + f_n) * sum_k A16[m, k] * W16[n, k]
//   W16[n, k] = fp16((q - z) * fp16(scale * 2^-f_n))
//
// replacing, for prefill-sized M, the reference's dequantisation of all of B
// into fp32 followed by matmulKernel (onnx_qlinear_ops.dart:127-154,
// gemm_kernel_simd.dart:27-309).  A16 is the activation converted once per
// call to fp16 with a power-of-two row normalisation e_m; f_n normalises
// each weight column so its largest |(q - z) * scale| lies in [2^14, 2^15).
// Packed weights are read once per 256-row band of A straight from their
// upload layout; no 16-bit copy of the weights is written to HBM.
//
// Persistent kernel, one CTA per SM, tiles of 256 (m) x 128 (n), 64-k stages.
// The converted weight tile is the expensive operand, so each one serves 256
// rows of A.  The MMA takes it as its A operand (M = 128 weight columns)
// and the activation tile as B (N = 256 rows): one M=128, N=256 MMA per
// 16-k step reads 12 KB of shared memory, where two M=128, N=128 MMAs
// sharing the weight tile as B read 16 KB; shared-memory bandwidth, which
// the MMAs share with the TMA writes and the converters, is what bounds the
// kernel.  D is then transposed (TMEM lane = weight column, TMEM column =
// activation row), so a warp's epilogue stores for one row are 32
// consecutive columns: coalesced with no shared-memory transpose.
//   warp 0      TMA producer: A tile (256 x 64 fp16, 128-byte swizzle), the
//               packed int4 tile (128 columns x 32 bytes, 32-byte swizzle)
//               and the stage's {1024 + z, scale'} table (fp16 pairs) into a
//               4-stage ring
//   warps 2-9   converters: threads n and n + 128 share weight column n of
//               the tile (k 0-31 and 32-63 of the stage); per 8 weights two
//               masks, four byte permutes (nibble | 0x6400 is the fp16 value
//               1024 + q), four exact subtractions of 1024 + z and four
//               multiplies by the scale (one rounding), stored as the MMA's
//               K-major 128-byte-swizzled A tile
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32
//               accumulators); an elect.sync leader waits once per stage and
//               issues 4 MMAs (M=128, N=256, K=16), tcgen05.commit frees the
//               stage and the converted tile
//   warps 10-13 epilogue: tcgen05.ld of the finished accumulator while the
//               MMAs fill the other one (warp q owns weight columns
//               32q .. 32q + 31 of the tile), exact 2^(e_m + f_n) scaling,
//               one coalesced 128-byte store per row and warp
// Every wait is bounded; on expiry the kernel records an error and returns.
#include <cuda_fp16.h>

#include <algorithm>

#include <atomic>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace ortc {
namespace {

constexpr int PBM = 256, PBN = 128, PBK = 64;
constexpr int kHalf = 128;                           // rows of one MMA (M)
constexpr int kRaw = 4;                              // producer ring depth
constexpr int kConv = 4;                             // converted weight tiles
constexpr uint32_t kABytes = PBM * PBK * 2;          // 32 KB fp16 A tile
constexpr uint32_t kQBytes = PBN * PBK / 2;          // 4 KB packed int4 tile
constexpr uint32_t kSZBytes = PBN * 4 * 4;           // up to 4 blocks per stage
constexpr uint32_t kRawBytes = kABytes + kQBytes + kSZBytes;  // 38 KB
constexpr uint32_t kCBytes = PBN * PBK * 2;          // 16 KB fp16 weight tile
constexpr int kConvWarp0 = 2, kConvWarps = 8, kEpiWarp0 = 10;
constexpr int kThreadsP = 14 * 32;
constexpr size_t kSmemP = 1024 + kRaw * kRawBytes + kConv * kCBytes + 256;

struct PParams {
  float* Y;
  int64_t ldy;
  const int* row_exp;  // [M]
  const int* col_exp;  // [N]
  int* err;
  int M, N, K;
  int m_tiles, tiles;
  int bps;       // quantisation blocks per 64-k stage (>= 1)
  int bs_shift;  // log2(block size)
  uint32_t stage_tx;
  PrefillPush push;  // world == 0: no peers
  // a fused group's parts (nseg > 0): columns [seg_start[j], seg_start[j+1])
  // go to seg_y[j] with row pitch seg_ld[j]; every boundary is a multiple of
  // 32, so one 32-column chunk of the epilogue stays within one part
  int nseg = 0;
  int64_t seg_start[kMaxSegs + 1] = {};
  float* seg_y[kMaxSegs] = {};
  int64_t seg_ld[kMaxSegs] = {};
};

__device__ __forceinline__ float pow2f(int e) {
  return __uint_as_float((uint32_t)(e + 127) << 23);
}
__device__ __forceinline__ float scale_pow2(float v, int e) {
  while (e > 100) { v *= pow2f(100); e -= 100; }
  while (e < -100) { v *= pow2f(-100); e += 100; }
  return v * pow2f(e);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// (h - zz) * s on two fp16 lanes: the subtraction of small integers is exact,
// the product is rounded once.
__device__ __forceinline__ uint32_t deq2(uint32_t h, uint32_t zz, uint32_t s) {
  uint32_t d;
  asm("{\n\t.reg .b32 t;\n\t"
      "sub.rn.f16x2 t, %1, %2;\n\t"
      "mul.rn.f16x2 %0, t, %3;\n\t}"
      : "=r"(d)
      : "r"(h), "r"(zz), "r"(s));
  return d;
}

template <bool PUSH>
__global__ void __launch_bounds__(kThreadsP, 1)
    nbits_gemm_f16_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmSZ, const PParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* raw = smem;
  uint8_t* conv = smem + kRaw * kRawBytes;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(conv + kConv * kCBytes);
  uint64_t* raw_empty = raw_full + kRaw;
  uint64_t* conv_full = raw_empty + kRaw;
  uint64_t* conv_empty = conv_full + kConv;
  uint64_t* tm_full = conv_empty + kConv;
  uint64_t* tm_empty = tm_full + 2;
  uint64_t* fin = tm_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.K + PBK - 1) / PBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRaw; s++) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 1);
    }
    for (int c = 0; c < kConv; c++) {
      mbar_init(&conv_full[c], kConvWarps);
      mbar_init(&conv_empty[c], 1);
    }
    for (int d = 0; d < 2; d++) {
      mbar_init(&tm_full[d], 1);
      mbar_init(&tm_empty[d], 4);
    }
    mbar_init(fin, 1);
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&tmA);
      prefetch_tensormap(&tmQ);
      prefetch_tensormap(&tmSZ);
      uint32_t g = 0;
      int armed[kRaw];
      for (int s = 0; s < kRaw; s++) armed[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const int m0 = (t % p.m_tiles) * PBM, n0 = (t / p.m_tiles) * PBN;
        for (int kb = 0; kb < nk; kb++, g++) {
          const int s = g % kRaw;
          const uint32_t ph = (g / kRaw) & 1;
          if (!mbar_wait(&raw_empty[s], ph ^ 1)) {
            record_error(p.err, KERR_WAIT_EMPTY);
            ok = false;
            break;
          }
          uint8_t* st = raw + s * kRawBytes;
          armed[s] = (int)ph;
          mbar_arrive_expect_tx(&raw_full[s], p.stage_tx);
          tma_load_2d(st, &tmA, &raw_full[s], kb * PBK, m0);
          tma_load_2d(st + kABytes, &tmQ, &raw_full[s], kb * (PBK / 2), n0);
          tma_load_2d(st + kABytes + kQBytes, &tmSZ, &raw_full[s], n0,
                      (kb * PBK) >> p.bs_shift);
        }
      }
      if (!ok)
        for (int s = 0; s < kRaw; s++)
          if (armed[s] >= 0 && !mbar_wait(&raw_full[s], (uint32_t)armed[s]))
            record_error(p.err, KERR_WAIT_DRAIN);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_f16(0, kHalf, PBM);
      uint32_t g = 0, tcount = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, tcount++) {
        const int d = tcount & 1;
        if (!mbar_wait(&tm_empty[d], ((tcount >> 1) & 1) ^ 1)) {
          record_error(p.err, KERR_WAIT_EMPTY);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + d * PBM;  // 256 columns: one per row of the A tile
        for (int kb = 0; kb < nk; kb++, g++) {
          const int s = g % kRaw, c = g % kConv;
          if (!mbar_wait(&conv_full[c], (g / kConv) & 1)) {
            record_error(p.err, KERR_WAIT_FULL);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(raw + s * kRawBytes);
          const uint32_t sb = smem_u32(conv + c * kCBytes);
#pragma unroll
          for (int kk = 0; kk < PBK / 16; kk++)  // D[n, m] += W16[n, k] . A16[m, k]
            mma_f16_ss(dt, smem_desc_sw128(sb + kk * 32), smem_desc_sw128(sa + kk * 32), idesc,
                       (kb | kk) != 0);
          mma_commit(&raw_empty[s]);
          mma_commit(&conv_empty[c]);
        }
        if (ok) mma_commit(&tm_full[d]);
      }
      mma_commit(fin);
      if (!mbar_wait(fin, 0)) record_error(p.err, KERR_WAIT_MMA);
    }
    __syncwarp();
  } else if (warp < kConvWarp0 + kConvWarps) {
    // ---------------- converters: column n, words 4 hw .. 4 hw + 3 -------
    const int tid = threadIdx.x - kConvWarp0 * 32;
    const int n = tid & (PBN - 1), hw = tid / PBN;
    const uint32_t rowoff = (uint32_t)((n >> 3) * 1024 + (n & 7) * 128);
    const int sw = n & 7;
    uint32_t g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < nk; kb++, g++) {
        const int s = g % kRaw, c = g % kConv;
        if (!mbar_wait(&raw_full[s], (g / kRaw) & 1) ||
            !mbar_wait(&conv_empty[c], ((g / kConv) & 1) ^ 1)) {
          record_error(p.err, KERR_WAIT_FULL);
          ok = false;
          break;
        }
        const uint8_t* st = raw + s * kRawBytes;
        // the packed tile lands with the 32-byte swizzle (16-byte half h of
        // column n at n*32 + ((h ^ bit 2 of n) << 4)): the 8 columns a
        // quarter-warp reads then cover all 32 banks once
        const uint32_t qa = smem_u32(st + kABytes) + n * 32;
        const uint32_t sza = smem_u32(st + kABytes + kQBytes);  // the stage's table
        const uint32_t qsw = (uint32_t)((n >> 2) & 1) << 4;
        const uint4 w4 = lds128(qa + ((uint32_t)(hw << 4) ^ qsw));
        const uint32_t words[4] = {w4.x, w4.y, w4.z, w4.w};
        const uint32_t cb = smem_u32(conv + c * kCBytes) + rowoff;
        // word i holds k 8i..8i+7 and takes the {1024 + z, scale} entry of
        // its block within the stage's table
        auto convert = [&](const uint32_t (&vs)[4]) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int i = 4 * hw + j;
            const uint32_t v = vs[j];
            const uint32_t zz = prmt(v, v, 0x1010), sc = prmt(v, v, 0x3232);
            const uint32_t lo = words[j] & 0x0F0F0F0Fu, hi = (words[j] >> 4) & 0x0F0F0F0Fu;
            const uint32_t r0 = deq2(prmt(lo, 0x64646464u, 0x4140), zz, sc);  // k0, k1
            const uint32_t r1 = deq2(prmt(lo, 0x64646464u, 0x4342), zz, sc);  // k2, k3
            const uint32_t r2 = deq2(prmt(hi, 0x64646464u, 0x4140), zz, sc);  // k4, k5
            const uint32_t r3 = deq2(prmt(hi, 0x64646464u, 0x4342), zz, sc);  // k6, k7
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(cb + ((i ^ sw) << 4)),
                         "r"(r0), "r"(r1), "r"(r2), "r"(r3)
                         : "memory");
          }
        };
        if (p.bs_shift >= 6) {
          // a block of 64 or more k: one entry serves the whole stage (one
          // load, and its halves split once instead of per word)
          uint32_t v;
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(sza + (uint32_t)(n * 4)));
          const uint32_t vs[4] = {v, v, v, v};
          convert(vs);
        } else {
          uint32_t vs[4];  // all four loads issued before any use
#pragma unroll
          for (int j = 0; j < 4; j++)
            asm volatile("ld.shared.u32 %0, [%1];"
                         : "=r"(vs[j])
                         : "r"(sza + (uint32_t)((((8 * (4 * hw + j)) >> p.bs_shift) * PBN + n) * 4)));
          convert(vs);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv_full[c]);
      }
    }
  } else {
    // ---------------- epilogue ---------------------------------------------
    // warp q reads TMEM lanes 32q .. 32q + 31: weight columns n0 + 32q + lane
    const int q = warp & 3;
    uint32_t tcount = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, tcount++) {
      const int m0 = (t % p.m_tiles) * PBM, n0 = (t / p.m_tiles) * PBN;
      const int d = tcount & 1;
      const int n = n0 + q * 32 + lane;
      const int f = n < p.N ? p.col_exp[n] : 0;
      // the warp's destination: Y, or the part of a fused group its 32
      // columns lie in
      float* yb = p.Y;
      int64_t ld = p.ldy, cs = 0;
      if (p.nseg) {
        const int nc = n0 + q * 32;
#pragma unroll
        for (int u = 0; u < kMaxSegs; u++)
          if (u < p.nseg && nc >= p.seg_start[u]) {
            yb = p.seg_y[u];
            ld = p.seg_ld[u];
            cs = p.seg_start[u];
          }
      }
      if (!mbar_wait(&tm_full[d], (tcount >> 1) & 1)) {
        record_error(p.err, KERR_WAIT_MMA);
        break;
      }
      tc_fence_after();
      for (int c0 = 0; c0 < PBM; c0 += 32) {
        const int rbase = m0 + c0;
        const int my_e = rbase + lane < p.M ? p.row_exp[rbase + lane] : 0;
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + d * PBM + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int e = __shfl_sync(0xffffffffu, my_e, j);
          const int row = rbase + j;
          if (row < p.M && n < p.N) {
            const float v = scale_pow2(__uint_as_float(r[j]), e + f);
            yb[(int64_t)row * ld + (n - cs)] = v;
            if constexpr (PUSH) {  // the same value into every peer's landing block
#pragma unroll
              for (int u = 0; u < 8; u++)
                if (u < p.push.world && u != p.push.rank)
                  p.push.land[u][(int64_t)row * p.push.ns + n] = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tm_empty[d]);
    }
  }
  // push mode: this thread's stores to the peers are visible system-wide
  // before the CTA counts itself done; the last CTA posts the epoch
  if (PUSH) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (PUSH && threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(p.push.ticket, 1u) == gridDim.x - 1) {
      *p.push.ticket = 0u;
      __threadfence_system();
      for (int r = 0; r < p.push.world; r++)
        if (r != p.push.rank)
          asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.push.flag[r]),
                       "l"(p.push.epoch)
                       : "memory");
    }
  }
}

// {1024 + z, scale * 2^-f_n} per (block, column) as two fp16 halves, block
// major like the scales.
__global__ void nbits_sz16_kernel(const float* __restrict__ S, int64_t s_pitch,
                                  const uint8_t* __restrict__ Z, int64_t z_pitch, int nb, int nl,
                                  const int* __restrict__ col_exp, uint32_t* __restrict__ out) {
  const int64_t total = (int64_t)nb * nl;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / nl), n = (int)(i % nl);
    const float z = Z ? (float)nbits_zp(Z, z_pitch, n, b) : 8.0f;
    const float s = scale_pow2(S[(int64_t)b * s_pitch + n], -col_exp[n]);
    const uint32_t zh = __half_as_ushort(__float2half_rn(1024.0f + z));
    const uint32_t sh = __half_as_ushort(__float2half_rn(s));
    out[(int64_t)b * s_pitch + n] = zh | (sh << 16);
  }
}

}  // namespace

bool nbits_gemm_f16_layout_ok(const Weight& w) {
  const int64_t col_bytes = (int64_t)w.nb * w.bs / 2;
  return col_bytes % 16 == 0 && w.bs >= 16 && (w.bs & (w.bs - 1)) == 0;
}

bool nbits_gemm_f16_ok(const Weight& w) { return w.nl > 0 && nbits_gemm_f16_layout_ok(w); }

int prepare_nbits_sz16(const Weight& w, const int* col_exp, uint32_t* out, cudaStream_t st,
                       int64_t* launches) {
  const int64_t total = (int64_t)w.nb * w.nl;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 4096);
  nbits_sz16_kernel<<<blocks, 256, 0, st>>>(w.scales, w.s_pitch, w.has_zp ? w.zp : nullptr,
                                            w.z_pitch, w.nb, (int)w.nl, col_exp, out);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

int launch_nbits_gemm_f16(Weight& w, const uint16_t* A16, const int* row_exp, int64_t M,
                          const uint32_t* sz16, const int* col_exp, float* Y, int64_t ldy,
                          int* err, int sm_count, cudaStream_t st, int64_t* launches,
                          int reserve_sms, const PrefillPush* push, const YSel* seg) {
  if (M == 0 || w.nl == 0) return ORT_CUDA_OK;
  const int64_t K = w.K, nl = w.nl, col_bytes = (int64_t)w.nb * w.bs / 2;
  CUtensorMap tmA;
  int rc = encode_tma_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A16, (uint64_t)K, (uint64_t)M,
                         (uint64_t)K * 2, PBK, PBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  int bs_shift = 0;
  while ((1 << bs_shift) < w.bs) bs_shift++;
  const int bps = w.bs >= PBK ? 1 : PBK / w.bs;
  if (!w.prefill_maps) {  // the weight's views, once
    rc = encode_tma_2d(&w.tmQp, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.B, (uint64_t)col_bytes,
                       (uint64_t)nl, (uint64_t)col_bytes, PBK / 2, PBN, CU_TENSOR_MAP_SWIZZLE_32B);
    if (rc) return rc;
    rc = encode_tma_2d(&w.tmSZp, CU_TENSOR_MAP_DATA_TYPE_UINT32, sz16, (uint64_t)nl,
                       (uint64_t)w.nb, (uint64_t)w.s_pitch * 4, PBN, bps,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    w.prefill_maps = true;
  }
  const CUtensorMap& tmQ = w.tmQp;
  const CUtensorMap& tmSZ = w.tmSZp;
  PParams p;
  p.Y = Y;
  p.ldy = ldy;
  p.row_exp = row_exp;
  p.col_exp = col_exp;
  p.err = err;
  p.M = (int)M;
  p.N = (int)nl;
  p.K = (int)K;
  p.m_tiles = (int)((M + PBM - 1) / PBM);
  p.tiles = p.m_tiles * (int)((nl + PBN - 1) / PBN);
  p.bps = bps;
  p.bs_shift = bs_shift;
  p.stage_tx = kABytes + kQBytes + (uint32_t)bps * PBN * 4;
  if (push) p.push = *push;
  if (seg && seg->nseg > 0) {
    p.nseg = seg->nseg;
    for (int j = 0; j <= seg->nseg; j++) p.seg_start[j] = seg->seg_start[j];
    for (int j = 0; j < seg->nseg; j++) {
      p.seg_y[j] = seg->seg_y[j];
      p.seg_ld[j] = seg->seg_ld[j];
    }
  }
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load() >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(nbits_gemm_f16_kernel<false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemP));
    ORTC_CUDA(cudaFuncSetAttribute(nbits_gemm_f16_kernel<true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemP));
    if (dev < 64) configured.fetch_or(1ull << dev);
  }
  // persistent: one CTA per SM, leaving reserve_sms SMs to a kernel that
  // runs beside it (this GEMM's shared memory leaves no room on its SMs)
  const int grid = std::min(p.tiles, std::max(1, sm_count - reserve_sms));
  if (push)
    nbits_gemm_f16_kernel<true><<<grid, kThreadsP, kSmemP, st>>>(tmA, tmQ, tmSZ, p);
  else
    nbits_gemm_f16_kernel<false><<<grid, kThreadsP, kSmemP, st>>>(tmA, tmQ, tmSZ, p);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

}  // namespace ortc
