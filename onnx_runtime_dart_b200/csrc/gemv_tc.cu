// int4 block-quantised GEMV for decode (M <= 8) on tcgen05 tensor cores
// (kind::i8), exact integer products.
//
// Replaces, for small M, the reference's per-call dequantisation of all of B
// into an fp32 [K x N] buffer followed by matmulKernel's _gemv
// (onnx_qlinear_ops.dart:127-154, gemm_kernel_simd.dart:183-246).  Packed B
// streams from HBM exactly once.
//
// Arithmetic.  Y[m,n] = sum_b s[n,b] * sum_{k in b} a[m,k] * (q[k,n] - z[n,b]).
// Each activation row is turned into fixed point per 512-k chunk,
// X = rint(a * 2^S) with |X| <= 2^22 (S from the row's largest magnitude in
// the chunk), and split into three balanced base-256 digits
// X = c2*2^16 + c1*2^8 + c0.  The tensor core multiplies q (0..15) by each
// digit and accumulates in int32 with no rounding at all.  Per block, the
// epilogue forms D - z * sum(X) (the X build supplies sum(X) per block and
// row), then applies the fp32 block scale, and 2^-S at the end.  The only
// roundings are the fixed-point step of a (2^-23 of the chunk row's largest
// magnitude) and the fp32 operations of the epilogue.
//
// MMA orientation:
//   D[n, j] (128 TMEM lanes = 128 weight columns; NM = 16 or 32 columns j)
//     += Q[n, k..k+32) (A operand, int8, in TMEM) . X[j, k..k+32) (B, smem)
//   X is block-diagonal: within a region of G quantisation blocks, block
//   slot g owns columns j = (g*M + m)*3 + t (row m, digit t), so every block
//   of the region accumulates into its own D columns.  One MMA covers 128
//   columns x 32 k = 4096 weights.
//
// Roles (576 threads, one CTA per SM):
//   warp 16    TMA producer: per work item (128 columns x 512 k) the packed
//              tile (2 boxes, 128-byte swizzle), its scales and zero points,
//              into a shared-memory ring of up to 6 stages.
//   warps 0-7  dequantisers, 2 groups x 4 lane quarters: thread (quarter q,
//              lane l) owns weight column n = 32q + l.  Per 32-k stage: one
//              conflict-free 16-byte shared load and one mask (and a shift)
//              per 4 weights turn nibbles into bytes, then tcgen05.st of 8
//              TMEM columns.  They also build X per chunk.  This role is
//              instruction-bound: keep its per-weight work minimal.
//   warp 17    TMEM allocator; an elect.sync leader waits once per item and
//              issues its 16 MMAs (A from TMEM, stage table precomputed on
//              the host); tcgen05.commit frees A, X and D buffers.
//   warps 8-15 epilogue, 2 groups of 4 taking alternate items (tile-major:
//              alternate tiles): tcgen05.ld of D, zero points, block scales,
//              and the chunk partial of each column.
// Synchronisation is batched per item because an mbarrier wait costs about
// 200 cycles even when its phase has completed.
// Decomposition: tile-major (a CTA owns whole 128-column tiles and loops
// over the 512-k chunks, adding chunk partials in chunk order in shared
// memory) when the tiles spread evenly over the SMs, else split-K (CTAs own
// one chunk; a second kernel adds the chunk partials in chunk order).  Both
// form ((0 + p_0) + p_1) + ... from identical partials, and the partials
// depend on K only, so results never depend on N or on which columns a GPU
// owns: N-sharded results are bitwise equal to 1-GPU results.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

#include <atomic>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace ortc {
namespace {

constexpr int kTile = 128;          // weight columns per item (MMA M)
constexpr int kChunkK = 512;        // k per item
constexpr int kItemStages = 16;     // 32-k stages per item, one MMA each
constexpr int kAItems = 2;          // TMEM A ring: two items of 16 x 8 columns
constexpr int kMaxBStages = 6;      // shared-memory ring depth (runtime <= 6)
constexpr int kDeWarps = 8;         // dequantisers: 2 groups x 4 lane quarters
constexpr int kEpiWarp0 = 8;        // epilogue: 2 groups of 4 warps, 8..15
constexpr int kEpiWarps = 8;
constexpr int kProducerWarp = 16, kMmaWarp = 17, kXWarp = 18;
constexpr int kThreadsTC = 19 * 32;
constexpr int kMinBs = 32;          // one MMA never spans two blocks
constexpr uint32_t kPackedBytes = kTile * kChunkK / 2;  // 32 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAItemCols = kItemStages * 8;        // 128 columns per item
constexpr uint32_t kDCol = kAItems * kAItemCols;         // D starts at column 256
constexpr uint32_t kDCols = kTmemCols - kDCol;          // 256 columns for D
constexpr int kMaxBpi = kChunkK / kMinBs;               // blocks per item
constexpr uint32_t kXBytesMax = 32 * kChunkK;           // X for NM = 32
// X buffer: X, then the rows' largest-magnitude bits [8] and exponents [8],
// the blocks' sums of X [bpi][M] (exact, int64) and their fp32 values.
constexpr uint32_t kXRmax = kXBytesMax, kXRexp = kXBytesMax + 32, kXCsum = kXBytesMax + 64;
constexpr uint32_t kXXsum = kXCsum + kMaxBpi * 8 * 3 * 4;
constexpr uint32_t kXBufBytes = (kXXsum + kMaxBpi * 8 * 4 + 1023) & ~1023u;
constexpr size_t kSmemLimit = 227 * 1024;
constexpr int kNonFinite = -100000;  // exponent of a chunk row holding an inf or NaN

// Shared memory staging two chunks of A for the X builder: M >= 3 rows
// (M <= 2 keep the next chunk in registers) when the rows allow 16-byte
// bulk copies.
__host__ __device__ constexpr uint32_t a_stage_bytes(int64_t M, int a_vec) {
  return (M >= 3 && a_vec) ? (uint32_t)(2 * M * kChunkK * 4) : 0u;
}

// Compile-time shape of the X operand for M rows.
template <int M>
struct XShape {
  static constexpr int G = M == 1 ? 5 : (M == 2 ? 2 : 1);     // blocks per D region
  static constexpr int NM = (3 * M * G <= 16) ? 16 : 32;      // MMA N
};

struct TcParams {
  const float* A;
  float* Y;
  float* part;   // split-K mode: [nch][M][tiles*128] chunk partials
  YSel ysel;     // tile-major output redirected to a peer-exchange half
  int* err;
  int64_t ldy;
  int N, K, bs, bs_log2, nch, tiles;  // bs a power of two
  int tile_major;  // 1: a CTA loops over chunks [c0, c1) of its tile set
  int csize;       // tile-major: CTAs per cluster (1: no cluster); rank r
                   // takes chunks [r*nch/csize, (r+1)*nch/csize)
  int ncl;         // tile-major: tile sets; set s owns tiles s + i*ncl
  uint32_t yacc_bytes;  // csize 1: chunk-order sums; else the partials inbox
  int tg;          // tile-major: tiles per group (chunks outer in a group)
  int cpc;         // split-K: CTAs per chunk
  int bpi, regions, has_zp, z_rows, nbst;
  int a_vec;       // A 16-byte aligned and K % 4 == 0: 16-byte activation loads
  int nd;          // D buffers: 2, or 1 when an item needs more than 128 columns
  uint32_t dstride;
  // Per 32-k stage of an item: D column offset of its region and whether it
  // accumulates (bit st of acc_mask).  Computed on the host so the issuing
  // thread does no integer division.
  uint32_t op_d[kItemStages];
  uint32_t acc_mask;
  int s16;         // block scales streamed as fp16 (widened exactly in the epilogue)
  uint32_t stage_bytes, stage_tx, s_off, z_off, yacc_off;
  uint32_t a_off;  // M >= 3 with 16-byte activation rows: staging of 2 chunks of A
};

// Calls f(tile, chunk, tile_in_group) for this CTA's work items, in the
// order every role of the CTA follows; stops early when f returns false.
template <typename F>
__device__ __forceinline__ void for_each_item(const TcParams& p, F&& f) {
  if (p.tile_major) {
    const int set = (int)blockIdx.x / p.csize, rank = (int)blockIdx.x % p.csize;
    const int c0 = rank * p.nch / p.csize, c1 = (rank + 1) * p.nch / p.csize;
    const int span = p.ncl * p.tg;
    for (int g0 = set; g0 < p.tiles; g0 += span)
      for (int c = c0; c < c1; c++)
        for (int i = 0; i < p.tg; i++) {
          const int t = g0 + i * p.ncl;
          if (t >= p.tiles) break;
          if (!f(t, c, i)) return;
        }
  } else {
    const int c = blockIdx.x % p.nch;
    for (int t = blockIdx.x / p.nch; t < p.tiles; t += p.cpc)
      if (!f(t, c, 0)) return;
  }
}

// Bounded barrier among a fixed set of warps: every participating warp
// arrives once (lane 0) and all lanes wait for the phase to complete.
__device__ __forceinline__ bool warp_group_sync(uint64_t* bar, uint32_t& phase, int* err) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1;
  if (!ok) record_error(err, KERR_WAIT_FULL);
  return ok;
}

__device__ __forceinline__ float pow2f(int e) {
  return __uint_as_float((uint32_t)(e + 127) << 23);
}
// v * 2^e for |e| up to a few hundred, exact unless the result leaves the
// normal range.
__device__ __forceinline__ float scale_pow2(float v, int e) {
  while (e > 100) { v *= pow2f(100); e -= 100; }
  while (e < -100) { v *= pow2f(-100); e += 100; }
  return v * pow2f(e);
}

// X (int8, K-major, 128-byte swizzle): 128-k atoms of NM rows x 128 bytes,
// 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint32_t x_addr(uint32_t base, int nm, int j, int k) {
  const int atom = k >> 7, kin = k & 127, r = j & 7;
  return base + atom * (nm * 128) + (j >> 3) * 1024 + r * 128 + (((kin >> 4) ^ r) << 4) +
         (kin & 15);
}

// Scale of one row of a chunk: S with |rint(a * 2^S)| <= 2^22 for every a
// of the row (mb: its largest magnitude as bits; inf and NaN compare above
// 0x7f7fffff and give kNonFinite), and 2^S as two exact power-of-two
// factors applied as (a * f1) * f2, since |S| may exceed a float exponent.
struct RowScale {
  int S;
  float f1, f2;
};
__device__ __forceinline__ RowScale row_scale(unsigned mb) {
  RowScale r;
  r.S = 0;
  if (mb > 0x7f7fffffu) {
    r.S = kNonFinite;
  } else if (mb != 0) {
    int ex;
    frexpf(__uint_as_float(mb), &ex);  // max < 2^ex
    r.S = 22 - ex;
  }
  const int e = r.S == kNonFinite ? 0 : r.S;
  if (e > 100) {
    r.f1 = pow2f(100);
    r.f2 = pow2f(e - 100);
  } else if (e < -100) {
    r.f1 = pow2f(-100);
    r.f2 = pow2f(e + 100);
  } else {
    r.f1 = pow2f(e);
    r.f2 = 1.0f;
  }
  return r;
}

// X = rint(a * 2^S) of four consecutive activations of a row, as three
// words of int8 digits (word t holds digit t of the four values, X = c2 *
// 65536 + c1 * 256 + c0 with every c in [-128, 127]) and the sum of the four
// X.  With U = X + 0x808080 (0 <= U < 2^24 since |X| <= 2^22), byte t of
// U ^ 0x808080 is c_t as an int8; byte permutes gather the words.
__device__ __forceinline__ void x_digits(float4 a, const RowScale& r, uint32_t& w0, uint32_t& w1,
                                         uint32_t& w2, int& sx) {
  int X0 = 0, X1 = 0, X2 = 0, X3 = 0;
  if (r.S != kNonFinite) {
    X0 = __float2int_rn((a.x * r.f1) * r.f2);
    X1 = __float2int_rn((a.y * r.f1) * r.f2);
    X2 = __float2int_rn((a.z * r.f1) * r.f2);
    X3 = __float2int_rn((a.w * r.f1) * r.f2);
  }
  sx = (X0 + X1) + (X2 + X3);
  const uint32_t V0 = (uint32_t)(X0 + 0x808080) ^ 0x808080u;
  const uint32_t V1 = (uint32_t)(X1 + 0x808080) ^ 0x808080u;
  const uint32_t V2 = (uint32_t)(X2 + 0x808080) ^ 0x808080u;
  const uint32_t V3 = (uint32_t)(X3 + 0x808080) ^ 0x808080u;
  const uint32_t lo01 = __byte_perm(V0, V1, 0x5140), lo23 = __byte_perm(V2, V3, 0x5140);
  const uint32_t hi01 = __byte_perm(V0, V1, 0x7362), hi23 = __byte_perm(V2, V3, 0x7362);
  w0 = __byte_perm(lo01, lo23, 0x5410);
  w1 = __byte_perm(lo01, lo23, 0x7632);
  w2 = __byte_perm(hi01, hi23, 0x5410);
}

// EXT: the stores go through ysel_store (push to peers, segmented output of
// a fused group, fused ArgMax keys); without it, the plain stores of a
// single-GPU or pull-mode call, with none of those branches in the epilogue.
template <int M, bool EXT>
__global__ void __launch_bounds__(kThreadsTC, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmS,
                   const __grid_constant__ CUtensorMap tmZ, const TcParams p) {
  constexpr int G = XShape<M>::G, NM = XShape<M>::NM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* Xs = smem;  // two buffers, each X then the digit sums
  uint8_t* Bs = smem + 2 * kXBufBytes;
  float* yacc = reinterpret_cast<float*>(smem + p.yacc_off);  // [tg][M][128]
  uint8_t* As = smem + p.a_off;  // [2][M][kChunkK] fp32 when staging
  uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + p.a_off + a_stage_bytes(M, p.a_vec));
  uint64_t* bempty = bfull + kMaxBStages;
  // ready[h]: item j = 2p + h may be issued (phase p): its A is written (8
  // dequantiser warps) and its D buffer is free (4 epilogue warps, after
  // reading item j - nd).  One barrier, so the issuer waits once per item.
  uint64_t* ready = bempty + kMaxBStages;
  uint64_t* aempty = ready + kAItems;      // [2] an item's A consumed (MMA commit)
  // dfull[2 g + d]: the D of epilogue group g's next item in D buffer d is
  // complete (MMA commit).  Each barrier is waited by one group, in item
  // order, and the MMA cannot commit that group's next item in buffer d
  // before the group released the previous one, so a barrier never runs a
  // phase ahead of its waiter.  (A parity wait on a barrier two phases ahead
  // would never return: one barrier per group alone allows that when a group
  // owns two consecutive items in different D buffers.)
  uint64_t* dfull = aempty + kAItems;
  uint64_t* xfull = dfull + 4;    // [2] X buffer written
  uint64_t* xempty = xfull + 2;   // [2] X buffer released (MMA commit + 8 epilogue warps)
  uint64_t* fin = xempty + 2;
  uint64_t* xsync = fin + 1;      // dequantisers, inside a split-K X build
  // cluster mode: every epilogue warp of the cluster has delivered its
  // partials of this CTA's tiles (remote arrivals, csize x 8)
  uint64_t* ibar = xsync + 1;
  uint64_t* abar = ibar + 1;  // [2] a chunk of A staged (bulk copies, M >= 3)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(abar + 2);
  // fused ArgMax: the CTA's row keys, column-0 NaN flags, last-CTA flag
  unsigned long long* s_amax = reinterpret_cast<unsigned long long*>(tmem_slot + 2);
  unsigned* s_nan0 = reinterpret_cast<unsigned*>(s_amax + 8);
  unsigned* s_last = s_nan0 + 1;
  const bool clustered = p.tile_major && p.csize > 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxBStages; s++) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], kDeWarps + 4);
    }
    for (int h = 0; h < kAItems; h++) {
      mbar_init(&ready[h], kDeWarps + 4);
      mbar_init(&aempty[h], 1);
    }
    for (int d = 0; d < 4; d++) mbar_init(&dfull[d], 1);
    for (int d = 0; d < 2; d++) {
      mbar_init(&xfull[d], p.tile_major ? 1 : kDeWarps);
      mbar_init(&xempty[d], 1 + kEpiWarps);
    }
    mbar_init(fin, 1);
    mbar_init(xsync, kDeWarps);
    if (EXT) {
      for (int m = 0; m < 8; m++) s_amax[m] = 0ull;
      *s_nan0 = 0u;
    }
    mbar_init(ibar, p.csize * kEpiWarps);
    mbar_init(&abar[0], 1);
    mbar_init(&abar[1], 1);
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // other CTAs of the cluster may arrive on ibar once every CTA has passed
  // this point (each thread waits before its first remote access)
  if (clustered) cluster_arrive_relaxed();
  const uint32_t tmem = *tmem_slot;
  // The next kernel in the stream may start its prologue and weight stream
  // as our CTAs retire; it waits for our completion before touching
  // activations or outputs (griddep_wait).
  griddep_launch_dependents();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      prefetch_tensormap(&tmB);
      prefetch_tensormap(&tmS);
      if (p.has_zp) prefetch_tensormap(&tmZ);
      const uint64_t pol = policy_evict_first();
      int j = 0, armed[kMaxBStages];
      for (int s = 0; s < kMaxBStages; s++) armed[s] = -1;
      bool ok = true;
      for_each_item(p, [&](int tile, int chunk, int) {
        const int bst = j % p.nbst;
        const uint32_t ph = (j / p.nbst) & 1;
        if (!mbar_wait(&bempty[bst], ph ^ 1)) {
          record_error(p.err, KERR_WAIT_EMPTY);
          return ok = false;
        }
        uint8_t* st = Bs + bst * p.stage_bytes;
        armed[bst] = (int)ph;
        mbar_arrive_expect_tx(&bfull[bst], p.stage_tx);
        const int first_b = chunk * p.bpi;
        tma_load_2d_hint(st, &tmB, &bfull[bst], chunk * 256, tile * kTile, pol);
        tma_load_2d_hint(st + 16384, &tmB, &bfull[bst], chunk * 256 + 128, tile * kTile, pol);
        tma_load_2d(st + p.s_off, &tmS, &bfull[bst], tile * kTile, first_b);
        if (p.has_zp) tma_load_2d(st + p.z_off, &tmZ, &bfull[bst], tile * kTile, first_b >> 1);
        j++;
        return true;
      });
      if (!ok)
        for (int s = 0; s < p.nbst; s++)
          if (armed[s] >= 0 && !mbar_wait(&bfull[s], (uint32_t)armed[s]))
            record_error(p.err, KERR_WAIT_DRAIN);
    }
  } else if (warp == kMmaWarp) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_i8(128, NM);
      // the stage table and D layout, read before the first wait (a first
      // read of a kernel parameter can miss the constant cache)
      asm volatile("" ::"r"(p.op_d[0]), "r"(p.op_d[kItemStages - 1]), "r"(p.acc_mask), "r"(p.nd),
                   "r"(p.dstride));
      int j = 0, cur = -1, nbuild = 0;
      for_each_item(p, [&](int, int chunk, int tig) {
        if (chunk != cur) {
          if (cur >= 0) mma_commit(&xempty[(nbuild - 1) & 1]);  // X free once its MMAs end
          if (!mbar_wait(&xfull[nbuild & 1], (nbuild >> 1) & 1)) {
            record_error(p.err, KERR_WAIT_FULL);
            return false;
          }
          cur = chunk;
          nbuild++;
        }
        const uint32_t xb = smem_u32(Xs + ((nbuild - 1) & 1) * kXBufBytes);
        const int d = j % p.nd;
        const uint32_t dbase = tmem + kDCol + d * p.dstride;
        // One wait per item: a wait on the issuing thread stalls behind the
        // MMAs still in flight, so it is paid once per 16 MMAs.
        const int h = j % kAItems;
        if (!mbar_wait(&ready[h], (j / kAItems) & 1)) {
          record_error(p.err, KERR_WAIT_FULL);
          return false;
        }
        tc_fence_after();
        const uint32_t abase = tmem + h * kAItemCols;
        const uint64_t xd0 = smem_desc_sw128(xb);
#pragma unroll
        for (int st = 0; st < kItemStages; st++) {
          // X atom (st / 4), 32-byte k step (st % 4) inside the swizzle atom
          const uint32_t xoff = ((st >> 2) * (NM * 128) + (st & 3) * 32) >> 4;
          mma_i8_ts(dbase + p.op_d[st], abase + st * 8, xd0 + xoff, idesc, (p.acc_mask >> st) & 1u);
        }
        mma_commit(&aempty[h]);
        mma_commit(&dfull[(((p.tile_major && !clustered) ? tig : j) & 1) * 2 + d]);
        j++;
        return true;
      });
      mma_commit(fin);
      if (!mbar_wait(fin, 0)) record_error(p.err, KERR_WAIT_MMA);
    }
    __syncwarp();
  } else if (warp == kXWarp && p.tile_major) {
    // ---------------- X builder (tile-major) ----------------
    // One warp builds X, the row exponents and the blocks' sums of X for
    // chunk c + 1 as soon as its buffer is free, while the dequantisers
    // stream chunk c.  (Split-K CTAs build their single chunk once, at the
    // start and on the critical path: the dequantiser warps do that
    // together, below.)  Unit i (< 4M) of a lane is 4 consecutive k of row
    // i / 4 at k = 4 (lane + 32 (i % 4)); for M <= 2 the next chunk's units
    // are loaded right after a build, so a build does not wait for them.
    for (int i = lane; i < 2 * (int)kXBufBytes / 16; i += 32)
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(smem_u32(Xs) + i * 16), "r"(0u)
                   : "memory");
    // Every parameter the builds use, read before the dependency wait: a
    // first read of a kernel parameter can miss the constant cache, and
    // after the wait it would delay the first X.
    const int seg = min(32, p.bs / 4);  // lanes whose units share a block
    // the aligned run of `seg` lanes holding this lane's block
    const unsigned segmask =
        seg == 32 ? 0xffffffffu : ((1u << seg) - 1u) << (lane & ~(seg - 1));
    const int rank = (int)blockIdx.x % p.csize;
    const int c_first = rank * p.nch / p.csize, c_end = (rank + 1) * p.nch / p.csize;
    const float* const Ap = p.A;
    const int K = p.K, a_vec = p.a_vec, bs_log2 = p.bs_log2, bpi = p.bpi;
    asm volatile("" ::"l"(Ap), "r"(K), "r"(a_vec), "r"(bs_log2), "r"(bpi), "r"(c_first),
                 "r"(c_end), "r"(segmask));
    __syncwarp();
    griddep_wait();  // activations come from the previous kernel in the stream
    auto load = [&](int chunk, int i) {
      const int m = i >> 2, k = chunk * kChunkK + (lane + 32 * (i & 3)) * 4;
      const float* src = Ap + (int64_t)m * K + k;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a_vec && k + 3 < K) {
        a = __ldg(reinterpret_cast<const float4*>(src));
      } else {
        if (k < K) a.x = src[0];
        if (k + 1 < K) a.y = src[1];
        if (k + 2 < K) a.z = src[2];
        if (k + 3 < K) a.w = src[3];
      }
      return a;
    };
    constexpr int kPre = M <= 2 ? 4 * M : 1;
    float4 pre[kPre];  // M <= 2: the units of chunk pre_chunk
    int pre_chunk = -1;
    // M >= 3: chunks of A arrive by bulk copies into two staging buffers,
    // build n reading buffer n & 1; the copy for the next chunk is issued as
    // soon as a build starts, so it lands while the build runs
    const bool staged = a_stage_bytes(M, a_vec) != 0;
    auto issue = [&](int chunk, int buf) {
      const int k0 = chunk * kChunkK;
      const uint32_t bytes = (uint32_t)min(kChunkK, K - k0) * 4;
      mbar_arrive_expect_tx(&abar[buf], bytes * M);
#pragma unroll
      for (int m = 0; m < M; m++)
        bulk_load(As + (buf * M + m) * kChunkK * 4, Ap + (int64_t)m * K + k0, bytes, &abar[buf]);
    };
    int issued = 0, waited = 0;  // staged copies requested / completed (copy n: build n)
    bool ok = true;
    int cur = -1, nbuild = 0;
    for_each_item(p, [&](int, int chunk, int) {
      if (!ok) return false;
      if (chunk == cur) return true;
      cur = chunk;
      if (M <= 2 && pre_chunk != chunk) {
#pragma unroll
        for (int i = 0; i < kPre; i++) pre[i] = load(chunk, i);
      }
      const uint8_t* abuf = As + (nbuild & 1) * M * kChunkK * 4;
      if (staged) {
        if (issued == nbuild) {  // the first build: nothing was prefetched
          if (lane == 0) issue(chunk, nbuild & 1);
          issued++;
        }
        if (!mbar_wait(&abar[nbuild & 1], (nbuild >> 1) & 1)) {
          record_error(p.err, KERR_WAIT_FULL);
          return ok = false;
        }
        waited++;
        // buffer (n + 1) & 1 was last read by build n - 1, which has ended
        const int nx = chunk + 1 < c_end ? chunk + 1 : c_first;
        if (lane == 0) issue(nx, (nbuild + 1) & 1);
        issued++;
      }
      const int k0s = chunk * kChunkK;
      // unit i of this lane: registers (M <= 2), the staging buffer, or A
      auto unit = [&](int i) {
        if (M <= 2) return pre[M <= 2 ? i : 0];
        if (!staged) return load(chunk, i);
        const int m = i >> 2, kk = (lane + 32 * (i & 3)) * 4;
        if (k0s + kk >= K) return make_float4(0.f, 0.f, 0.f, 0.f);
        return lds128f(smem_u32(abuf + (m * kChunkK + kk) * 4));
      };
      const int xbuf = nbuild & 1;
      if (!mbar_wait(&xempty[xbuf], ((nbuild >> 1) & 1) ^ 1)) {
        record_error(p.err, KERR_WAIT_EMPTY);
        return ok = false;
      }
      uint8_t* xbase = Xs + xbuf * kXBufBytes;
      int* rexp = reinterpret_cast<int*>(xbase + kXRexp);              // [8]
      long long* csum = reinterpret_cast<long long*>(xbase + kXCsum);  // [bpi][M]
      float* xsum = reinterpret_cast<float*>(xbase + kXXsum);          // [bpi][M]
      for (int i = lane; i < bpi * M; i += 32) csum[i] = 0;
      RowScale rs[M];
#pragma unroll
      for (int m = 0; m < M; m++) {
        unsigned mb = 0;
#pragma unroll
        for (int i = 4 * m; i < 4 * m + 4; i++) {
          const float4 a = unit(i);
          mb = max(mb, max(max(__float_as_uint(a.x) & 0x7fffffffu, __float_as_uint(a.y) & 0x7fffffffu),
                           max(__float_as_uint(a.z) & 0x7fffffffu, __float_as_uint(a.w) & 0x7fffffffu)));
        }
        rs[m] = row_scale(__reduce_max_sync(0xffffffffu, mb));
        if (lane == 0) rexp[m] = rs[m].S;
      }
      __syncwarp();
      const uint32_t xb = smem_u32(xbase);
      // per row, three passes, so that the units' independent work overlaps:
      // digits and stores, the blocks' sums over their runs of lanes, the
      // leaders' adds (|sum| <= 2^29; a block always has the same leader
      // lane, so its adds are ordered)
#pragma unroll
      for (int m = 0; m < M; m++) {
        int sx[4];
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) {
          const int i = 4 * m + q4, k = (lane + 32 * q4) * 4;
          const int slot = (k >> bs_log2) % G;
          uint32_t w0, w1, w2;
          x_digits(unit(i), rs[m], w0, w1, w2, sx[q4]);
          const int jr = (slot * M + m) * 3;
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(x_addr(xb, NM, jr, k)), "r"(w0) : "memory");
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(x_addr(xb, NM, jr + 1, k)), "r"(w1)
                       : "memory");
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(x_addr(xb, NM, jr + 2, k)), "r"(w2)
                       : "memory");
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) sx[q4] = __reduce_add_sync(segmask, sx[q4]);
        if ((lane & (seg - 1)) == 0) {
#pragma unroll
          for (int q4 = 0; q4 < 4; q4++)
            csum[(((lane + 32 * q4) * 4) >> bs_log2) * M + m] += sx[q4];
        }
      }
      if (M <= 2) {  // the next chunk this CTA builds (or a harmless reload)
        const int nx = chunk + 1 < c_end ? chunk + 1 : c_first;
#pragma unroll
        for (int i = 0; i < kPre; i++) pre[i] = load(nx, i);
        pre_chunk = nx;
      }
      __syncwarp();
      // each block's sum of X per row, for the zero-point term z * sum X
      for (int i = lane; i < bpi * M; i += 32) xsum[i] = (float)csum[i];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&xfull[xbuf]);
      nbuild++;
      return true;
    });
    // copies still in flight (the last prefetch) land before the CTA's
    // shared memory is released; copy j is phase j >> 1 of abar[j & 1]
    for (int j = waited; j < issued; j++)
      if (!mbar_wait(&abar[j & 1], (j >> 1) & 1)) {
        record_error(p.err, KERR_WAIT_DRAIN);
        break;
      }
  } else if (warp < kDeWarps) {
    // ---------------- dequantisers ----------------
    const int q = warp & 3, grp = warp >> 2;
    const int nl = q * 32 + lane;  // column within the tile = TMEM lane
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    bool ok = true;
    if (!p.tile_major) {
      // the CTA's one chunk: X, digit sums, row exponents, all 8 warps
      for (int i = threadIdx.x; i < 2 * (int)kXBufBytes / 16; i += kDeWarps * 32)
        asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(smem_u32(Xs) + i * 16),
                     "r"(0u)
                     : "memory");
      uint32_t xph = 0;
      ok = warp_group_sync(xsync, xph, p.err);
      // parameters of the build, read before the dependency wait
      asm volatile("" ::"l"(p.A), "r"(p.K), "r"(p.a_vec), "r"(p.bs_log2), "r"(p.bs), "r"(p.bpi));
      griddep_wait();  // activations come from the previous kernel in the stream
      constexpr int kU = kChunkK / 4;  // 4-k units per row
      constexpr int kPer = (M * kU + kDeWarps * 32 - 1) / (kDeWarps * 32);
      const int chunk = (int)(blockIdx.x % p.nch), xbuf = 0;
      {
        // into buffer 0 (first use: free)
        uint8_t* xbase = Xs + xbuf * kXBufBytes;
        unsigned* rmax = reinterpret_cast<unsigned*>(xbase + kXRmax);    // [8]
        int* rexp = reinterpret_cast<int*>(xbase + kXRexp);              // [8]
        long long* csum = reinterpret_cast<long long*>(xbase + kXCsum);  // [bpi][M]
        float* xsum = reinterpret_cast<float*>(xbase + kXXsum);          // [bpi][M]
        if (threadIdx.x < 8) rmax[threadIdx.x] = 0;
        for (int i = threadIdx.x; i < p.bpi * M; i += kDeWarps * 32) csum[i] = 0;
        if (ok && !warp_group_sync(xsync, xph, p.err)) ok = false;
        // Activations of the chunk, unit u = 4 consecutive k of row u / kU.
        // A warp's 32 units lie in one row.
        const int k0 = chunk * kChunkK;
        float4 av[kPer];
#pragma unroll
        for (int i = 0; i < kPer; i++) {
          const int u = threadIdx.x + i * kDeWarps * 32;
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
          if (u < M * kU) {
            const int m = u / kU, k = k0 + (u % kU) * 4;
            const float* src = p.A + (int64_t)m * p.K + k;
            if (p.a_vec && k + 3 < p.K) {
              a = __ldg(reinterpret_cast<const float4*>(src));
            } else {
              if (k < p.K) a.x = src[0];
              if (k + 1 < p.K) a.y = src[1];
              if (k + 2 < p.K) a.z = src[2];
              if (k + 3 < p.K) a.w = src[3];
            }
            // largest magnitude as bits; inf and NaN compare above 0x7f7fffff
            const unsigned mb = max(max(__float_as_uint(a.x) & 0x7fffffffu, __float_as_uint(a.y) & 0x7fffffffu),
                                    max(__float_as_uint(a.z) & 0x7fffffffu, __float_as_uint(a.w) & 0x7fffffffu));
            const unsigned wm = __reduce_max_sync(0xffffffffu, mb);
            if (lane == 0) atomicMax(&rmax[m], wm);
          }
          av[i] = a;
        }
        if (ok && !warp_group_sync(xsync, xph, p.err)) ok = false;
        const uint32_t xb = smem_u32(xbase);
#pragma unroll
        for (int i = 0; i < kPer; i++) {
          const int u = threadIdx.x + i * kDeWarps * 32;
          if (u >= M * kU) continue;
          const int m = u / kU, k = (u % kU) * 4;
          const int bl = k >> p.bs_log2, slot = bl % G;
          const RowScale rs = row_scale(rmax[m]);
          if ((u % kU) == 0) rexp[m] = rs.S;
          uint32_t w0, w1, w2;
          int sx;
          x_digits(av[i], rs, w0, w1, w2, sx);
          const int jr = (slot * M + m) * 3;
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(x_addr(xb, NM, jr, k)), "r"(w0) : "memory");
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(x_addr(xb, NM, jr + 1, k)), "r"(w1)
                       : "memory");
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(x_addr(xb, NM, jr + 2, k)), "r"(w2)
                       : "memory");
          // the block's sum of X: a warp's 32 units are 128 consecutive k of
          // one row, a block an aligned run of min(32, bs / 4) of its lanes;
          // one reduction per run, one atomic per run (blocks over 128 k
          // span several warps)
          const int seg = min(32, p.bs / 4);
          const unsigned segmask =
              seg == 32 ? 0xffffffffu : ((1u << seg) - 1u) << (lane & ~(seg - 1));
          sx = __reduce_add_sync(segmask, sx);
          if ((lane & (seg - 1)) == 0)
            atomicAdd(reinterpret_cast<unsigned long long*>(csum + bl * M + m),
                      (unsigned long long)(long long)sx);
        }
        if (ok && !warp_group_sync(xsync, xph, p.err)) ok = false;
        // each block's sum of X per row, for the zero-point term z * sum X
        for (int i = threadIdx.x; i < p.bpi * M; i += kDeWarps * 32) xsum[i] = (float)csum[i];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&xfull[xbuf]);
      }
    }
    int j = 0;
    for_each_item(p, [&](int, int, int) {
      if (!ok) return false;
      const int bst = j % p.nbst;
      if (!mbar_wait(&bfull[bst], (j / p.nbst) & 1)) {
        record_error(p.err, KERR_WAIT_FULL);
        return ok = false;
      }
      const uint32_t sB = smem_u32(Bs + bst * p.stage_bytes);
      const int h = j % kAItems;
      if (!mbar_wait(&aempty[h], ((j / kAItems) & 1) ^ 1)) {
        record_error(p.err, KERR_WAIT_EMPTY);
        return ok = false;
      }
      tc_fence_after();
      const uint32_t abase = tmem + lane_addr + h * kAItemCols;
#pragma unroll
      for (int i = 0; i < kItemStages / 2; i++) {
        const int s = 2 * i + grp;
        // 16 bytes = 32 k of column nl: words hold k 0-7, 8-15, 16-23, 24-31;
        // low nibbles of a word's bytes are its first 4 k, high nibbles the next 4.
        const uint4 w4 = lds128(sB + (s >> 3) * 16384 + nl * 128 + (((s & 7) ^ (nl & 7)) << 4));
        const uint4 lo = make_uint4(w4.x & 0x0F0F0F0Fu, (w4.x >> 4) & 0x0F0F0F0Fu,
                                    w4.y & 0x0F0F0F0Fu, (w4.y >> 4) & 0x0F0F0F0Fu);
        const uint4 hi = make_uint4(w4.z & 0x0F0F0F0Fu, (w4.z >> 4) & 0x0F0F0F0Fu,
                                    w4.w & 0x0F0F0F0Fu, (w4.w >> 4) & 0x0F0F0F0Fu);
        tmem_st8(abase + s * 8, lo, hi);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[h]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bempty[bst]);
      j++;
      return true;
    });
  } else if (warp < kEpiWarp0 + kEpiWarps) {
    // ---------------- epilogue ----------------
    // Two groups share the items.  Tile-major without a cluster: a tile's
    // items always go to the group of its tile-in-group parity, so its chunk
    // sums in shared memory stay in chunk order; otherwise items alternate.
    const int q = warp & 3, egrp = (warp - kEpiWarp0) >> 2;
    const int nl = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    // the first nd items find their D buffers free
    if (lane == 0 && egrp == 0)
      for (int e = 0; e < p.nd; e++) mbar_arrive(&ready[e]);
    griddep_wait();  // outputs and split-K scratch may still be in use upstream
    const unsigned long long ep = EXT ? ysel_epoch(p.ysel) : 0ull;  // push mode's tag
    __syncwarp();    // .aligned cluster barrier: the whole warp, converged
    if (clustered) cluster_wait();
    const int set = (int)blockIdx.x / p.csize;
    bool ok = true;
    int S_m[M];
    int j = 0, cur = -1, nbuild = 0, mine[2] = {0, 0};  // waits done per D buffer
    for_each_item(p, [&](int tile, int chunk, int tig) {
      if (!ok) return false;
      if (chunk != cur) {
        if (cur >= 0) {  // done with the previous buffer's digit sums
          __syncwarp();
          if (lane == 0) mbar_arrive(&xempty[(nbuild - 1) & 1]);
        }
        if (!mbar_wait(&xfull[nbuild & 1], (nbuild >> 1) & 1)) {
          record_error(p.err, KERR_WAIT_FULL);
          return ok = false;
        }
        const int* rexp = reinterpret_cast<const int*>(Xs + (nbuild & 1) * kXBufBytes + kXRexp);
#pragma unroll
        for (int m = 0; m < M; m++) S_m[m] = rexp[m];
        cur = chunk;
        nbuild++;
      }
      if ((((p.tile_major && !clustered) ? tig : j) & 1) != egrp) {
        j++;
        return true;
      }
      const int bst = j % p.nbst, d = j % p.nd;
      if (!mbar_wait(&bfull[bst], (j / p.nbst) & 1) ||
          !mbar_wait(&dfull[egrp * 2 + d], mine[d] & 1)) {
        record_error(p.err, KERR_WAIT_MMA);
        return ok = false;
      }
      mine[d]++;
      tc_fence_after();
      float y[M];
#pragma unroll
      for (int m = 0; m < M; m++) y[m] = 0.0f;
      const uint8_t* stg = Bs + bst * p.stage_bytes;
      const float* stile = reinterpret_cast<const float*>(stg + p.s_off);
      const __half* stile16 = reinterpret_cast<const __half*>(stg + p.s_off);
      const float* xsum =
          reinterpret_cast<const float*>(Xs + ((nbuild - 1) & 1) * kXBufBytes + kXXsum);
      // zero points of the item's blocks for column nl: block b is nibble
      // b + (first block odd) of zbits (the tile's rows hold block pairs)
      uint64_t zbits = 0x8888888888888888ull;
      int zsh = 0;
      if (p.has_zp) {
        zbits = 0;
        for (int r = 0; r < p.z_rows; r++)
          zbits |= (uint64_t)stg[p.z_off + r * kTile + nl] << (8 * r);
        zsh = ((chunk * p.bpi) & 1) * 4;
      }
      const uint32_t dcol = tmem + lane_addr + kDCol + d * p.dstride;
      for (int rg = 0; rg < p.regions; rg++) {
        uint32_t v[NM];
        if constexpr (NM == 16)
          tmem_ld16(dcol + rg * NM, v);
        else
          tmem_ld32(dcol + rg * NM, v);
        tmem_ld_wait();
#pragma unroll
        for (int slot = 0; slot < G; slot++) {
          const int b = rg * G + slot;
          if (b < p.bpi) {
            const float sc = p.s16 ? __half2float(stile16[b * kTile + nl]) : stile[b * kTile + nl];
            const float zf = (float)((uint32_t)(zbits >> (4 * b + zsh)) & 0xFu);
#pragma unroll
            for (int m = 0; m < M; m++) {
              // D_t = sum q * c_t over the block (exact int32); the block's
              // sum (q - z) * X is D - z * sum X
              const int c = (slot * M + m) * 3;
              const float dq = ((float)(int)v[c + 2] * 65536.0f + (float)(int)v[c + 1] * 256.0f) +
                               (float)(int)v[c];
              y[m] = fmaf(sc, fmaf(-zf, xsum[b * M + m], dq), y[m]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ready[(j + p.nd) % kAItems]);  // D buffer d free for item j + nd
        mbar_arrive(&bempty[bst]);
      }
      j++;
      float part[M];
#pragma unroll
      for (int m = 0; m < M; m++)
        part[m] = S_m[m] == kNonFinite ? __int_as_float(0x7fc00000) : scale_pow2(y[m], -S_m[m]);
      const int n = tile * kTile + nl;
      if (p.tile_major && !clustered) {
        // chunk partials summed in chunk order: ((0 + p0) + p1) + ...
        float* ya = yacc + (size_t)tig * M * kTile;
#pragma unroll
        for (int m = 0; m < M; m++) {
          const float acc = chunk == 0 ? 0.0f + part[m] : ya[m * kTile + nl] + part[m];
          ya[m * kTile + nl] = acc;
          if (chunk == p.nch - 1 && n < p.N) {
            if constexpr (EXT) {
              ysel_store(ysel_base(p.Y, p.ysel), p.ldy, p.ysel, ep, m, n, acc);
              if (p.ysel.amax) amax_add(p.ysel, s_amax, s_nan0, m, n, acc);
            } else {
              ysel_base(p.Y, p.ysel)[m * p.ldy + n] = acc;
            }
          }
        }
      } else if (clustered) {
        // into the inbox of the CTA that sums this tile: rank ti % csize,
        // slot ti / csize, laid out [slot][chunk][m][128]
        const int ti = (tile - set) / p.ncl;
        const uint32_t dst = dsmem_addr(
            smem_u32(yacc) + (uint32_t)((((ti / p.csize) * p.nch + chunk) * M * kTile + nl) * 4),
            (uint32_t)(ti % p.csize));
#pragma unroll
        for (int m = 0; m < M; m++) st_dsmem_f32(dst + (uint32_t)(m * kTile * 4), part[m]);
      } else {
        const int64_t npad = (int64_t)p.tiles * kTile;
#pragma unroll
        for (int m = 0; m < M; m++) p.part[((int64_t)chunk * M + m) * npad + n] = part[m];
      }
      return true;
    });
    if (clustered) {
      // Deliver (also after an error, so that no CTA waits for a delivery
      // that cannot come): the warp's inbox stores are ordered before lane
      // 0's cluster fence by the warp barrier, the fence before the relaxed
      // arrivals, one per summing CTA of the set, from lanes 0 .. nsum-1.
      const int ntile = (p.tiles - 1 - set) / p.ncl + 1;
      const int nsum = min(p.csize, ntile);
      __syncwarp();
      if (lane == 0) fence_acq_rel_cluster();
      __syncwarp();
      if (lane < nsum) mbar_arrive_remote_relaxed(dsmem_addr(smem_u32(ibar), (uint32_t)lane));
      // Sum the inbox: tiles ti = rank, rank + csize, ... of the set, every
      // column's nch partials in chunk order ((0 + p_0) + p_1) + ..., the
      // sum the other paths form.  Only epilogue threads (past
      // griddepcontrol.wait) write outputs.
      const int rank = (int)blockIdx.x % p.csize;
      if (rank < nsum) {
        if (!mbar_wait_cluster(ibar, 0)) {
          record_error(p.err, KERR_WAIT_PEER);
        } else {
          // every epilogue thread takes (tile, row, column) triples of the
          // CTA's tiles; partials loaded 8 at a time, added in chunk order
          const int et = threadIdx.x - kEpiWarp0 * 32;
          float* Yb = ysel_base(p.Y, p.ysel);
          const int per = M * kTile, nmine = (ntile - rank + p.csize - 1) / p.csize;
          for (int i = et; i < nmine * per; i += kEpiWarps * 32) {
            const int sl = i / per, r = i % per;  // inbox slot = tile rank + sl * csize
            const int m = r / kTile, n = (set + (rank + sl * p.csize) * p.ncl) * kTile + r % kTile;
            const float* col = yacc + (size_t)sl * p.nch * per + r;
            float acc = 0.0f;
            int c = 0;
            for (; c + 8 <= p.nch; c += 8) {
              float v[8];
#pragma unroll
              for (int u = 0; u < 8; u++) v[u] = col[(size_t)(c + u) * per];
#pragma unroll
              for (int u = 0; u < 8; u++) acc = acc + v[u];
            }
            for (; c < p.nch; c++) acc = acc + col[(size_t)c * per];
            if (n < p.N) {
              if constexpr (EXT) {
                ysel_store(Yb, p.ldy, p.ysel, ep, m, n, acc);
                if (p.ysel.amax) amax_add(p.ysel, s_amax, s_nan0, m, n, acc);
              } else {
                Yb[m * p.ldy + n] = acc;
              }
            }
          }
        }
      }
    }
  }
  // the other warps' half of the cluster barrier begun after setup
  __syncwarp();
  if (clustered && !(warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps)) cluster_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // the split-K GEMV stores partials only; its chunk-sum kernel does this
  if constexpr (EXT)
    if (p.ysel.amax && p.tile_major) amax_finish(p.ysel, s_amax, s_nan0, s_last, M);
}

// Split-K: Y[m, n] = ((0 + part[0]) + part[1]) + ... in chunk order, the same
// sum the tile-major path forms, so both give identical bits.  Launched as a
// programmatic dependent of the GEMV: its small CTAs become resident beside
// the GEMV's and wait in griddepcontrol.wait, so no launch gap follows.
template <bool EXT>
__global__ void __launch_bounds__(128) gemv_tc_reduce_kernel(const float* __restrict__ part,
                                                           float* Y, int64_t ldy, int M, int N,
                                                           int nch, int64_t npad, YSel ysel) {
  __shared__ unsigned long long s_amax[8];
  __shared__ unsigned s_nan0, s_last;
  griddep_launch_dependents();
  if (EXT) {
    if (threadIdx.x < 8) s_amax[threadIdx.x] = 0ull;
    if (threadIdx.x == 0) s_nan0 = 0u;
    __syncthreads();
  }
  griddep_wait();
  Y = ysel_base(Y, ysel);
  const unsigned long long ep = EXT ? ysel_epoch(ysel) : 0ull;
  const int64_t total = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    const float* src = part + (int64_t)m * npad + n;
    const int64_t cs = (int64_t)M * npad;
    // all of a column's partials in flight at once (up to 32), then added in
    // chunk order
    float acc = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      float v[32];
#pragma unroll
      for (int c = 0; c < 32; c++) v[c] = c0 + c < nch ? __ldcg(src + (c0 + c) * cs) : 0.0f;
#pragma unroll
      for (int c = 0; c < 32; c++)
        if (c0 + c < nch) acc = acc + v[c];
    }
    if constexpr (EXT) {
      ysel_store(Y, ldy, ysel, ep, m, n, acc);
      if (ysel.amax) amax_add(ysel, s_amax, &s_nan0, m, n, acc);
    } else {
      Y[m * ldy + n] = acc;
    }
  }
  if constexpr (EXT) {
    if (ysel.amax) {
      __syncthreads();
      amax_finish(ysel, s_amax, &s_nan0, &s_last, M);
    }
  }
}

// Shared memory of one pipeline stage: the packed item, its block scales
// (fp16 when they were uploaded as fp16, else fp32) and its zero points.
uint32_t tc_stage_bytes(const Weight& w) {
  const int bpi = kChunkK / w.bs, z_rows = bpi >= 2 ? bpi / 2 : 1;
  const uint32_t z_off = kPackedBytes + (uint32_t)bpi * kTile * (w.scales16 ? 2 : 4);
  const uint32_t zbytes = w.has_zp ? (uint32_t)z_rows * kTile : 0;
  return (z_off + zbytes + 1023) & ~1023u;
}

// Raises the GEMV's shared-memory limit, once per device.
template <int M>
int configure_m() {
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load() >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(gemv_tc_kernel<M, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit));
    ORTC_CUDA(cudaFuncSetAttribute(gemv_tc_kernel<M, true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit));
    if (dev < 64) configured.fetch_or(1ull << dev);
  }
  return ORT_CUDA_OK;
}

// Clusters of `csize` GEMV CTAs (one CTA per SM) resident at once on this
// device, cached; -1 when none can be launched.
template <int M>
int max_clusters_m(int csize) {
  static std::atomic<int> cache[64][9];  // 0: not asked yet (racing threads ask twice)
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& mc = cache[dev & 63][csize];
  if (mc.load() == 0) {
    int n = 0;
    if (configure_m<M>() == ORT_CUDA_OK) {
      cudaLaunchConfig_t qc = {};
      qc.gridDim = dim3((unsigned)csize);
      qc.blockDim = dim3(kThreadsTC);
      qc.dynamicSmemBytes = kSmemLimit;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = (unsigned)csize;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      qc.attrs = qa;
      qc.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, gemv_tc_kernel<M, false>, &qc) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    mc = n > 0 ? n : -1;
  }
  return mc;
}

int max_clusters(int64_t M, int csize) {
  switch (M) {
    case 1: return max_clusters_m<1>(csize);
    case 2: return max_clusters_m<2>(csize);
    case 3: return max_clusters_m<3>(csize);
    case 4: return max_clusters_m<4>(csize);
    case 5: return max_clusters_m<5>(csize);
    case 6: return max_clusters_m<6>(csize);
    case 7: return max_clusters_m<7>(csize);
    case 8: return max_clusters_m<8>(csize);
  }
  return -1;
}

// Work decomposition.  Every candidate sums a column's chunk partials in
// chunk order, ((0 + p_0) + p_1) + ..., from identical partials, so the
// choice never changes a bit:
//  - tile-major: a CTA owns whole tiles and loops over all their chunks;
//  - clusters of csize CTAs: a cluster owns a tile set, rank r takes chunks
//    [r*nch/csize, (r+1)*nch/csize) and stores its partials into the shared
//    memory of the CTA that sums the tile;
//  - split-K: CTAs own one chunk of a tile set, a second kernel sums.
// plan_candidates lists the feasible ones in that order (a cluster inbox
// must leave room for three pipeline stages); which is fastest depends on
// the shape and on DRAM locality, so the first eager call times them
// (tune_tc_gemv) and the weight keeps the winner.  heuristic_plan is the
// choice before that: the busiest CTA's cost in items, where a chunk of T
// tiles costs max(T, 1.5) (the builder warp takes about 1.5 items' time
// for a chunk's X and hides it only behind that chunk's items) and split-K
// pays about three items for the boundary before its sum; ties go to more
// CTAs, then to the earlier candidate.
struct Plan {
  bool tile_major;
  int nch, tiles, grid, cpc, tg, csize, ncl;
  uint32_t yacc_bytes;
  size_t partial_floats;
  int64_t cost2;  // heuristic cost in half items
};

std::vector<Plan> plan_candidates(const Weight& w, int64_t M, int sm_count) {
  std::vector<Plan> out;
  Plan base = {};
  base.nch = (int)((w.K + kChunkK - 1) / kChunkK);
  base.tiles = (int)((w.nl + kTile - 1) / kTile);
  const size_t stage = tc_stage_bytes(w);
  const size_t tile_bytes = (size_t)M * kTile * 4;
  auto chunk_cost = [](int T) { return (int64_t)std::max(2 * T, 3); };
  Plan tm = base;
  tm.tile_major = true;
  tm.csize = 1;
  tm.ncl = std::min(base.tiles, sm_count);
  tm.tg = std::max<int>(1, (int)(32 / M));
  tm.grid = tm.ncl;
  tm.yacc_bytes = (uint32_t)(tm.tg * tile_bytes);
  tm.cost2 = chunk_cost((base.tiles + tm.ncl - 1) / tm.ncl) * base.nch;
  out.push_back(tm);
  for (int c = 2; c <= 8 && c <= base.nch; c++) {
    const int mc = max_clusters(M, c);
    if (mc <= 0) continue;
    const int ncl = std::min(base.tiles, mc), T = (base.tiles + ncl - 1) / ncl;
    const size_t inbox = (size_t)((T + c - 1) / c) * base.nch * tile_bytes;
    if (1024 + 2 * (size_t)kXBufBytes + inbox + a_stage_bytes(M, w.K % 4 == 0) + 1024 +
            3 * stage >
        kSmemLimit)
      continue;
    Plan cl = base;
    cl.tile_major = true;
    cl.csize = c;
    cl.ncl = ncl;
    cl.tg = T;
    cl.grid = ncl * c;
    cl.yacc_bytes = (uint32_t)inbox;
    cl.cost2 = chunk_cost(T) * ((base.nch + c - 1) / c);
    out.push_back(cl);
  }
  if (base.nch <= sm_count) {
    Plan sk = base;
    sk.tile_major = false;
    sk.csize = 1;
    sk.cpc = std::min(base.tiles, sm_count / base.nch);
    sk.grid = sk.cpc * base.nch;
    sk.tg = 1;
    sk.partial_floats = (size_t)base.nch * M * base.tiles * kTile;
    sk.cost2 = 2 * ((int64_t)((base.tiles + sk.cpc - 1) / sk.cpc) + 3);
    out.push_back(sk);
  }
  return out;
}

// The heuristic's choice among the candidates whose partial sums fit in
// `max_partial_floats` (-1: none fits).
int heuristic_plan(const std::vector<Plan>& c, size_t max_partial_floats = (size_t)-1) {
  int best = -1;
  for (int i = 0; i < (int)c.size(); i++) {
    if (c[i].partial_floats > max_partial_floats) continue;
    if (best < 0 || c[i].cost2 < c[best].cost2 ||
        (c[i].cost2 == c[best].cost2 && c[i].grid > c[best].grid))
      best = i;
  }
  return best;
}

// TMEM layout of D for one item: regions of G blocks, NM columns each.  Two
// D buffers when one fits in 128 columns.
struct DPlan {
  int regions, nm, nd;  // nd = 0: does not fit
};

DPlan d_plan(int64_t M, int bs) {
  const int G = M == 1 ? 5 : (M == 2 ? 2 : 1);
  DPlan d;
  d.nm = (3 * M * G <= 16) ? 16 : 32;
  d.regions = (kChunkK / bs + G - 1) / G;
  const int per = d.regions * d.nm;
  d.nd = per <= (int)kDCols / 2 ? 2 : (per <= (int)kDCols ? 1 : 0);
  return d;
}

template <int M>
int launch_m(const Weight& w, TcParams& p, const Plan& pl, cudaStream_t st) {
  const DPlan dp = d_plan(M, w.bs);
  p.regions = dp.regions;
  p.nd = dp.nd;
  p.dstride = p.nd == 2 ? kDCols / 2 : 0;
  // stage st covers k [32 st, 32 st + 32) of the item: block 32 st / bs,
  // region block / G; the first stage of a region starts its accumulator
  constexpr int G = XShape<M>::G;
  p.acc_mask = 0;
  for (int st = 0; st < kItemStages; st++) {
    const int blk = st * 32 / w.bs, rg = blk / G;
    p.op_d[st] = (uint32_t)(rg * dp.nm);
    if ((st * 32) % (G * w.bs) != 0) p.acc_mask |= 1u << st;
  }
  ORTC_CHECK(configure_m<M>() == ORT_CUDA_OK, ORT_CUDA_ERR_CUDA, "tc gemv: configure");
  const uint32_t yacc_bytes = pl.yacc_bytes;
  const int grid = pl.grid;
  p.yacc_bytes = yacc_bytes;
  const size_t fixed = 1024 + 2 * kXBufBytes + yacc_bytes + a_stage_bytes(M, p.a_vec) + 1024;
  int nbst = (int)((kSmemLimit - fixed) / p.stage_bytes);
  if (nbst > kMaxBStages) nbst = kMaxBStages;
  if (nbst < 2) return fail(ORT_CUDA_ERR_UNSUPPORTED, "tc gemv: shared memory too small");
  p.nbst = nbst;
  p.yacc_off = 2 * kXBufBytes + nbst * p.stage_bytes;
  p.a_off = p.yacc_off + yacc_bytes;
  const size_t smem = fixed + (size_t)nbst * p.stage_bytes;
  // Programmatic dependent launch: this kernel's prologue and weight stream
  // may overlap the previous kernel's tail; it reads activations and writes
  // outputs only after griddepcontrol.wait.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreadsTC);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)pl.csize;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pl.csize > 1 ? 2 : 1;
  const bool ext = p.ysel.push || p.ysel.nseg > 0 || p.ysel.amax != nullptr;
  if (ext)
    ORTC_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_kernel<M, true>, w.tmB, w.tmS,
                                 w.has_zp ? w.tmZ : w.tmS, p));
  else
    ORTC_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_kernel<M, false>, w.tmB, w.tmS,
                                 w.has_zp ? w.tmZ : w.tmS, p));
  return ORT_CUDA_OK;
}

}  // namespace

// TMA views of a MatMulNBits weight for the tensor-core GEMV.
// Shape conditions of the tensor-core GEMV that hold on every rank of an
// N-sharded group alike (they do not depend on the rank's column count).
static bool tc_layout_ok(const Weight& w) {
  const int64_t col_bytes = (int64_t)w.nb * w.bs / 2;
  return w.bs >= kMinBs && w.bs <= kChunkK && (w.bs & (w.bs - 1)) == 0 && col_bytes % 16 == 0;
}

int prepare_nbits_tc(Weight& w) {
  w.tc_ok = false;
  const int64_t col_bytes = (int64_t)w.nb * w.bs / 2;
  if (!tc_layout_ok(w) || w.nl == 0) return ORT_CUDA_OK;
  const int bpi = kChunkK / w.bs;
  int rc = encode_tma_2d(&w.tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.B, (uint64_t)col_bytes,
                         (uint64_t)w.nl, (uint64_t)col_bytes, 128, kTile,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (w.scales16)
    rc = encode_tma_2d(&w.tmS, CU_TENSOR_MAP_DATA_TYPE_UINT16, w.scales16, (uint64_t)w.nl,
                       (uint64_t)w.nb, (uint64_t)w.s16_pitch * 2, kTile, bpi,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    rc = encode_tma_2d(&w.tmS, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.scales, (uint64_t)w.nl,
                       (uint64_t)w.nb, (uint64_t)w.s_pitch * 4, kTile, bpi,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (w.has_zp) {
    rc = encode_tma_2d(&w.tmZ, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.zp, (uint64_t)w.nl,
                       (uint64_t)((w.nb + 1) / 2), (uint64_t)w.z_pitch, kTile,
                       bpi >= 2 ? bpi / 2 : 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  w.tc_ok = true;
  return ORT_CUDA_OK;
}

// The tensor-core GEMV takes M <= 8 when one item's D columns fit in TMEM
// beside the A ring (384 columns).
bool tc_gemv_ok(const Weight& w, int64_t M) {
  if (!w.tc_ok || M < 1 || M > 8) return false;
  return d_plan(M, w.bs).nd > 0;
}

bool tc_gemv_shape_ok(const Weight& w, int64_t M) {
  if (w.kind != W_NBITS || !tc_layout_ok(w) || M < 1 || M > 8) return false;
  return d_plan(M, w.bs).nd > 0;
}

namespace {

int launch_plan(const Weight& w, const Plan& pl, const float* A, int64_t M, float* Y,
                int64_t ldy, float* partials, int* err, int sm_count, cudaStream_t st,
                int64_t* launches, const YSel* ysel) {
  TcParams p;
  p.A = A;
  p.Y = Y;
  p.err = err;
  p.ldy = ldy;
  p.N = (int)w.nl;
  p.K = (int)w.K;
  p.bs = w.bs;
  p.bs_log2 = 0;
  while ((1 << p.bs_log2) < w.bs) p.bs_log2++;
  p.nch = pl.nch;
  p.tiles = pl.tiles;
  p.tile_major = pl.tile_major ? 1 : 0;
  p.csize = pl.csize;
  p.ncl = pl.ncl;
  p.tg = pl.tg;
  p.cpc = pl.cpc;
  p.part = pl.tile_major ? nullptr : partials;
  p.ysel = ysel ? *ysel : YSel();
  p.a_vec = ((reinterpret_cast<uintptr_t>(A) & 15) == 0 && w.K % 4 == 0) ? 1 : 0;
  p.bpi = kChunkK / w.bs;
  p.has_zp = w.has_zp ? 1 : 0;
  const int z_rows = p.bpi >= 2 ? p.bpi / 2 : 1;
  p.z_rows = z_rows;
  p.s16 = w.scales16 ? 1 : 0;
  const uint32_t sbytes = (uint32_t)p.bpi * kTile * (p.s16 ? 2 : 4);
  p.s_off = kPackedBytes;
  p.z_off = kPackedBytes + sbytes;
  const uint32_t zbytes = p.has_zp ? (uint32_t)z_rows * kTile : 0;
  p.stage_bytes = tc_stage_bytes(w);
  p.stage_tx = kPackedBytes + sbytes + zbytes;
  int rc;
  switch (M) {
    case 1: rc = launch_m<1>(w, p, pl, st); break;
    case 2: rc = launch_m<2>(w, p, pl, st); break;
    case 3: rc = launch_m<3>(w, p, pl, st); break;
    case 4: rc = launch_m<4>(w, p, pl, st); break;
    case 5: rc = launch_m<5>(w, p, pl, st); break;
    case 6: rc = launch_m<6>(w, p, pl, st); break;
    case 7: rc = launch_m<7>(w, p, pl, st); break;
    case 8: rc = launch_m<8>(w, p, pl, st); break;
    default: return fail(ORT_CUDA_ERR_INVALID_ARG, "tc gemv: M out of range");
  }
  if (rc) return rc;
  (*launches)++;
  if (!pl.tile_major) {
    const int64_t total = M * w.nl;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<int64_t>((total + 127) / 128, (int64_t)sm_count * 4));
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool ext = p.ysel.push || p.ysel.nseg > 0 || p.ysel.amax != nullptr;
    if (ext)
      ORTC_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_reduce_kernel<true>, (const float*)partials, Y,
                                   ldy, (int)M, (int)w.nl, pl.nch, (int64_t)pl.tiles * kTile,
                                   p.ysel));
    else
      ORTC_CUDA(cudaLaunchKernelEx(&cfg, gemv_tc_reduce_kernel<false>, (const float*)partials, Y,
                                   ldy, (int)M, (int)w.nl, pl.nch, (int64_t)pl.tiles * kTile,
                                   p.ysel));
    (*launches)++;
  }
  return ORT_CUDA_OK;
}

}  // namespace

int tc_gemv_plan(const Weight& w, int64_t M, int sm_count, size_t max_partial_floats) {
  const std::vector<Plan> c = plan_candidates(w, M, sm_count);
  const int t = (M >= 1 && M <= 8) ? w.gemv_plan[M] : -1;
  if (t >= 0 && t < (int)c.size() && c[t].partial_floats <= max_partial_floats) return t;
  return heuristic_plan(c, max_partial_floats);
}

int tc_gemv_plan_count(const Weight& w, int64_t M, int sm_count) {
  return (int)plan_candidates(w, M, sm_count).size();
}

size_t tc_gemv_partial_floats(const Weight& w, int64_t M, int sm_count, int plan) {
  const std::vector<Plan> c = plan_candidates(w, M, sm_count);
  if (plan < 0) {
    size_t mx = 0;
    for (const Plan& q : c) mx = std::max(mx, q.partial_floats);
    return mx;
  }
  return plan < (int)c.size() ? c[plan].partial_floats : 0;
}

int launch_tc_gemv(const Weight& w, int plan, const float* A, int64_t M, float* Y, int64_t ldy,
                   float* partials, int* err, int sm_count, cudaStream_t st, int64_t* launches,
                   const YSel* ysel) {
  if (w.nl == 0) return ORT_CUDA_OK;
  const std::vector<Plan> c = plan_candidates(w, M, sm_count);
  ORTC_CHECK(plan >= 0 && plan < (int)c.size(), ORT_CUDA_ERR_INVALID_ARG, "tc gemv: bad plan");
  return launch_plan(w, c[plan], A, M, Y, ldy, partials, err, sm_count, st, launches, ysel);
}

// Times every candidate plan on this call's operands and keeps the fastest
// in w.gemv_plan[M]: per candidate one warm launch, then kTuneReps back to
// back between two events, best of kTuneRounds rounds (rounds interleave
// the candidates, so a slow moment does not single one out).  All plans
// give identical bits, so the choice only moves time.  `partials` holds
// tc_gemv_partial_floats(w, M, sm, -1) floats.
int tune_tc_gemv(Weight& w, const float* A, int64_t M, float* Y, int64_t ldy, float* partials,
                 int* err, int sm_count, cudaStream_t st, const YSel* ysel) {
  constexpr int kTuneReps = 4, kTuneRounds = 2;
  if (M < 1 || M > 8 || w.nl == 0) return ORT_CUDA_OK;
  const std::vector<Plan> c = plan_candidates(w, M, sm_count);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  ORTC_CUDA(cudaEventCreate(&e0));
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return fail(ORT_CUDA_ERR_CUDA, "tc gemv tune: cudaEventCreate");
  }
  std::vector<float> ms_best(c.size(), -1.0f);
  int rc = ORT_CUDA_OK;
  int64_t uncounted = 0;
  for (int round = 0; round < kTuneRounds && rc == ORT_CUDA_OK; round++) {
    for (int i = 0; i < (int)c.size() && rc == ORT_CUDA_OK; i++) {
      rc = launch_plan(w, c[i], A, M, Y, ldy, partials, err, sm_count, st, &uncounted, ysel);
      if (rc) break;
      if (cudaEventRecord(e0, st) != cudaSuccess) {
        rc = fail(ORT_CUDA_ERR_CUDA, "tc gemv tune: record");
        break;
      }
      for (int r = 0; r < kTuneReps && rc == ORT_CUDA_OK; r++)
        rc = launch_plan(w, c[i], A, M, Y, ldy, partials, err, sm_count, st, &uncounted, ysel);
      if (rc) break;
      float ms = 0.0f;
      if (cudaEventRecord(e1, st) != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess ||
          cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess) {
        rc = fail(ORT_CUDA_ERR_CUDA, "tc gemv tune: timing");
        break;
      }
      if (ms_best[i] < 0.0f || ms < ms_best[i]) ms_best[i] = ms;
    }
  }
  int best = -1;
  for (int i = 0; i < (int)c.size(); i++)
    if (ms_best[i] >= 0.0f && (best < 0 || ms_best[i] < ms_best[best])) best = i;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc == ORT_CUDA_OK && best >= 0) w.gemv_plan[M] = (int8_t)best;
  return rc;
}

}  // namespace ortc
