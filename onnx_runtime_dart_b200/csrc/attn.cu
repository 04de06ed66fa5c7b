// Attention of a decoder step on the device, fp32: the body of
// GroupQueryAttention (opGroupQueryAttention, lib/src/onnx_ops.dart:
// 1507-1650), MultiHeadAttention (opMultiHeadAttention, :1656-1725) and the
// fused MatMul/Softmax/MatMul pattern (opFusedSDPA, :1733-1774), plus the
// standalone RotaryEmbedding (opRotaryEmbedding, :2121-2172).
//
// The reference forms the full score matrix QK^T per head with matmulKernel,
// scales it (double, stored fp32), adds the bias, applies the causal mask
// (key j <= past + i), takes a row softmax and multiplies by V.  Here one CTA
// owns a tile of query rows of one (batch, KV head) and streams that head's
// keys in 64-key tiles (cp.async into padded shared memory, two stages):
// scores in registers, online softmax (running max and sum per row), P.V
// accumulated in registers, normalised at the end.  Query rows are ordered
// token-major within the group of query heads sharing the KV head, so every
// K/V tile is read once for all of them (GQA reuse) and the causal limit of
// a tile of rows is that of its last token.  RoPE is applied in shared
// memory (double arithmetic, stored fp32, as the reference computes it); the
// CTAs of the last query tile also write the present K/V cache from shared
// memory, so the past is read once.  Decode-sized row counts split the keys
// across CTAs; the last CTA of a row tile (an atomic ticket) merges the
// partial (max, sum, P.V) triples in split order.
//
// Results differ from the reference's by fp32 rounding only (FMA dot
// products, expf, one division by the running sum).
#include <algorithm>
#include <climits>

#include <atomic>

#include "common.cuh"
#include "ptx.cuh"

namespace ortc {
namespace {

constexpr int kKT = 64;  // keys per tile
constexpr int kSmemMax = 224 * 1024;  // dynamic shared memory cap per CTA
// Split-key scratch: a fixed ticket area (keys are split only when there are
// fewer row tiles than SMs), then the partials.
constexpr int kMaxTickets = 1024;
constexpr size_t kTicketBytes = kMaxTickets * sizeof(unsigned);
// The merge keeps 2 * nsplit * rows floats in the tile buffers, which hold
// at least 2 * 32 * 64 + 8 * 64 floats (64-row tiles, head size 8).
constexpr int kMaxSplit = 32;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ const float* k_row(const AttnArgs& p, int b, int g, int j) {
  if (j < p.cached) return p.pk + b * p.psb + g * p.psh + (int64_t)j * p.D;
  return p.k + b * p.ksb + g * p.ksh + (int64_t)(j - p.cached) * p.ksj;
}
__device__ __forceinline__ const float* v_row(const AttnArgs& p, int b, int g, int j) {
  if (j < p.cached) return p.pv + b * p.psb + g * p.psh + (int64_t)j * p.Dv;
  return p.v + b * p.vsb + g * p.vsh + (int64_t)(j - p.cached) * p.vsj;
}

// Rotates pair i of a head vector in place at position pos: (i, i + half)
// (GPT-NeoX halves) or (2i, 2i + 1) (GPT-J pairs); x0*c - x1*s and
// x1*c + x0*s in double (the products of two floats are exact there),
// stored fp32.
__device__ __forceinline__ void rope_pair(float* row, int i, int half, int interleaved,
                                          const float* cos, const float* sin, int pos) {
  const int a0 = interleaved ? 2 * i : i, a1 = interleaved ? 2 * i + 1 : i + half;
  const double c = cos[(int64_t)pos * half + i], s = sin[(int64_t)pos * half + i];
  const double x0 = row[a0], x1 = row[a1];
  row[a0] = (float)(x0 * c - x1 * s);
  row[a1] = (float)(x1 * c + x0 * s);
}

// K/V tile [j0, j0 + KT) of (b, g) into shared memory, rows of PD / PDV
// floats; rows j >= T and the columns up to the next multiple of 4 are zero.
template <int NT, int KT>
__device__ __forceinline__ void load_kv_tile(const AttnArgs& p, int b, int g, int j0, float* ks,
                                             float* vs, int PD, int PDV) {
  const int D4 = (p.D + 3) & ~3, Dv4 = (p.Dv + 3) & ~3;
  if (p.vec) {  // 16-byte rows chunks, asynchronous
    const int kq = D4 >> 2, vq = Dv4 >> 2;
    for (int e = threadIdx.x; e < KT * kq; e += NT) {
      const int jj = e / kq, c = e - jj * kq, j = j0 + jj;
      const bool in = j < p.T;
      cp_async16(ks + jj * PD + 4 * c, in ? k_row(p, b, g, j) + 4 * c : p.q, in ? 16 : 0);
    }
    for (int e = threadIdx.x; e < KT * vq; e += NT) {
      const int jj = e / vq, c = e - jj * vq, j = j0 + jj;
      const bool in = j < p.T;
      cp_async16(vs + jj * PDV + 4 * c, in ? v_row(p, b, g, j) + 4 * c : p.q, in ? 16 : 0);
    }
    return;
  }
  // element loads: feature-fastest when K rows are contiguous, else
  // key-fastest (K given transposed)
  const bool dfast = p.ksd == 1;
  for (int e = threadIdx.x; e < KT * D4; e += NT) {
    const int jj = dfast ? e / D4 : e % KT, d = dfast ? e % D4 : e / KT, j = j0 + jj;
    float x = 0.0f;
    if (j < p.T && d < p.D) x = j < p.cached ? k_row(p, b, g, j)[d] : k_row(p, b, g, j)[d * p.ksd];
    ks[jj * PD + d] = x;
  }
  for (int e = threadIdx.x; e < KT * Dv4; e += NT) {
    const int jj = e / Dv4, d = e % Dv4, j = j0 + jj;
    vs[jj * PDV + d] = (j < p.T && d < p.Dv) ? v_row(p, b, g, j)[d] : 0.0f;
  }
}

// Split keys, after this CTA wrote its partial (max, sum, unnormalised P.V)
// rows: the last CTA of row-tile group x (an atomic ticket) merges every
// split's partials into the output.  Its (max, sum) pairs go to shared memory
// in one parallel pass (the tile buffers are free; 2 * nsplit * RT floats),
// then per row the weights exp(m_s - M) / L, then out = sum_s w_s * partial_s
// with independent loads.
template <int NT>
__device__ void take_ticket_and_merge(const AttnArgs& p, int x, int RT, int nrows, int b, int g,
                                      int row0, float* smem) {
  const int tid = threadIdx.x;
  const int64_t ngrp = (int64_t)p.nqt * p.batch * p.heads_kv;
  const float* po = p.part;                                  // [grp][split][RT][Dv]
  const float* pml = p.part + ngrp * p.nsplit * RT * p.Dv;   // [grp][split][RT][2]
  // the CTA's partial writes, ordered by the barrier, are released by
  // thread 0's acquire-release ticket (cumulative); the last CTA's thread 0
  // acquires every split's writes, which the barrier passes on to its CTA
  __syncthreads();
  __shared__ bool last;
  if (tid == 0) last = atom_add_acq_rel_gpu(&p.tickets[x], 1u) == (unsigned)(p.nsplit - 1);
  __syncthreads();
  if (!last) return;
  const int64_t gbase = (int64_t)x * p.nsplit * RT;
  float* mm = smem;                    // [nsplit][RT] maxima, then weights
  float* ll = smem + p.nsplit * RT;    // [nsplit][RT] sums
  for (int e = tid; e < p.nsplit * nrows; e += NT) {
    const int sp = e / nrows, r = e % nrows;
    mm[sp * RT + r] = __ldcg(pml + (gbase + sp * RT + r) * 2);
    ll[sp * RT + r] = __ldcg(pml + (gbase + sp * RT + r) * 2 + 1);
  }
  __syncthreads();
  // a warp per row, a lane per split (nsplit <= 32)
  const int lane = tid & 31;
  for (int r = tid >> 5; r < nrows; r += NT / 32) {
    const float ms = lane < p.nsplit ? mm[lane * RT + r] : -INFINITY;
    float M = ms;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float w = ms == -INFINITY ? 0.0f : expf(ms - M);
    float L = lane < p.nsplit ? w * ll[lane * RT + r] : 0.0f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (lane < p.nsplit) mm[lane * RT + r] = w / L;
  }
  __syncthreads();
  for (int e = tid; e < nrows * p.Dv; e += NT) {
    const int r = e / p.Dv, d = e % p.Dv;
    float acc = 0.0f;
#pragma unroll 16
    for (int sp = 0; sp < p.nsplit; sp++)
      acc = fmaf(mm[sp * RT + r], __ldcg(po + (gbase + sp * RT + r) * p.Dv + d), acc);
    const int gr = row0 + r, i = gr / p.group, h = g * p.group + gr % p.group;
    p.out[b * p.osb + (int64_t)i * p.osi + (int64_t)h * p.osh + d] = acc;
  }
  if (tid == 0) p.tickets[x] = 0;  // ready for the next call
}

// TX lanes share a query row (TX = 16: a half warp; 32: a warp); TY groups
// of them; RM rows per thread, KC keys per thread (key tx + TX*c): tiles of
// TX*KC keys (32 for heads above 64 in 64-row tiles, so that two CTAs fit
// an SM; else 64).
template <int TX, int TY, int RM, int KC>
__global__ void __launch_bounds__(TX* TY) attn_kernel(const AttnArgs p) {
  constexpr int NT = TX * TY, RT = TY * RM, DQ = (32 + TX - 1) / TX, KT = TX * KC;
  extern __shared__ __align__(16) float smem[];
  const int D4 = (p.D + 3) & ~3, Dv4 = (p.Dv + 3) & ~3;
  const int PD = D4 + 4, PDV = Dv4 + 4, PP = KT + 4;
  float* qs = smem;                 // RT x PD
  float* ks = qs + RT * PD;         // 2 x KT x PD
  float* vs = ks + 2 * KT * PD;    // 2 x KT x PDV
  float* ps = vs + 2 * KT * PDV;   // RT x PP

  int x = blockIdx.x;
  const int split = x % p.nsplit;
  x /= p.nsplit;  // row-tile group: (query tile, batch x KV head)
  const int nbh = p.batch * p.heads_kv;
  const int bh = x % nbh, qt = p.nqt - 1 - x / nbh;  // heaviest (last) tiles first
  const int b = bh / p.heads_kv, g = bh % p.heads_kv;
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int row0 = qt * RT, nrows = min(RT, p.rows_total - row0);

  int limit = p.T;  // keys [0, limit) are read by this row tile
  if (p.causal) limit = min(p.T, p.past + (row0 + nrows - 1) / p.group + 1);
  const int ntiles = (limit + KT - 1) / KT;
  const int tps = (ntiles + p.nsplit - 1) / p.nsplit;
  const int t0 = split * tps, t1 = min(ntiles, t0 + tps);
  const bool writer = p.prk != nullptr && qt == p.nqt - 1;

  // query rows of the tile (row r: token (row0 + r) / group, head
  // g * group + (row0 + r) % group), RoPE'd at position past + token
  for (int e = tid; e < RT * D4; e += NT) {
    const int r = e / D4, d = e % D4;
    float val = 0.0f;
    if (r < nrows && d < p.D) {
      const int gr = row0 + r, i = gr / p.group, h = g * p.group + gr % p.group;
      val = p.q[b * p.qsb + (int64_t)i * p.qsi + (int64_t)h * p.qsh + d];
    }
    qs[r * PD + d] = val;
  }
  if (p.rotary) {
    __syncthreads();
    for (int e = tid; e < RT * p.half_rot; e += NT) {
      const int r = e / p.half_rot, i = e % p.half_rot;
      if (r < nrows)
        rope_pair(qs + r * PD, i, p.half_rot, p.interleaved, p.cos, p.sin,
                  p.past + (row0 + r) / p.group);
    }
  }

  float m[RM], l[RM], o[RM][DQ][4];
  int klim[RM];  // last key row a may see (inclusive)
#pragma unroll
  for (int a = 0; a < RM; a++) {
    m[a] = -INFINITY;
    l[a] = 0.0f;
    const int r = ty * RM + a;
    klim[a] = r < nrows ? (p.causal ? p.past + (row0 + r) / p.group : p.T - 1) : -1;
#pragma unroll
    for (int c = 0; c < DQ; c++) o[a][c][0] = o[a][c][1] = o[a][c][2] = o[a][c][3] = 0.0f;
  }

  if (t0 < t1) {
    load_kv_tile<NT, KT>(p, b, g, t0 * KT, ks, vs, PD, PDV);
    cp_async_commit();
  }
  for (int t = t0; t < t1; t++) {
    const int stg = (t - t0) & 1;
    if (t + 1 < t1) {
      load_kv_tile<NT, KT>(p, b, g, (t + 1) * KT, ks + (stg ^ 1) * KT * PD,
                       vs + (stg ^ 1) * KT * PDV, PD, PDV);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float* kt = ks + stg * KT * PD;
    float* vt = vs + stg * KT * PDV;
    const int j0 = t * KT;
    const int jn0 = max(j0, p.cached), jn1 = min(j0 + KT, p.T);  // this call's keys
    if (p.rotary && jn0 < jn1) {  // RoPE at position j
      for (int e = tid; e < (jn1 - jn0) * p.half_rot; e += NT) {
        const int j = jn0 + e / p.half_rot, i = e % p.half_rot;
        rope_pair(kt + (j - j0) * PD, i, p.half_rot, p.interleaved, p.cos, p.sin, j);
      }
      __syncthreads();
    }
    if (writer) {  // present K/V rows of this tile (the past too, unless in place)
      const int jw0 = p.write_past ? j0 : jn0;
      for (int e = tid; e < (jn1 - jw0) * p.D; e += NT) {
        const int j = jw0 + e / p.D, d = e % p.D;
        p.prk[b * p.rsb + g * p.rsh + (int64_t)j * p.D + d] = kt[(j - j0) * PD + d];
      }
      for (int e = tid; e < (jn1 - jw0) * p.Dv; e += NT) {
        const int j = jw0 + e / p.Dv, d = e % p.Dv;
        p.prv[b * p.rsb + g * p.rsh + (int64_t)j * p.Dv + d] = vt[(j - j0) * PDV + d];
      }
    }

    // scores S[row][key] = q . k over the feature dimension
    float sc[RM][KC];
#pragma unroll
    for (int a = 0; a < RM; a++)
#pragma unroll
      for (int c = 0; c < KC; c++) sc[a][c] = 0.0f;
    for (int d = 0; d < D4; d += 4) {
      float4 qv[RM], kv[KC];
#pragma unroll
      for (int a = 0; a < RM; a++)
        qv[a] = *reinterpret_cast<const float4*>(qs + (ty * RM + a) * PD + d);
#pragma unroll
      for (int c = 0; c < KC; c++)
        kv[c] = *reinterpret_cast<const float4*>(kt + (tx + TX * c) * PD + d);
#pragma unroll
      for (int a = 0; a < RM; a++)
#pragma unroll
        for (int c = 0; c < KC; c++) {
          float s = sc[a][c];
          s = fmaf(qv[a].x, kv[c].x, s);
          s = fmaf(qv[a].y, kv[c].y, s);
          s = fmaf(qv[a].z, kv[c].z, s);
          s = fmaf(qv[a].w, kv[c].w, s);
          sc[a][c] = s;
        }
    }

    // scale (double, as the reference), bias, mask; online softmax
#pragma unroll
    for (int a = 0; a < RM; a++) {
      const int r = ty * RM + a;
      const int tok = (row0 + r) / p.group, h = g * p.group + (row0 + r) % p.group;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < KC; c++) {
        const int j = j0 + tx + TX * c;
        if (j <= klim[a] && j < p.T) {
          double t2 = (double)sc[a][c] * p.scale;
          if (p.bias)
            t2 += (double)p.bias[b * p.bsb + (int64_t)(h % p.bh) * p.bsh + (int64_t)tok * p.bsi +
                                 (int64_t)j * p.bsj];
          sc[a][c] = (float)t2;
          mx = fmaxf(mx, sc[a][c]);
        } else {
          sc[a][c] = -INFINITY;
        }
      }
#pragma unroll
      for (int off = TX / 2; off > 0; off >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[a], mx);
      float corr = 1.0f, psum = 0.0f;
      if (mn != -INFINITY) {
        corr = expf(m[a] - mn);
#pragma unroll
        for (int c = 0; c < KC; c++) {
          const float pr = expf(sc[a][c] - mn);
          sc[a][c] = pr;
          psum += pr;
        }
      } else {
#pragma unroll
        for (int c = 0; c < KC; c++) sc[a][c] = 0.0f;
      }
#pragma unroll
      for (int off = TX / 2; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l[a] = l[a] * corr + psum;
      m[a] = mn;
#pragma unroll
      for (int c = 0; c < DQ; c++) {
        o[a][c][0] *= corr;
        o[a][c][1] *= corr;
        o[a][c][2] *= corr;
        o[a][c][3] *= corr;
      }
#pragma unroll
      for (int c = 0; c < KC; c++) ps[r * PP + tx + TX * c] = sc[a][c];
    }
    __syncthreads();

    // O += P . V
    for (int j = 0; j < KT; j += 4) {
      float4 pv[RM];
#pragma unroll
      for (int a = 0; a < RM; a++)
        pv[a] = *reinterpret_cast<const float4*>(ps + (ty * RM + a) * PP + j);
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
#pragma unroll
        for (int c = 0; c < DQ; c++) {
          const int qd = 4 * (tx + TX * c);
          if (qd < Dv4) {
            const float4 vv = *reinterpret_cast<const float4*>(vt + (j + jj) * PDV + qd);
#pragma unroll
            for (int a = 0; a < RM; a++) {
              const float pr = jj == 0 ? pv[a].x : jj == 1 ? pv[a].y : jj == 2 ? pv[a].z : pv[a].w;
              o[a][c][0] = fmaf(pr, vv.x, o[a][c][0]);
              o[a][c][1] = fmaf(pr, vv.y, o[a][c][1]);
              o[a][c][2] = fmaf(pr, vv.z, o[a][c][2]);
              o[a][c][3] = fmaf(pr, vv.w, o[a][c][3]);
            }
          }
        }
      }
    }
    __syncthreads();  // the stage and P are rewritten next
  }

  if (p.nsplit == 1) {
#pragma unroll
    for (int a = 0; a < RM; a++) {
      const int r = ty * RM + a;
      if (r >= nrows) continue;
      const int gr = row0 + r, i = gr / p.group, h = g * p.group + gr % p.group;
      float* dst = p.out + b * p.osb + (int64_t)i * p.osi + (int64_t)h * p.osh;
#pragma unroll
      for (int c = 0; c < DQ; c++) {
        const int qd = 4 * (tx + TX * c);
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (qd + e < p.Dv) dst[qd + e] = o[a][c][e] / l[a];
      }
    }
    return;
  }

  // split keys: partial (max, sum, unnormalised P.V) per row, then the last
  // CTA of the row tile merges them
  const int64_t base = ((int64_t)x * p.nsplit + split) * RT;
  const int64_t ngrp = (int64_t)p.nqt * nbh;
  float* po = p.part;                                  // [grp][split][RT][Dv]
  float* pml = p.part + ngrp * p.nsplit * RT * p.Dv;   // [grp][split][RT][2]
#pragma unroll
  for (int a = 0; a < RM; a++) {
    const int r = ty * RM + a;
    if (r >= nrows) continue;
    if (tx == 0) {
      pml[(base + r) * 2] = m[a];
      pml[(base + r) * 2 + 1] = l[a];
    }
#pragma unroll
    for (int c = 0; c < DQ; c++) {
      const int qd = 4 * (tx + TX * c);
#pragma unroll
      for (int e = 0; e < 4; e++)
        if (qd + e < p.Dv) po[(base + r) * p.Dv + qd + e] = o[a][c][e];
    }
  }
  take_ticket_and_merge<NT>(p, x, RT, nrows, b, g, row0, smem);
}

// Decode: at most 16 query rows per (batch, KV head) -- the query heads of
// one KV head for one to a few tokens -- against a long key sequence, which
// makes the call a stream over the K/V cache with a short critical path.
// Eight warps each own 8 keys of every 64-key tile and keep their own
// online-softmax state (a flash-decoding split inside the CTA), so a tile
// needs no CTA-wide reduction; the warp states are merged once at the end.
// The cached rows of a tile are contiguous in memory and arrive as one bulk
// copy each for K and V (unpadded rows, 3-stage ring on mbarriers); this
// call's rows and Q are loaded and RoPE'd in registers by all threads while
// those copies are in flight.  Score lane (row r, key kk) forms one dot
// product with four independent FMA chains, walking the features from a
// lane-dependent start so that the 8 key rows a warp reads at once fall in
// different banks; for P.V a lane owns a 4-float slice of the head for all
// rows.  Needs head % 4 == 0, equal K and V head sizes and 16-byte aligned
// rows (launch_attention checks).
constexpr int kDecStages = 3;
constexpr int kDecWarps = 8;

// Element c of the RoPE'd copy of a head vector: pairs (i, i + half) or
// (2i, 2i + 1) for i < half, the tail copied; src[d * stride] is feature d.
__device__ __forceinline__ void rope_store(float* dst, const float* src, int64_t stride, int c,
                                           int half, int interleaved, const float* cos,
                                           const float* sin, int pos) {
  if (c >= half) {  // tail feature c + half
    dst[c + half] = src[(int64_t)(c + half) * stride];
    return;
  }
  const int a0 = interleaved ? 2 * c : c, a1 = interleaved ? 2 * c + 1 : c + half;
  const double cs = cos[(int64_t)pos * half + c], sn = sin[(int64_t)pos * half + c];
  const double x0 = src[(int64_t)a0 * stride], x1 = src[(int64_t)a1 * stride];
  dst[a0] = (float)(x0 * cs - x1 * sn);
  dst[a1] = (float)(x1 * cs + x0 * sn);
}

template <int RTP>
__global__ void __launch_bounds__(kDecWarps * 32) attn_decode_kernel(const AttnArgs p) {
  constexpr int NT = kDecWarps * 32;
  constexpr int KW = 32 / RTP;                   // keys per warp and step (score lanes)
  constexpr int KPW = kKT / kDecWarps;           // keys per warp and tile (8)
  constexpr int SPT = KPW / KW;                  // steps per tile
  static_assert(SPT >= 1 && SPT * KW == KPW, "row padding of 4, 8 or 16");
  extern __shared__ __align__(16) float smem[];
  __shared__ __align__(8) uint64_t full[kDecStages];
  const int D = p.D, D4 = D >> 2, PDQ = D + 4;
  float* qs = smem;                                // RTP x PDQ
  float* ks = qs + RTP * PDQ;                      // stages x 64 x D
  float* vs = ks + kDecStages * kKT * D;           // stages x 64 x D
  float* pw = vs + kDecStages * kKT * D;           // warps x 8 keys x RTP probabilities

  int x = blockIdx.x;
  const int split = x % p.nsplit;
  x /= p.nsplit;
  const int b = x / p.heads_kv, g = x % p.heads_kv;  // one row tile (nqt == 1)
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nrows = p.rows_total;
  int limit = p.T;
  if (p.causal) limit = min(p.T, p.past + (nrows - 1) / p.group + 1);
  const int ntiles = (limit + kKT - 1) / kKT;
  const int tps = (ntiles + p.nsplit - 1) / p.nsplit;
  const int t0 = split * tps, t1 = min(ntiles, t0 + tps);
  const bool writer = p.prk != nullptr;
  const int hr = p.rotary ? p.half_rot : 0;      // RoPE pairs per head vector

  // thread 0: the cached rows [j0, min(j0 + 64, cached)) of K and V into a stage
  auto issue = [&](int t, int stg) {
    const int j0 = t * kKT, nc = max(0, min(kKT, p.cached - j0));
    mbar_arrive_expect_tx(&full[stg], (uint32_t)(nc * D * 8));
    if (nc) {
      bulk_load(ks + stg * kKT * D, k_row(p, b, g, j0), (uint32_t)(nc * D * 4), &full[stg]);
      bulk_load(vs + stg * kKT * D, v_row(p, b, g, j0), (uint32_t)(nc * D * 4), &full[stg]);
    }
  };
  if (tid == 0) {
    for (int s2 = 0; s2 < kDecStages; s2++) mbar_init(&full[s2], 1);
    fence_mbarrier_init();
    for (int t = t0; t < min(t1, t0 + kDecStages - 1); t++) issue(t, t - t0);
  }
  // Q rows (RoPE'd at position past + token) while the copies fly
  for (int e = tid; e < RTP * (D - hr); e += NT) {
    const int r = e / (D - hr), c = e % (D - hr);
    float* dst = qs + r * PDQ;
    if (r >= nrows) {  // item c covers features c and c + hr (a pair or the tail)
      if (c < hr) dst[c] = 0.0f;
      dst[c + hr] = 0.0f;
      continue;
    }
    const int h = g * p.group + r % p.group;
    const float* src = p.q + b * p.qsb + (int64_t)(r / p.group) * p.qsi + (int64_t)h * p.qsh;
    if (hr)
      rope_store(dst, src, 1, c, hr, p.interleaved, p.cos, p.sin, p.past + r / p.group);
    else
      dst[c] = src[c];
  }
  __syncthreads();  // Q rows and the barrier initialisation

  const int rs = lane / KW, kk = lane % KW;  // score lane: row, key
  const int klim = rs < nrows ? (p.causal ? p.past + rs / p.group : p.T - 1) : -1;
  const int tok_s = rs / p.group, h_s = g * p.group + rs % p.group;
  const int KH = 32 / D4;                    // P.V: keys in parallel per warp
  const int dq = lane % D4, kh = lane / D4;  // P.V lane: feature slice, key slot
  const bool pv_lane = lane < KH * D4;
  float m_s = -INFINITY, l_s = 0.0f;
  float o[RTP][4];
#pragma unroll
  for (int r = 0; r < RTP; r++) o[r][0] = o[r][1] = o[r][2] = o[r][3] = 0.0f;

  int failed = -1;  // the tile whose copies did not land
  for (int t = t0; t < t1; t++) {
    const int stg = (t - t0) % kDecStages;
    if (tid == 0 && t + kDecStages - 1 < t1) {
      fence_proxy_async_smem();  // the stage's last reads (generic) before the copies
      issue(t + kDecStages - 1, (t + kDecStages - 1 - t0) % kDecStages);
    }
    const int j0 = t * kKT;
    float* kt = ks + stg * kKT * D;
    float* vt = vs + stg * kKT * D;
    // this call's rows (RoPE'd at position j) and the rows past the sequence
    const int jn0 = max(j0, p.cached), jn1 = min(j0 + kKT, p.T);
    for (int e = tid; e < max(0, jn1 - jn0) * (D - hr); e += NT) {
      const int j = jn0 + e / (D - hr), c = e % (D - hr);
      const float* src = k_row(p, b, g, j);
      if (hr)
        rope_store(kt + (j - j0) * D, src, p.ksd, c, hr, p.interleaved, p.cos, p.sin, j);
      else
        kt[(j - j0) * D + c] = src[(int64_t)c * p.ksd];
    }
    for (int e = tid; e < max(0, jn1 - jn0) * D; e += NT) {
      const int j = jn0 + e / D, d = e % D;
      vt[(j - j0) * D + d] = v_row(p, b, g, j)[d];
    }
    for (int e = tid; e < max(0, j0 + kKT - max(j0, p.T)) * D; e += NT) {
      const int jj = max(j0, p.T) - j0 + e / D, d = e % D;
      kt[jj * D + d] = 0.0f;
      vt[jj * D + d] = 0.0f;
    }
    const bool ok = mbar_wait(&full[stg], (uint32_t)(((t - t0) / kDecStages) & 1));
    if (__syncthreads_or(!ok)) {
      failed = t;
      break;
    }
    if (writer) {  // present rows: this call's (and the past, unless in place)
      const int jw0 = p.write_past ? j0 : jn0;
      for (int e = tid; e < max(0, jn1 - jw0) * D; e += NT) {
        const int j = jw0 + e / D, d = e % D;
        p.prk[b * p.rsb + g * p.rsh + (int64_t)j * D + d] = kt[(j - j0) * D + d];
        p.prv[b * p.rsb + g * p.rsh + (int64_t)j * D + d] = vt[(j - j0) * D + d];
      }
    }

    // scores of this warp's keys w*8 + st*KW + kk
    float sc[SPT];
#pragma unroll
    for (int st = 0; st < SPT; st++) {
      const int jj = w * KPW + st * KW + kk, j = j0 + jj;
      const float* qr = qs + rs * PDQ;
      const float* kr = kt + jj * D;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int c = kk % D4;
#pragma unroll 4
      for (int q = 0; q < D4; q++) {
        const float4 qv = *reinterpret_cast<const float4*>(qr + 4 * c);
        const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * c);
        acc.x = fmaf(qv.x, kv.x, acc.x);
        acc.y = fmaf(qv.y, kv.y, acc.y);
        acc.z = fmaf(qv.z, kv.z, acc.z);
        acc.w = fmaf(qv.w, kv.w, acc.w);
        c = c + 1 == D4 ? 0 : c + 1;
      }
      const float dot = (acc.x + acc.y) + (acc.z + acc.w);
      if (j <= klim && j < p.T) {
        double t2 = (double)dot * p.scale;
        if (p.bias)
          t2 += (double)p.bias[b * p.bsb + (int64_t)(h_s % p.bh) * p.bsh + (int64_t)tok_s * p.bsi +
                               (int64_t)j * p.bsj];
        sc[st] = (float)t2;
      } else {
        sc[st] = -INFINITY;
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int st = 0; st < SPT; st++) mx = fmaxf(mx, sc[st]);
#pragma unroll
    for (int off = KW / 2; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float mn = fmaxf(m_s, mx);
    float corr = 1.0f, psum = 0.0f;
    if (mn != -INFINITY) {
      corr = expf(m_s - mn);
#pragma unroll
      for (int st = 0; st < SPT; st++) {
        sc[st] = expf(sc[st] - mn);
        psum += sc[st];
      }
    } else {
#pragma unroll
      for (int st = 0; st < SPT; st++) sc[st] = 0.0f;
    }
#pragma unroll
    for (int off = KW / 2; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
    l_s = l_s * corr + psum;
    m_s = mn;
#pragma unroll
    for (int st = 0; st < SPT; st++) pw[(w * KPW + st * KW + kk) * RTP + rs] = sc[st];
#pragma unroll
    for (int r = 0; r < RTP; r++) {
      const float cr = __shfl_sync(0xffffffffu, corr, r * KW);
      o[r][0] *= cr;
      o[r][1] *= cr;
      o[r][2] *= cr;
      o[r][3] *= cr;
    }
    __syncwarp();
    if (pv_lane) {
      for (int kidx = kh; kidx < KPW; kidx += KH) {
        const float4 vv = *reinterpret_cast<const float4*>(vt + (w * KPW + kidx) * D + 4 * dq);
        const float* pp = pw + (w * KPW + kidx) * RTP;
#pragma unroll
        for (int r4 = 0; r4 < RTP; r4 += 4) {
          const float4 p4 = *reinterpret_cast<const float4*>(pp + r4);
          const float pr[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
          for (int u = 0; u < 4; u++) {
            o[r4 + u][0] = fmaf(pr[u], vv.x, o[r4 + u][0]);
            o[r4 + u][1] = fmaf(pr[u], vv.y, o[r4 + u][1]);
            o[r4 + u][2] = fmaf(pr[u], vv.z, o[r4 + u][2]);
            o[r4 + u][3] = fmaf(pr[u], vv.w, o[r4 + u][3]);
          }
        }
      }
    }
    __syncthreads();  // the stage and this warp's probabilities are rewritten next
  }
  if (failed >= 0) {  // a copy never landed: record it, let the issued copies drain, stop
    if (tid == 0) {
      record_error(p.err, KERR_WAIT_FULL);
      for (int t = failed; t < min(t1, failed + kDecStages); t++)  // issued, not consumed
        if (!mbar_wait(&full[(t - t0) % kDecStages], (uint32_t)(((t - t0) / kDecStages) & 1)))
          record_error(p.err, KERR_WAIT_DRAIN);
    }
    __syncthreads();
    return;
  }

  // merge the warps' states: (m, l) per row, sum over key slots of P.V
  float* mw = smem;                  // [warp][RTP]
  float* lw = mw + kDecWarps * RTP;  // [warp][RTP]
  float* ow = lw + kDecWarps * RTP;  // [warp][RTP][D]
  if (kk == 0) {
    mw[w * RTP + rs] = m_s;
    lw[w * RTP + rs] = l_s;
  }
  for (int k2 = 0; k2 < KH; k2++) {
    if (pv_lane && kh == k2)
#pragma unroll
      for (int r = 0; r < RTP; r++)
#pragma unroll
        for (int u = 0; u < 4; u++) {
          float* dst = ow + (w * RTP + r) * D + 4 * dq + u;
          *dst = k2 == 0 ? o[r][u] : *dst + o[r][u];
        }
    __syncwarp();
  }
  float* rM = ow + kDecWarps * RTP * D;  // [RTP] CTA maximum, then [RTP] sum
  float* rL = rM + RTP;
  __syncthreads();
  for (int r = tid; r < nrows; r += NT) {  // per row: the warps' weights, once
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < kDecWarps; w2++) M = fmaxf(M, mw[w2 * RTP + r]);
    float L = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < kDecWarps; w2++) {
      const float ms = mw[w2 * RTP + r];
      const float wt = ms == -INFINITY ? 0.0f : expf(ms - M);
      mw[w2 * RTP + r] = wt;
      L = fmaf(wt, lw[w2 * RTP + r], L);
    }
    rM[r] = M;
    rL[r] = L;
  }
  __syncthreads();
  const int64_t base = ((int64_t)x * p.nsplit + split) * RTP;
  const int64_t ngrp = (int64_t)p.batch * p.heads_kv;
  float* po = p.part;
  float* pml = p.part ? p.part + ngrp * p.nsplit * RTP * D : nullptr;
  for (int e = tid; e < nrows * D; e += NT) {
    const int r = e / D, d = e % D;
    const float M = rM[r], L = rL[r];
    float acc = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < kDecWarps; w2++)
      acc = fmaf(mw[w2 * RTP + r], ow[(w2 * RTP + r) * D + d], acc);
    if (p.nsplit == 1) {
      const int h = g * p.group + r % p.group;
      p.out[b * p.osb + (int64_t)(r / p.group) * p.osi + (int64_t)h * p.osh + d] = acc / L;
    } else {
      po[(base + r) * D + d] = acc;
      if (d == 0) {
        pml[(base + r) * 2] = M;
        pml[(base + r) * 2 + 1] = L;
      }
    }
  }
  if (p.nsplit == 1) return;
  __syncthreads();  // the merge reuses the buffers read above
  take_ticket_and_merge<NT>(p, x, RTP, nrows, b, g, 0, smem);
}

// Present K/V rows of a prefill with RoPE, once, ahead of the attention
// kernel: this call's K rows RoPE'd at position j, its V rows copied, and
// the past copied when the present cache does not alias it.  One thread per
// present element; a K element reads its pair partner from the input row.
__global__ void kv_prepare_kernel(const AttnArgs p) {
  const int D = p.D, j_lo = p.write_past ? 0 : p.past;
  const int64_t nrow = (int64_t)(p.T - j_lo), n = (int64_t)p.batch * p.heads_kv * nrow * D;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(e % D);
    const int64_t r = e / D;
    const int j = j_lo + (int)(r % nrow);
    const int bg = (int)(r / nrow), b = bg / p.heads_kv, g = bg % p.heads_kv;
    const int64_t dst = b * p.rsb + g * p.rsh + (int64_t)j * D + d;
    if (j < p.past) {
      p.prk[dst] = p.pk[b * p.psb + g * p.psh + (int64_t)j * D + d];
      p.prv[dst] = p.pv[b * p.psb + g * p.psh + (int64_t)j * D + d];
      continue;
    }
    const float* kr = p.k + b * p.ksb + g * p.ksh + (int64_t)(j - p.past) * p.ksj;
    const float* vr = p.v + b * p.vsb + g * p.vsh + (int64_t)(j - p.past) * p.vsj;
    p.prv[dst] = vr[d];
    const int half = p.half_rot;
    float val = kr[d];
    if (d < 2 * half) {
      int i, first;
      if (p.interleaved) {
        i = d >> 1;
        first = (d & 1) == 0;
      } else {
        i = d < half ? d : d - half;
        first = d < half;
      }
      const int a0 = p.interleaved ? 2 * i : i, a1 = p.interleaved ? 2 * i + 1 : i + half;
      const double c = p.cos[(int64_t)j * half + i], sn = p.sin[(int64_t)j * half + i];
      const double x0 = kr[a0], x1 = kr[a1];
      val = first ? (float)(x0 * c - x1 * sn) : (float)(x1 * c + x0 * sn);
    }
    p.prk[dst] = val;
  }
}

__global__ void rotary_kernel(const float* __restrict__ X, float* __restrict__ Y,
                              const int64_t* __restrict__ pos, int pos_per_batch,
                              const float* __restrict__ cos, const float* __restrict__ sin,
                              int64_t max_pos, int half, int rdim, int64_t batch, int64_t seq,
                              int64_t heads, int64_t head, int x_bhsd, int interleaved) {
  // one thread per (b, s, h, feature) of the output
  const int64_t n = batch * seq * heads * head;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = e % head, rest = e / head;
    const int64_t s = x_bhsd ? rest % seq : (rest / heads) % seq;
    const int64_t b = x_bhsd ? rest / seq / heads : rest / heads / seq;
    const float* row = X + (e - d);
    if (d >= rdim) {
      Y[e] = row[d];
      continue;
    }
    const int64_t pp = pos[(pos_per_batch ? b : 0) * seq + s];
    if (pp < 0 || pp >= max_pos) {  // the reference raises; no read outside the caches
      Y[e] = __int_as_float(0x7fc00000);
      continue;
    }
    // pairs (i, i + rdim/2) or (2i, 2i + 1); cos/sin rows hold `half` values
    const int ph = rdim / 2;
    int i, first;
    if (interleaved) {
      i = (int)(d >> 1);
      first = (d & 1) == 0;
    } else {
      i = (int)(d < ph ? d : d - ph);
      first = d < ph;
    }
    const int a0 = interleaved ? 2 * i : i, a1 = interleaved ? 2 * i + 1 : i + ph;
    const double c = cos[pp * half + i], sn = sin[pp * half + i];
    const double x0 = row[a0], x1 = row[a1];
    Y[e] = first ? (float)(x0 * c - x1 * sn) : (float)(x1 * c + x0 * sn);
  }
}

struct AttnCfg {
  int tx, ty, rm, rows, kt;
};

AttnCfg pick_cfg(int rows_total, int D) {
  if (rows_total <= 4) return {32, 4, 1, 4, 64};
  if (rows_total <= 8) return {32, 8, 1, 8, 64};
  if (rows_total <= 16) return {16, 16, 1, 16, 64};
  return {16, 16, 4, 64, D > 64 ? 32 : 64};
}

size_t attn_smem_bytes(const AttnArgs& a, const AttnCfg& c) {
  const int PD = ((a.D + 3) & ~3) + 4, PDV = ((a.Dv + 3) & ~3) + 4;
  return sizeof(float) *
         ((size_t)c.rows * PD + 2 * c.kt * PD + 2 * c.kt * PDV + c.rows * (c.kt + 4));
}

size_t decode_smem_bytes(const AttnArgs& a, int rows) {
  return sizeof(float) * ((size_t)rows * (a.D + 4) + 2 * kDecStages * kKT * a.D + kKT * rows);
}

// The decode kernel: few rows, head % 4 == 0, equal K and V head sizes,
// contiguous 16-byte aligned K/V rows (bulk copies), fits in shared memory.
bool decode_ok(const AttnArgs& a, const AttnCfg& c) {
  return c.rows <= 16 && a.vec && a.D == a.Dv && decode_smem_bytes(a, c.rows) <= (size_t)kSmemMax;
}

template <int RTP>
int launch_dec(const AttnArgs& a, size_t smem, int64_t grid, cudaStream_t st) {
  static std::atomic<unsigned long long> attr_set{0};  // per device
  int dev = 0;
  ORTC_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !(attr_set.load() >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(attn_decode_kernel<RTP>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
    if (dev < 64) attr_set.fetch_or(1ull << dev);
  }
  attn_decode_kernel<RTP><<<(unsigned)grid, kDecWarps * 32, smem, st>>>(a);
  ORTC_CUDA(cudaGetLastError());
  return ORT_CUDA_OK;
}

template <int TX, int TY, int RM, int KC>
int launch_cfg(const AttnArgs& a, size_t smem, int64_t grid, cudaStream_t st) {
  static std::atomic<unsigned long long> attr_set{0};  // per device
  int dev = 0;
  ORTC_CUDA(cudaGetDevice(&dev));
  if (dev >= 64 || !(attr_set.load() >> dev & 1ull)) {
    ORTC_CUDA(cudaFuncSetAttribute(attn_kernel<TX, TY, RM, KC>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax));
    if (dev < 64) attr_set.fetch_or(1ull << dev);
  }
  attn_kernel<TX, TY, RM, KC><<<(unsigned)grid, TX * TY, smem, st>>>(a);
  ORTC_CUDA(cudaGetLastError());
  return ORT_CUDA_OK;
}

}  // namespace

namespace {

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }
bool mult4(int64_t v) { return (v & 3) == 0; }

// 16-byte (vector or bulk) loads of every K/V row: head sizes % 4, rows of
// this call contiguous and aligned, cached rows aligned.
bool vec_ok(const AttnArgs& t) {
  return t.D % 4 == 0 && t.Dv % 4 == 0 &&
         (t.cached >= t.T ||
          (t.ksd == 1 && aligned16(t.k) && aligned16(t.v) && mult4(t.ksb) && mult4(t.ksh) &&
           mult4(t.ksj) && mult4(t.vsb) && mult4(t.vsh) && mult4(t.vsj))) &&
         (t.cached == 0 ||
          (aligned16(t.pk) && aligned16(t.pv) && mult4(t.psb) && mult4(t.psh)));
}

struct AttnPlan {
  AttnCfg c;
  bool decode = false, prepass = false;
  AttnArgs pre;  // the arguments of the RoPE pre-pass
};

// Settles the path -- the decode kernel, or the tile kernel after an
// optional RoPE pre-pass into the present cache -- and the key split, and
// updates `a` for it.
AttnPlan plan_attention(AttnArgs& a, int sm_count) {
  AttnPlan pl;
  if (a.cached < 0) a.cached = a.past;
  pl.c = pick_cfg(a.seq * a.group, std::max(a.D, a.Dv));
  a.rows_total = a.seq * a.group;
  a.nqt = (a.rows_total + pl.c.rows - 1) / pl.c.rows;
  a.vec = vec_ok(a);
  pl.decode = decode_ok(a, pl.c);
  if (!pl.decode && a.rotary && a.prk && a.D == a.Dv && a.D % 4 == 0 && aligned16(a.prk) &&
      aligned16(a.prv) && mult4(a.rsb) && mult4(a.rsh)) {
    // prefill with RoPE into a present cache: K rotated once by the
    // pre-pass, then every key is read from the cache
    pl.prepass = true;
    pl.pre = a;
    a.pk = a.prk, a.pv = a.prv, a.psb = a.rsb, a.psh = a.rsh;
    a.cached = a.T;
    a.prk = a.prv = nullptr;
    a.vec = vec_ok(a);
    pl.decode = decode_ok(a, pl.c);
  }
  const int64_t groups = (int64_t)a.nqt * a.batch * a.heads_kv;
  const int ntiles = (a.T + kKT - 1) / kKT;
  int64_t want = 1;
  if (pl.decode) {  // one wave of CTAs: the split's fixed costs are paid once
    const size_t smem = decode_smem_bytes(a, pl.c.rows) + 1024;
    const int64_t occ =
        std::max<int64_t>(1, std::min<int64_t>(232448 / smem, pl.c.rows == 4 ? 3 : 2));
    want = std::max<int64_t>(1, sm_count * occ / groups);
  } else if (groups < sm_count) {
    want = (2 * sm_count + groups - 1) / groups;
  }
  int64_t nsplit = groups <= kMaxTickets
                       ? std::min<int64_t>({want, (int64_t)ntiles, (int64_t)kMaxSplit})
                       : 1;
  if (nsplit > 1) {  // as many splits as it takes at ceil(tiles / want) tiles each: none idle
    const int64_t tps = (ntiles + nsplit - 1) / nsplit;
    nsplit = (ntiles + tps - 1) / tps;
  }
  a.nsplit = (int)std::max<int64_t>(1, nsplit);
  return pl;
}

}  // namespace

size_t attention_scratch_bytes(const AttnArgs& a0, int sm_count) {
  AttnArgs a = a0;
  const AttnPlan pl = plan_attention(a, sm_count);
  if (a.nsplit == 1) return 0;
  const int64_t groups = (int64_t)a.nqt * a.batch * a.heads_kv;
  return kTicketBytes + sizeof(float) * (size_t)groups * a.nsplit * pl.c.rows * (a.Dv + 2);
}

int launch_attention(AttnArgs a, void* scratch, int sm_count, cudaStream_t st, int64_t* launches) {
  ORTC_CHECK(a.D >= 1 && a.D <= 128 && a.Dv >= 1 && a.Dv <= 128, ORT_CUDA_ERR_UNSUPPORTED,
             "attention: head sizes above 128 are not supported");
  if (a.seq == 0 || a.batch == 0 || a.heads_kv == 0) return ORT_CUDA_OK;
  ORTC_CHECK(a.T >= 1, ORT_CUDA_ERR_INVALID_ARG, "attention: no keys");
  const AttnPlan pl = plan_attention(a, sm_count);
  const AttnCfg& c = pl.c;
  const int64_t groups = (int64_t)a.nqt * a.batch * a.heads_kv;
  const int64_t grid = groups * a.nsplit;
  ORTC_CHECK(grid <= INT_MAX, ORT_CUDA_ERR_INVALID_ARG, "attention: too many row tiles");
  if (a.nsplit > 1) {
    ORTC_CHECK(scratch != nullptr, ORT_CUDA_ERR_INVALID_ARG, "attention: scratch missing");
    a.tickets = static_cast<unsigned*>(scratch);
    a.part = reinterpret_cast<float*>(static_cast<char*>(scratch) + kTicketBytes);
  }
  if (pl.prepass) {
    const AttnArgs& q = pl.pre;
    const int64_t n = (int64_t)q.batch * q.heads_kv * (q.T - (q.write_past ? 0 : q.past)) * q.D;
    if (n > 0) {
      const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sm_count * 16);
      kv_prepare_kernel<<<(unsigned)blocks, 256, 0, st>>>(q);
      ORTC_CUDA(cudaGetLastError());
      (*launches)++;
    }
  }
  int rc;
  if (pl.decode) {
    const size_t smem = decode_smem_bytes(a, c.rows);
    if (c.rows == 4)
      rc = launch_dec<4>(a, smem, grid, st);
    else if (c.rows == 8)
      rc = launch_dec<8>(a, smem, grid, st);
    else
      rc = launch_dec<16>(a, smem, grid, st);
  } else {
    const size_t smem = attn_smem_bytes(a, c);
    ORTC_CHECK(smem <= (size_t)kSmemMax, ORT_CUDA_ERR_UNSUPPORTED,
               "attention: tile does not fit");
    if (c.rows == 4)
      rc = launch_cfg<32, 4, 1, 2>(a, smem, grid, st);
    else if (c.rows == 8)
      rc = launch_cfg<32, 8, 1, 2>(a, smem, grid, st);
    else if (c.rows == 16)
      rc = launch_cfg<16, 16, 1, 4>(a, smem, grid, st);
    else if (c.kt == 32)
      rc = launch_cfg<16, 16, 4, 2>(a, smem, grid, st);
    else
      rc = launch_cfg<16, 16, 4, 4>(a, smem, grid, st);
  }
  if (rc) return rc;
  (*launches)++;
  return ORT_CUDA_OK;
}

int launch_rotary(const float* X, float* Y, const int64_t* pos, int pos_per_batch,
                  const float* cos, const float* sin, int64_t max_pos, int half_rot, int rdim,
                  int64_t batch, int64_t seq, int64_t heads, int64_t head, int x_bhsd,
                  int interleaved, cudaStream_t st, int64_t* launches) {
  const int64_t n = batch * seq * heads * head;
  if (n == 0) return ORT_CUDA_OK;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  rotary_kernel<<<(unsigned)blocks, 256, 0, st>>>(X, Y, pos, pos_per_batch, cos, sin, max_pos,
                                                  half_rot, rdim, batch, seq, heads, head, x_bhsd,
                                                  interleaved);
  ORTC_CUDA(cudaGetLastError());
  (*launches)++;
  return ORT_CUDA_OK;
}

}  // namespace ortc
