"""CPU ORACLE wrapper — test infrastructure only, never the product path.

ctypes front-end over ``oracle/liboracle.so`` (built from ``oracle.c`` by
``oracle/Makefile``), plus numpy helpers that generate the seeded synthetic
inputs of each benchmark configuration.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and its
``--impl reference`` arm) may import this module; the CUDA path in
``onnx_runtime_dart_b200`` never does.

Each function names the reference (CrispStrobe/onnx_runtime_dart 0.10.3)
file:line whose arithmetic it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc, no GPU)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_half_to_float_bits.restype = ctypes.c_uint32
        L.orc_half_to_float_bits.argtypes = [ctypes.c_uint32]
        L.orc_half_to_float_array.argtypes = [_u16p, _f32p, ctypes.c_int64]
        L.orc_dequant_nbits.argtypes = [_u8p, _f32p, _u8p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, _f32p]
        L.orc_matmul_kernel.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int]
        L.orc_matmul_kernel_scalar.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64,
                                               ctypes.c_int, ctypes.c_int]
        L.orc_matmul_nbits.restype = ctypes.c_int
        L.orc_matmul_nbits.argtypes = [_f32p, ctypes.c_int64, _u8p, _f32p, _u8p, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                       ctypes.c_int]
        L.orc_transpose.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_gemm.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                               ctypes.c_float, ctypes.c_float, _f32p, ctypes.c_int64,
                               ctypes.c_int64, _f32p, ctypes.c_int]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else ctypes.cast(None, t)


def half_to_float(h: np.ndarray) -> np.ndarray:
    """onnx_proto_loader.dart:29-47 halfToFloat32Bits over an array of
    fp16 bit patterns (uint16) -> fp32."""
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_half_to_float_array(_p(h, _u16p), _p(out, _f32p), h.size)
    return out


def dequant_nbits(B, scales, zp, K, N, block_size) -> np.ndarray:
    """onnx_qlinear_ops.dart:127-149: the [K, N] fp32 weight opMatMulNBits
    builds before its GEMM."""
    B = np.ascontiguousarray(B, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    zp = None if zp is None else np.ascontiguousarray(zp, np.uint8)
    W = np.empty((K, N), np.float32)
    lib().orc_dequant_nbits(_p(B, _u8p), _p(scales, _f32p), _p(zp, _u8p), K, N, block_size,
                            _p(W, _f32p))
    return W


def matmul_kernel(a, b, threads: int = 1) -> np.ndarray:
    """gemm_kernel_simd.dart:27-309 matmulKernel for a [m, k] x [k, n]."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    out = np.empty((m, n), np.float32)
    lib().orc_matmul_kernel(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, k, n, threads)
    return out


def matmul_kernel_scalar(a, b) -> np.ndarray:
    """gemm_kernel_scalar.dart:10-41 (the web build's kernel)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), np.float32)
    lib().orc_matmul_kernel_scalar(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, k, n)
    return out


def matmul_nbits(A, B, scales, zp, K, N, bits, block_size, threads: int = 1) -> np.ndarray:
    """onnx_qlinear_ops.dart:114-156 opMatMulNBits.  A has any rank with a
    trailing K; Y has shape A.shape[:-1] + [N]."""
    if bits != 4:
        raise NotImplementedError(f"MatMulNBits: only bits=4 supported, got {bits}")
    A = np.ascontiguousarray(A, np.float32)
    M = A.size // K
    B = np.ascontiguousarray(B, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    zp = None if zp is None else np.ascontiguousarray(zp, np.uint8)
    Y = np.empty((M, N), np.float32)
    rc = lib().orc_matmul_nbits(_p(A, _f32p), M, _p(B, _u8p), _p(scales, _f32p), _p(zp, _u8p),
                                K, N, bits, block_size, _p(Y, _f32p), threads)
    if rc != 0:
        raise RuntimeError(f"orc_matmul_nbits failed: {rc}")
    return Y.reshape(tuple(A.shape[:-1]) + (N,))


def gemm(A, B, C=None, alpha=1.0, beta=1.0, transA=False, transB=False, threads: int = 1):
    """onnx_ops.dart:1777-1793 opGemm (with the transposes of :1782-1783
    materialised, as onnx_graph.dart:1156-1173 prepacks B)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    if transA:
        A = np.ascontiguousarray(A.T)
    if transB:
        B = np.ascontiguousarray(B.T)
    M, K = A.shape
    N = B.shape[1]
    Y = np.empty((M, N), np.float32)
    if C is not None:
        C = np.ascontiguousarray(C, np.float32)
        c2 = C.reshape((1,) * (2 - C.ndim) + C.shape) if C.ndim < 2 else C
        cr, cc = c2.shape
        if cr not in (1, M) or cc not in (1, N):
            raise ValueError(f"Gemm: C shape {C.shape} does not broadcast to {(M, N)}")
        c2 = np.ascontiguousarray(c2)
    else:
        c2, cr, cc = None, 0, 0
    lib().orc_gemm(_p(A, _f32p), _p(B, _f32p), M, K, N, float(alpha), float(beta),
                   _p(c2, _f32p), cr, cc, _p(Y, _f32p), threads)
    return Y


def matmul(a, b, threads: int = 1) -> np.ndarray:
    """onnx_ops.dart:1375-1431 opMatMul (float path): numpy-style batch
    broadcast, with the shared-weight collapse of :1389-1400 (B without
    batch dims turns all A batches into one [batch*m, k] GEMM)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    m, k = a.shape[-2:]
    k2, n = b.shape[-2:]
    assert k == k2, f"MatMul inner dims mismatch: {k} vs {k2}"
    a_batch, b_batch = a.shape[:-2], b.shape[:-2]
    out_batch = np.broadcast_shapes(a_batch, b_batch)
    count = int(np.prod(out_batch)) if out_batch else 1
    if count > 1 and int(np.prod(b_batch) if b_batch else 1) == 1:
        out = matmul_kernel(a.reshape(count * m, k), b.reshape(k, n), threads)
        return out.reshape(tuple(out_batch) + (m, n))
    ab = np.broadcast_to(a, tuple(out_batch) + (m, k)).reshape(count, m, k)
    bb = np.broadcast_to(b, tuple(out_batch) + (k, n)).reshape(count, k, n)
    out = np.stack([matmul_kernel(ab[i], bb[i], threads) for i in range(count)])
    return out.reshape(tuple(out_batch) + (m, n))


# Seeded synthetic inputs come from the package's workload definitions
# (data generation only; no arithmetic of the path lives there).
from onnx_runtime_dart_b200.workloads import make_nbits_weight, pack_nibbles  # noqa: E402,F401


def argminmax(x, axis: int = 0, keepdims: bool = True, is_max: bool = True,
              select_last: bool = False) -> np.ndarray:
    """ArgMax / ArgMin, restating opArgMinMax (lib/src/onnx_ops.dart:2198-2237):
    along `axis`, a scan from element 0 that replaces the best on a strictly
    better value (or also an equal one with select_last_index), with plain
    comparisons, so ties keep the first (last) index and a NaN wins only as
    element 0.  int64 result; plain Python loops (small inputs)."""
    x = np.asarray(x, dtype=np.float32)
    ax = axis + x.ndim if axis < 0 else axis
    xm = np.moveaxis(x, ax, -1)
    flat = xm.reshape(-1, xm.shape[-1])
    out = np.empty(flat.shape[0], np.int64)
    for r in range(flat.shape[0]):
        row = flat[r].tolist()
        best, best_i = row[0], 0
        for d in range(1, len(row)):
            v = row[d]
            if is_max:
                better = v >= best if select_last else v > best
            else:
                better = v <= best if select_last else v < best
            if better:
                best, best_i = v, d
        out[r] = best_i
    out = out.reshape(xm.shape[:-1])
    return np.expand_dims(out, ax) if keepdims else out


def matmul_integer(a, b, a_zp=None, b_zp=None) -> np.ndarray:
    """MatMulInteger, restating opMatMulInteger
    (lib/src/onnx_qlinear_ops.dart:26-79): Y = (A - a_zp) . (B - b_zp),
    exact integers (int64, as the reference stores them); a_zp scalar or per
    row [M], b_zp scalar or per column [N]; batch dims as in MatMul (equal or
    1)."""
    a = np.asarray(a).astype(np.int64)
    b = np.asarray(b).astype(np.int64)
    m, n = a.shape[-2], b.shape[-1]
    az = 0 if a_zp is None else np.asarray(a_zp).astype(np.int64).reshape(-1)
    bz = 0 if b_zp is None else np.asarray(b_zp).astype(np.int64).reshape(-1)
    if a_zp is not None and az.size not in (1, m):
        raise ValueError("MatMulInteger: a_zp must be scalar or per-row [M]")
    if b_zp is not None and bz.size not in (1, n):
        raise ValueError("MatMulInteger: b_zp must be scalar or per-column [N]")
    ac = a - (az.reshape(-1, 1) if np.size(az) == m and m != 1 else np.reshape(az, ()))
    bc = b - (np.reshape(bz, ()) if np.size(bz) == 1 else bz)
    # every product and partial sum is an integer of magnitude <= 255^2 K,
    # exact in float64 below 2^53, so the float64 matmul is the exact one
    assert 255 * 255 * a.shape[-1] < 2 ** 53
    return np.rint(np.matmul(ac.astype(np.float64), bc.astype(np.float64))).astype(np.int64)


def _round_even(v: float) -> int:
    """Round half to even (the reference's _roundEven,
    onnx_qlinear_ops.dart:17-24)."""
    f = np.floor(v)
    frac = v - f
    if frac > 0.5:
        return int(f) + 1
    if frac < 0.5:
        return int(f)
    i = int(f)
    return i if i % 2 == 0 else i + 1


def dynamic_quantize_linear(x):
    """DynamicQuantizeLinear, restating opDynamicQuantizeLinear
    (lib/src/onnx_ops.dart:2556-2580): range [min(0, min x), max(0, max x)];
    scale = fp32((mx - mn) / 255); zp = round-half-even(clamp(fp32(-mn /
    scale), 0, 255)); y = saturate(round-half-even(fp32(x / scale)) + zp).
    Returns (uint8 y, float32 scale, int zp)."""
    xf = np.asarray(x, dtype=np.float32).reshape(-1)
    mn = min(0.0, float(xf.min())) if xf.size else 0.0
    mx = max(0.0, float(xf.max())) if xf.size else 0.0
    scale = float(np.float32((mx - mn) / 255.0))
    zpf = 0.0 if scale == 0 else float(np.float32(-mn / scale))
    zp = _round_even(min(max(zpf, 0.0), 255.0))
    out = np.empty(xf.size, np.uint8)
    for k, v in enumerate(xf.tolist()):
        q = zp if scale == 0 else _round_even(float(np.float32(v / scale))) + zp
        out[k] = 0 if q < 0 else (255 if q > 255 else q)
    return out.reshape(np.shape(x)), np.float32(scale), zp


# ---- attention (the decoder step around the MatMulNBits projections) --------

def rotary_embedding(x, position_ids, cos_cache, sin_cache, interleaved: bool = False,
                     num_heads: int = 0, rotary_dim: int = 0) -> np.ndarray:
    """RotaryEmbedding, restating opRotaryEmbedding (lib/src/onnx_ops.dart:
    2121-2172): x [batch, seq, hidden] (or [batch, heads, seq, head]);
    cos/sin [max_pos, rotary_dim/2] indexed by position_ids [batch, seq] (or
    [seq], shared); the first rotary_dim features of each head are rotated
    (GPT-NeoX halves, or GPT-J pairs when interleaved), the rest copied.  Each
    output is x0*c -/+ x1*s in double, stored to float32, as in the
    reference."""
    x = np.asarray(x, np.float32)
    cos = np.asarray(cos_cache, np.float32)
    sin = np.asarray(sin_cache, np.float32)
    pos = np.asarray(position_ids).astype(np.int64)
    half_rot = cos.shape[-1]
    rdim = rotary_dim if rotary_dim > 0 else 2 * half_rot
    if x.ndim == 4:
        xs = np.transpose(x, (0, 2, 1, 3))  # -> [b, s, h, d]
    else:
        b, s, hidden = x.shape
        head = hidden // num_heads if num_heads > 0 else rdim
        xs = x.reshape(b, s, hidden // head, head)
    batch, seq = xs.shape[:2]
    p = pos.reshape(1, seq) if pos.ndim == 1 else pos.reshape(batch, seq)
    p = np.broadcast_to(p, (batch, seq))
    c = cos.reshape(-1, half_rot)[p][:, :, None, :rdim // 2].astype(np.float64)
    sn = sin.reshape(-1, half_rot)[p][:, :, None, :rdim // 2].astype(np.float64)
    out = xs.copy()
    x64 = xs.astype(np.float64)
    if interleaved:
        x0, x1 = x64[..., 0:rdim:2], x64[..., 1:rdim:2]
        out[..., 0:rdim:2] = (x0 * c - x1 * sn).astype(np.float32)
        out[..., 1:rdim:2] = (x1 * c + x0 * sn).astype(np.float32)
    else:
        h = rdim // 2
        x0, x1 = x64[..., :h], x64[..., h:rdim]
        out[..., :h] = (x0 * c - x1 * sn).astype(np.float32)
        out[..., h:rdim] = (x1 * c + x0 * sn).astype(np.float32)
    if x.ndim == 4:
        return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3)))
    return out.reshape(x.shape)


def _softmax_rows(sc64, stored32):
    """The reference's row softmax after the scale/bias pass
    (onnx_ops.dart:1604-1621): the maximum is taken over the unrounded double
    scores, exp(float32 score - max) is stored to float32 while its double
    value is summed in index order, and each stored exp is multiplied by
    1/sum (double) and stored to float32."""
    mx = np.max(sc64, axis=-1, keepdims=True)
    e = np.exp(stored32.astype(np.float64) - mx)
    e32 = e.astype(np.float32)
    total = np.cumsum(e, axis=-1)[..., -1:]
    return (e32.astype(np.float64) * (1.0 / total)).astype(np.float32)


def group_query_attention(q, k, v, num_heads: int, kv_num_heads: int, scale=None,
                          do_rotary: bool = False, rotary_interleaved: bool = False,
                          cos_cache=None, sin_cache=None, past_key=None, past_value=None,
                          attention_bias=None):
    """GroupQueryAttention (com.microsoft), restating opGroupQueryAttention
    (lib/src/onnx_ops.dart:1507-1650): q [batch, seq, H*D], k/v [batch, seq,
    Hkv*D], optional past [batch, Hkv, P, D]; RoPE on q and k at positions
    P..P+seq-1 when do_rotary; present = past ++ (roped k, raw v); query
    token i attends causally to keys 0..P+i; scores = QK^T (matmulKernel,
    fp32) * scale + bias, the reference's row softmax, then P.V
    (matmulKernel).  Returns (out [batch, seq, H*D], present_key,
    present_value [batch, Hkv, P+seq, D])."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    batch, seq = q.shape[:2]
    D = q.shape[2] // num_heads
    group = num_heads // kv_num_heads
    P = past_key.shape[2] if past_key is not None and np.ndim(past_key) == 4 else 0
    T = P + seq
    if do_rotary:
        # The reference builds these positions as a [1, seq] tensor
        # (onnx_ops.dart:1533-1536), which opRotaryEmbedding indexes with
        # b*seq + s (:2147): batch > 1 raises a RangeError there.  The same
        # positions for every batch row (ORT's definition; a rank-1 tensor)
        # is what batch 1 computes and what the restatement uses.
        pos = np.arange(P, P + seq, dtype=np.int64)
        q = rotary_embedding(q, pos, cos_cache, sin_cache, rotary_interleaved, num_heads)
        k = rotary_embedding(k, pos, cos_cache, sin_cache, rotary_interleaved, kv_num_heads)
    s = float(scale) if scale is not None else 1.0 / np.sqrt(D)
    kn = k.reshape(batch, seq, kv_num_heads, D).transpose(0, 2, 1, 3)
    vn = v.reshape(batch, seq, kv_num_heads, D).transpose(0, 2, 1, 3)
    if P:
        pk = np.asarray(past_key, np.float32)
        pv = np.asarray(past_value, np.float32)
        present_k = np.concatenate([pk, kn], axis=2)
        present_v = np.concatenate([pv, vn], axis=2)
    else:
        present_k, present_v = np.ascontiguousarray(kn), np.ascontiguousarray(vn)
    bias = None if attention_bias is None else np.asarray(attention_bias, np.float32)
    bias_heads = 0 if bias is None else bias.shape[1]
    out = np.empty((batch, seq, num_heads * D), np.float32)
    for b in range(batch):
        for h in range(num_heads):
            kvh = h // group
            qh = np.ascontiguousarray(q[b, :, h * D:(h + 1) * D])
            scores = matmul_kernel(qh, np.ascontiguousarray(present_k[b, kvh].T))
            probs = np.zeros((seq, T), np.float32)
            for i in range(seq):
                last = P + i
                sc = scores[i, :last + 1].astype(np.float64) * s
                if bias is not None:  # batch-1 bias broadcasts (as in MHA)
                    bb = b if bias.shape[0] > 1 else 0
                    sc = sc + bias[bb, h % bias_heads, i, :last + 1].astype(np.float64)
                probs[i, :last + 1] = _softmax_rows(sc, sc.astype(np.float32))
            out[b, :, h * D:(h + 1) * D] = matmul_kernel(probs, np.ascontiguousarray(present_v[b, kvh]))
    return out, np.ascontiguousarray(present_k), np.ascontiguousarray(present_v)


def multi_head_attention(q, k, v, num_heads: int, scale=None, attention_bias=None):
    """MultiHeadAttention (com.microsoft), restating opMultiHeadAttention
    (lib/src/onnx_ops.dart:1656-1725): q [batch, seq, hidden], k/v [batch,
    kv_seq, hidden], no mask beyond the optional additive bias [batch,
    bias_heads, seq, kv_seq]."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    batch, seq, hidden = q.shape
    D = hidden // num_heads
    s = float(scale) if scale is not None else 1.0 / np.sqrt(D)
    bias = None if attention_bias is None else np.asarray(attention_bias, np.float32)
    out = np.empty_like(q)
    for b in range(batch):
        for h in range(num_heads):
            sl = slice(h * D, (h + 1) * D)
            scores = matmul_kernel(np.ascontiguousarray(q[b, :, sl]),
                                   np.ascontiguousarray(k[b, :, sl].T))
            sc = scores.astype(np.float64) * s
            if bias is not None:  # a batch-1 bias broadcasts (ORT; the reference
                # indexes b * bias_heads and raises for b > 0)
                sc = sc + bias[b if bias.shape[0] > 1 else 0, h % bias.shape[1]].astype(np.float64)
            probs = _softmax_rows(sc, sc.astype(np.float32))
            out[b, :, sl] = matmul_kernel(probs, np.ascontiguousarray(v[b, :, sl]))
    return out


def fused_sdpa(a, b, v, mask, scale: float):
    """_FusedSDPA, restating opFusedSDPA (lib/src/onnx_ops.dart:1733-1774):
    s = MatMul(a, b) (b is K already transposed), val = s*scale + mask
    (mask broadcast numpy-style, stored to float32), exp(val - max) stored,
    divided by the double sum, then MatMul(s, v).  `scale` is the fused
    node's float32 attribute (onnx_graph.dart:355-386 folds Div(c) as
    1/c)."""
    s = matmul(a, b)
    m = np.broadcast_to(np.asarray(mask, np.float32), s.shape)
    val = s.astype(np.float64) * float(scale) + m.astype(np.float64)
    mx = np.max(val, axis=-1, keepdims=True)
    e = np.exp(val.astype(np.float32).astype(np.float64) - mx)
    e32 = e.astype(np.float32)
    total = np.cumsum(e, axis=-1)[..., -1:]
    p = (e32.astype(np.float64) / total).astype(np.float32)
    return matmul(p, v)


# ---- selection after lm_head ------------------------------------------------

def topk(x, k: int, axis: int = -1, largest: bool = True):
    """TopK, restating opTopK (lib/src/onnx_ops.dart:2261-2303): along
    `axis`, the indices ordered by value (descending when largest, else
    ascending) with ties to the smaller index; Dart's compareTo ranks NaN
    above every number, and -0.0 == 0.0 is a tie.  Returns (values float32,
    indices int64) of shape x.shape with axis -> k.  Plain Python sort."""
    x = np.asarray(x, np.float32)
    ax = axis + x.ndim if axis < 0 else axis
    xm = np.moveaxis(x, ax, -1)
    flat = xm.reshape(-1, xm.shape[-1])
    vals = np.empty((flat.shape[0], k), np.float32)
    idx = np.empty((flat.shape[0], k), np.int64)
    for r in range(flat.shape[0]):
        row = flat[r].tolist()
        if largest:
            order = sorted(range(len(row)),
                           key=lambda d: (0 if row[d] != row[d] else 1, -row[d] if row[d] == row[d] else 0.0, d))
        else:
            order = sorted(range(len(row)),
                           key=lambda d: (1 if row[d] != row[d] else 0, row[d] if row[d] == row[d] else 0.0, d))
        idx[r] = order[:k]
        vals[r] = flat[r][order[:k]]
    shape = xm.shape[:-1] + (k,)
    return (np.moveaxis(vals.reshape(shape), -1, ax), np.moveaxis(idx.reshape(shape), -1, ax))


def slice_last_seq(x):
    """_SliceLastSeq (onnx_graph.dart:456-473): x[..., seq-1:seq, :]."""
    x = np.asarray(x)
    return np.ascontiguousarray(x[..., -1:, :]) if x.shape[-2] > 1 else x
