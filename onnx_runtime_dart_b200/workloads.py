"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved; weights are random-init).

Config ids follow the order of the benchmark description:
  cfg1  single MatMulNBits op, M=16, K=N=1024, bs 32, no zero points
  cfg2  fp32 Gemm (transB=1, bias) at the BERT-384 FFN shapes
  cfg3  Qwen3-0.6B decode projections at M=1 (bs 32, fp32 scales, zp)
  cfg4  Llama-3.2-1B int4 prefill (M=2048) + decode (M=4), bs 128, fp16 scales
  cfg5  Llama-3-8B shapes, M in {1, 16, 4096}, bs 128, fp16 scales, zp
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import numpy as np


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """Packs uint4 values pairwise: element 2j -> low nibble, 2j+1 -> high."""
    q = q.astype(np.uint8)
    return (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def make_nbits_weight(rng: np.random.Generator, K: int, N: int, block_size: int,
                      zero_points: bool, scale_sigma: float = 0.02,
                      scale_dtype=np.float32, scale_mean: float = 0.0):
    """Packed uint4 B [N, nb, bs/2] (nibbles uniform 0..15; padding of a
    partial last block zero), scales |N(mean, sigma)| [N*nb], optional
    packed uint4 zero points (flat, low nibble first, uniform 0..15)."""
    nb = (K + block_size - 1) // block_size
    if K % block_size == 0:
        # uniform bytes = two uniform nibbles; fast for large weights
        B = rng.integers(0, 256, size=(N, nb, block_size // 2), dtype=np.uint8)
    else:
        q = rng.integers(0, 16, size=(N, nb * block_size), dtype=np.uint8)
        q[:, K:] = 0
        B = pack_nibbles(q.reshape(N, nb, block_size))
    s = rng.standard_normal(N * nb, dtype=np.float32) * scale_sigma + scale_mean
    if scale_mean == 0.0:
        s = np.abs(s)
    scales = s.astype(scale_dtype)
    zp = None
    if zero_points:
        zp = rng.integers(0, 256, size=(N * nb + 1) // 2, dtype=np.uint8)
    return B, scales, zp


@dataclass
class Proj:
    name: str
    K: int
    N: int


# Llama-3-8B: hidden 4096, intermediate 14336, 32 q / 8 kv heads x 128, vocab 128256
LLAMA3_8B = [Proj("qkv", 4096, 6144), Proj("o", 4096, 4096), Proj("gate_up", 4096, 28672),
             Proj("down", 14336, 4096), Proj("lm_head", 4096, 128256)]
# Llama-3.2-1B: hidden 2048, 32 q / 8 kv heads x 64, intermediate 8192, vocab 128256
LLAMA32_1B = [Proj("q", 2048, 2048), Proj("k", 2048, 512), Proj("v", 2048, 512),
              Proj("o", 2048, 2048), Proj("gate", 2048, 8192), Proj("up", 2048, 8192),
              Proj("down", 8192, 2048)]
LLAMA32_1B_LM_HEAD = Proj("lm_head", 2048, 128256)
# Qwen3-0.6B decode sweep (hidden 1024, 16 q heads x 128, 8 kv heads, intermediate 3072)
QWEN3_06B = [Proj("q", 1024, 2048), Proj("k", 1024, 1024), Proj("v", 1024, 1024),
             Proj("o", 2048, 1024), Proj("gate", 1024, 3072), Proj("up", 1024, 3072),
             Proj("down", 3072, 1024), Proj("lm_head", 1024, 151936)]


def nbits_bytes(K: int, N: int, bs: int, M: int, scale_bytes: int, zp: bool) -> int:
    """Algorithmic bytes of one MatMulNBits call: packed B + scales + zp +
    A (fp32) + Y (fp32).  Dequantisation work is not counted."""
    nb = (K + bs - 1) // bs
    b = N * nb * (bs // 2) + N * nb * scale_bytes + 4 * M * K + 4 * M * N
    if zp:
        b += (N * nb + 1) // 2
    return b


def nbits_flops(K: int, N: int, M: int) -> int:
    return 2 * M * N * K


def shard_range(N: int, rank: int, world: int) -> Tuple[int, int]:
    """Column range [a, b) rank `rank` owns: ceil(N/world) rounded up to 4
    (mirrors shard_cols in csrc/session.cu)."""
    if world == 1:
        return 0, N
    per = ((N + world - 1) // world + 3) // 4 * 4
    a = min(N, per * rank)
    return a, min(N, a + per)


def nbits_column_shard(B: np.ndarray, scales: np.ndarray, zp: Optional[np.ndarray], K: int,
                       N: int, block_size: int, a: int, b: int):
    """The MatMulNBits inputs of output columns [a, b) of a weight: packed
    B rows, the columns' scales, and the zero points re-packed in the
    reference's flat layout (nibble (n - a) * nb + blk, low nibble first),
    which is what a rank of an N-sharded group holds after upload."""
    nb = (K + block_size - 1) // block_size
    Bs = np.ascontiguousarray(B.reshape(N, nb, block_size // 2)[a:b])
    ss = np.ascontiguousarray(scales[a * nb:b * nb])
    zs = None
    if zp is not None:
        nib = np.stack([zp & 0xF, zp >> 4], 1).ravel()[:N * nb]
        part = nib[a * nb:b * nb]
        if part.size % 2:
            part = np.concatenate([part, np.zeros(1, np.uint8)])
        zs = pack_nibbles(part)
    return Bs, ss, zs
