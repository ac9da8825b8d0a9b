"""Seeded synthetic inputs of the benchmark configurations (numpy, host side).

The shapes and value distributions follow the benchmark configurations of the
ternary GEMV: weights i.i.d. uniform over {-1, 0, +1}, one fp16 scale per
128-column block drawn as |N(0, 1)| * 0.02, activations fp32 N(0, 1).
Weights are emitted in the GGUF source format the library loads, PTQ1_0
(28-byte blocks: 128 base-3 trits + fp16 scale; byte layout of
ref/bonsai-decoder/src/types.cpp:289-320 and include/bd/types.hpp:67-78 of
the reference), so the repack path is exercised exactly as at model load.

There is no dataset or checkpoint behind these numbers: they stand in for
model weights with the same shapes and statistics.
"""
from __future__ import annotations

import numpy as np

# (K, N) of the per-layer GEMV shape set at batch 1 (benchmark configuration 1).
LAYER_SHAPES = (
    ("q", 5120, 6144),
    ("k", 5120, 1024),
    ("v", 5120, 1024),
    ("o", 6144, 5120),
    ("gate", 5120, 17408),
    ("up", 5120, 17408),
    ("down", 17408, 5120),
)
LM_HEAD = ("lm_head", 5120, 248320)

# base-3 digit weights: five digits per byte, first element most significant
_W5 = np.array([81, 27, 9, 3, 1], dtype=np.uint16)
_W4 = np.array([81, 27, 9, 3], dtype=np.uint16)  # 4-digit tail bytes carry a trailing zero digit
_IDX_A = (np.arange(16)[:, None] + 16 * np.arange(5)[None, :])        # bytes 0..15: m + 16n
_IDX_B = (80 + np.arange(8)[:, None] + 8 * np.arange(5)[None, :])     # bytes 16..23: 80 + m + 8n
_IDX_C = (120 + np.arange(2)[:, None] + 2 * np.arange(4)[None, :])    # bytes 24..25: 120 + h + 2n


def trits(N: int, K: int, seed: int = 0) -> np.ndarray:
    """int8 [N][K], i.i.d. uniform over {-1, 0, +1}."""
    return (np.random.default_rng(seed).integers(0, 3, size=(N, K), dtype=np.int8) - 1).astype(np.int8)


def block_scales(N: int, K: int, seed: int = 1) -> np.ndarray:
    """uint16 [N][K/128]: fp16 bits of |N(0,1)| * 0.02 (round to nearest even)."""
    g = np.random.default_rng(seed).standard_normal(size=(N, K // 128)).astype(np.float32)
    return (np.abs(g) * np.float32(0.02)).astype(np.float16).view(np.uint16)


def encode_ptq1_0(t: np.ndarray, scales: np.ndarray, chunk_rows: int = 2048) -> np.ndarray:
    """trits int8 [N][K] + fp16 scale bits [N][K/128] -> PTQ1_0 bytes uint8 [N][K/128*28]."""
    N, K = t.shape
    nb = K // 128
    out = np.empty((N, nb, 28), dtype=np.uint8)
    for r0 in range(0, N, chunk_rows):
        r1 = min(N, r0 + chunk_rows)
        d = (t[r0:r1].reshape(r1 - r0, nb, 128) + 1).astype(np.uint16)  # digits 0..2
        va = (d[..., _IDX_A] * _W5).sum(-1)
        vb = (d[..., _IDX_B] * _W5).sum(-1)
        vc = (d[..., _IDX_C] * _W4).sum(-1)
        v = np.concatenate([va, vb, vc], axis=-1).astype(np.uint32)
        out[r0:r1, :, :26] = ((v * 256 + 242) // 243).astype(np.uint8)
        sc = scales[r0:r1].astype(np.uint16)
        out[r0:r1, :, 26] = (sc & 0xFF).astype(np.uint8)
        out[r0:r1, :, 27] = (sc >> 8).astype(np.uint8)
    return out.reshape(N, nb * 28)


def ternary_ptq(N: int, K: int, seed: int = 0) -> np.ndarray:
    """PTQ1_0 bytes of a seeded [N][K] ternary matrix (weights seed, scales seed + 1)."""
    return encode_ptq1_0(trits(N, K, seed), block_scales(N, K, seed + 1))


def activations(M: int, K: int, seed: int = 2) -> np.ndarray:
    """fp32 [M][K] activations drawn from N(0, 1)."""
    return np.random.default_rng(seed).standard_normal(size=(M, K)).astype(np.float32)


def gemv_bytes(N: int, K: int, M: int = 1, add: bool = False) -> int:
    """Algorithmic HBM bytes of one GEMV launch: codes + fp16 scales + Q8 activation
    (q + d + s) + fp32 output (read too in add mode)."""
    b = N * K // 4 + N * (K // 128) * 2 + M * (K + (K // 32) * 8) + M * N * 4
    return b + (M * N * 4 if add else 0)
