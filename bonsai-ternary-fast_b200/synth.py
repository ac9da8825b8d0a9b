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


# ---------------------------------------------------------------- synthetic qwen35 GGUF
_GGUF_U32, _GGUF_F32, _GGUF_STR = 4, 6, 8
_T_F32, _T_PTQ1_0 = 0, 143


def qwen35_tensors(dims: dict):
    """(name, ne, type) of every tensor a qwen35 GGUF of this geometry holds, in
    the order bd::Model::bind reads them (ref/bonsai-decoder/src/model.cpp:157-205);
    ne[0] is the input width. Every layer il with (il + 1) % 4 != 0 is a gated
    delta-net layer, the others full attention."""
    E, F, V = dims["n_embd"], dims["n_ff"], dims["n_vocab"]
    H, HK, HD = dims["n_head"], dims["n_head_kv"], dims["head_dim"]
    NV, DK, NK, KC = dims["dt_rank"], dims["d_state"], dims["n_group"], dims["conv_kernel"]
    DI = dims.get("d_inner") or NV * DK
    C = 2 * DK * NK + DI
    out = [("token_embd.weight", (E, V), _T_PTQ1_0), ("output_norm.weight", (E,), _T_F32),
           ("output.weight", (E, V), _T_PTQ1_0)]
    for il in range(dims["n_layer"]):
        b = f"blk.{il}."
        out += [(b + "attn_norm.weight", (E,), _T_F32), (b + "post_attention_norm.weight", (E,), _T_F32),
                (b + "ffn_gate.weight", (E, F), _T_PTQ1_0), (b + "ffn_up.weight", (E, F), _T_PTQ1_0),
                (b + "ffn_down.weight", (F, E), _T_PTQ1_0)]
        if (il + 1) % 4:
            out += [(b + "attn_qkv.weight", (E, C), _T_PTQ1_0), (b + "attn_gate.weight", (E, DI), _T_PTQ1_0),
                    (b + "ssm_alpha.weight", (E, NV), _T_F32), (b + "ssm_beta.weight", (E, NV), _T_F32),
                    (b + "ssm_a", (NV,), _T_F32), (b + "ssm_dt.bias", (NV,), _T_F32),
                    (b + "ssm_conv1d.weight", (KC, C), _T_F32), (b + "ssm_norm.weight", (DI // NV,), _T_F32),
                    (b + "ssm_out.weight", (DI, E), _T_PTQ1_0)]
        else:
            out += [(b + "attn_q.weight", (E, 2 * H * HD), _T_PTQ1_0), (b + "attn_k.weight", (E, HK * HD), _T_PTQ1_0),
                    (b + "attn_v.weight", (E, HK * HD), _T_PTQ1_0), (b + "attn_output.weight", (H * HD, E), _T_PTQ1_0),
                    (b + "attn_q_norm.weight", (HD,), _T_F32), (b + "attn_k_norm.weight", (HD,), _T_F32)]
    return out


def _vector(name: str, n: int, fan_in: int, rng) -> np.ndarray:
    if name.endswith("ssm_a"):
        return -rng.uniform(0.05, 1.0, n).astype(np.float32)
    if name.endswith("ssm_dt.bias") or name.endswith("ssm_conv1d.weight"):
        return (rng.standard_normal(n) * (1.0 if "dt" in name else 0.3)).astype(np.float32)
    if name.endswith("ssm_alpha.weight") or name.endswith("ssm_beta.weight"):
        return (rng.standard_normal(n) / np.sqrt(fan_in)).astype(np.float32)
    return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)  # norms


def write_qwen35_gguf(path: str, dims: dict, seed: int = 0, pool_rows: int = 1024) -> int:
    """Writes a qwen35 GGUF (v3) of geometry `dims` (the btf_decoder_dims fields)
    with seeded weights: every ternary matrix in PTQ1_0, every vector in F32, no
    Hadamard metadata. It stands in for bd::make_synth_qwen35
    (ref/bonsai-decoder/src/synth.cpp), which has a fixed vocabulary.

    Matrix rows come from `pool_rows` encoded rows of the widest input. A prefix
    of whole 128-blocks of a PTQ1_0 row is a valid narrower row. Row r of
    matrix i is pool row (r + 7919 i) mod pool_rows, so a model of billions of
    weights writes at file speed. Returns the file size in bytes."""
    import struct

    rng = np.random.default_rng(seed)
    tensors = qwen35_tensors(dims)
    kmax = max(ne[0] for _, ne, t in tensors if t == _T_PTQ1_0)
    pool = ternary_ptq(pool_rows, kmax, seed=seed + 1)
    p = "qwen35."
    kv = [("general.architecture", _GGUF_STR, "qwen35"), ("general.alignment", _GGUF_U32, 32)]
    for key, field in (("block_count", "n_layer"), ("embedding_length", "n_embd"), ("feed_forward_length", "n_ff"),
                       ("attention.head_count", "n_head"), ("attention.head_count_kv", "n_head_kv"),
                       ("attention.key_length", "head_dim"), ("attention.value_length", "head_dim"),
                       ("rope.dimension_count", "n_rot"), ("ssm.conv_kernel", "conv_kernel"),
                       ("ssm.state_size", "d_state"), ("ssm.group_count", "n_group"),
                       ("ssm.time_step_rank", "dt_rank")):
        kv.append((p + key, _GGUF_U32, int(dims[field])))
    kv += [(p + "ssm.inner_size", _GGUF_U32, int(dims.get("d_inner") or dims["dt_rank"] * dims["d_state"])),
           (p + "full_attention_interval", _GGUF_U32, 4),
           (p + "rope.freq_base", _GGUF_F32, float(dims.get("rope_base", 1e7))),
           (p + "attention.layer_norm_rms_epsilon", _GGUF_F32, float(dims.get("rms_eps", 1e-6)))]

    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for key, t, v in kv:
        head += s(key) + struct.pack("<I", t)
        head += s(v) if t == _GGUF_STR else struct.pack("<I" if t == _GGUF_U32 else "<f", v)
    sizes, off = [], 0
    for name, ne, t in tensors:
        n = int(np.prod(ne))
        nbytes = n * 4 if t == _T_F32 else n // 128 * 28
        head += s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
        head += struct.pack("<IQ", t, off)
        sizes.append(nbytes)
        off += (nbytes + 31) // 32 * 32
    head += b"\0" * ((-len(head)) % 32)
    by_width = {}
    with open(path, "wb") as f:
        f.write(head)
        for i, ((name, ne, t), nbytes) in enumerate(zip(tensors, sizes)):
            if t == _T_F32:
                blob = _vector(name, int(np.prod(ne)), ne[0], rng).tobytes()
                f.write(blob)
            else:
                K, N = ne
                if K not in by_width:
                    by_width[K] = np.ascontiguousarray(pool[:, :K // 128 * 28])
                w = by_width[K]
                r, start = 0, (i * 7919) % pool_rows
                while r < N:  # contiguous runs of pool rows
                    n = min(N - r, pool_rows - start)
                    f.write(memoryview(w[start:start + n]))
                    r, start = r + n, 0
            f.write(b"\0" * ((-nbytes) % 32))
        return f.tell()
