"""numpy wrappers over the CPU oracle — TEST INFRASTRUCTURE ONLY.

Two libraries, built by oracle/Makefile:
  * ``_build/liboracle.so`` — oracle.c, the plain-C restatement of the
    reference path (always present once built; travels to GPU hosts);
  * ``_ref/libbtf_ref.so`` — the reference's own sources compiled in place,
    plus ref_shim.cpp (present where the reference tree was available at build
    time; the built file also travels);
  * ``_ref/libbtf_ref_gpu.so`` — the reference's own CUDA kernels
    (src/cuda/kernels.cu) for sm_100a with ref_gpu_shim.cu: its GPU GEMV, timed
    by bench.py as the GPU baseline.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
``--impl reference`` legs may import this module, and only as the checker or
the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libbtf_ref.so")
REF_GPU_SO = os.path.join(HERE, "_ref", "libbtf_ref_gpu.so")

_vp, _i32, _i64, _u16, _u32, _f32 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint16,
                                     ctypes.c_uint32, ctypes.c_float)


def build(quiet: bool = True) -> None:
    """Runs oracle/Makefile (the reference part only if the reference tree exists)."""
    subprocess.run(["make", "-C", HERE], check=True,
                   stdout=subprocess.DEVNULL if quiet else None, stderr=None)


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


class Oracle:
    """oracle.c: the C restatement."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        sig = {
            "orc_f32_to_f16": (_u16, [_f32]),
            "orc_f16_to_f32": (_f32, [_u16]),
            "orc_ptq_trit": (_i32, [_vp, _i32]),
            "orc_ptq_encode": (None, [_vp, _vp, _i64, _vp]),
            "orc_ptq_quant_row": (None, [_vp, _vp, _i64]),
            "orc_repack_t2": (None, [_vp, _i64, _i64, _vp, _vp]),
            "orc_t2_code": (_i32, [_vp, _i64]),
            "orc_q8_block": (_i32, [_vp, _vp, _vp]),
            "orc_q8_rows": (None, [_vp, _i64, _i32, _i32, _vp, _vp, _vp]),
            "orc_round_q8_0": (None, [_vp, _i64, _vp]),
            "orc_sub_dot": (_i32, [_u32, _u32, _vp]),
            "orc_idot": (None, [_vp, _i64, _i64, _vp, _vp, _i32, _vp]),
            "orc_gemv": (None, [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _vp, _i64, _i32, _i32]),
            "orc_gemv_swiglu": (None, [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _vp, _i64, _i32]),
            "orc_gemv_f64": (None, [_vp, _vp, _i64, _i64, _vp, _vp, _i32, _vp]),
            "orc_rmsnorm": (None, [_vp, _vp, _i64, _f32, _vp]),
            "orc_hadamard_input": (None, [_i32, _i32, _i32, _i32, _vp, _vp, _i64, _vp]),
            "orc_prep_rows": (None, [_vp, _i64, _i32, _i32, _vp, _f32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp,
                                     _vp]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L

    # -- PTQ1_0
    def ptq_encode(self, trits: np.ndarray, scales: np.ndarray) -> np.ndarray:
        t = np.ascontiguousarray(trits, dtype=np.int8)
        s = np.ascontiguousarray(scales, dtype=np.uint16)
        N, K = t.shape
        out = np.empty((N, K // 128 * 28), dtype=np.uint8)
        self.L.orc_ptq_encode(_p(t), _p(s), N * (K // 128), _p(out))
        return out

    def ptq_quant_rows(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        N, K = w.shape
        out = np.empty((N, K // 128 * 28), dtype=np.uint8)
        for r in range(N):
            self.L.orc_ptq_quant_row(w[r].ctypes.data, out[r].ctypes.data, K)
        return out

    def ptq_trits(self, src: np.ndarray, K: int) -> np.ndarray:
        """All trits of a PTQ1_0 [N][K/128*28] array, by the digit rule."""
        N = src.shape[0]
        blk = np.ascontiguousarray(src, dtype=np.uint8).reshape(N * (K // 128), 28)
        out = np.empty((N * (K // 128), 128), dtype=np.int8)
        for b in range(blk.shape[0]):
            p = blk[b].ctypes.data
            out[b] = [self.L.orc_ptq_trit(p, e) for e in range(128)]
        return out.reshape(N, K)

    # -- T2
    def repack_t2(self, src: np.ndarray, N: int, K: int):
        src = np.ascontiguousarray(src, dtype=np.uint8)
        codes = np.empty((N, K // 4), dtype=np.uint8)
        scales = np.empty((N, K // 128), dtype=np.uint16)
        self.L.orc_repack_t2(_p(src), N, K, _p(codes), _p(scales))
        return codes, scales

    # -- Q8
    def q8_rows(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M, K = x.shape
        q = np.empty((M, K), dtype=np.int8)
        d = np.empty((M, K // 32), dtype=np.float32)
        s = np.empty((M, K // 32), dtype=np.int32)
        self.L.orc_q8_rows(_p(x), K, M, K, _p(q), _p(d), _p(s))
        return q, d, s

    def round_q8_0(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.L.orc_round_q8_0(_p(x), x.size, _p(out))
        return out

    # -- dots and GEMV
    def idot(self, codes, K: int, q, s) -> np.ndarray:
        N = codes.shape[0]
        M = q.shape[0]
        out = np.empty((M, N, K // 32), dtype=np.int32)
        self.L.orc_idot(_p(np.ascontiguousarray(codes)), N, K, _p(np.ascontiguousarray(q)),
                        _p(np.ascontiguousarray(s)), M, _p(out))
        return out

    def gemv(self, codes, scales, K: int, q, d, s, y: Optional[np.ndarray] = None, add: bool = False,
             threads: int = 1) -> np.ndarray:
        N = codes.shape[0]
        M = q.shape[0]
        if y is None:
            y = np.zeros((M, N), dtype=np.float32)
        self.L.orc_gemv(_p(codes), _p(scales), N, K, _p(q), _p(d), _p(s), M, _p(y), y.shape[1], 1 if add else 0,
                        threads)
        return y

    def gemv_swiglu(self, gate, up, K: int, q, d, s, threads: int = 1) -> np.ndarray:
        (gc, gs), (uc, us) = gate, up
        N = gc.shape[0]
        M = q.shape[0]
        y = np.zeros((M, N), dtype=np.float32)
        self.L.orc_gemv_swiglu(_p(gc), _p(gs), _p(uc), _p(us), N, K, _p(q), _p(d), _p(s), M, _p(y), N, threads)
        return y

    def gemv_f64(self, codes, scales, K: int, q, d) -> np.ndarray:
        N = codes.shape[0]
        M = q.shape[0]
        y = np.zeros((M, N), dtype=np.float64)
        self.L.orc_gemv_f64(_p(codes), _p(scales), N, K, _p(q), _p(d), M, _p(y))
        return y


def _as_f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _prep_methods(prefix):
    """rmsnorm / hadamard_input wrappers shared by Oracle and Reference."""

    def rmsnorm(self, x, w, eps):
        x, w = _as_f32(x), _as_f32(w)
        y = np.empty_like(x)
        getattr(self.L, prefix + "rmsnorm")(_p(x), _p(w), x.size, eps, _p(y))
        return y

    def hadamard_input(self, x, block, perm=(0, 0, 0), signs=None):
        x, sg = _as_f32(x), _as_f32(signs)
        out = np.empty_like(x)
        getattr(self.L, prefix + "hadamard_input")(block, perm[0], perm[1], perm[2], _p(sg), _p(x), x.size, _p(out))
        return out

    return rmsnorm, hadamard_input


Oracle.rmsnorm, Oracle.hadamard_input = _prep_methods("orc_")


def _oracle_prep_rows(self, x, normw=None, eps=1e-6, block=0, perm=(0, 0, 0), signs=None):
    """Host prep of M rows (norm, transform, Q8): q, d, s and the normalised rows."""
    x = _as_f32(x)
    M, n = x.shape
    q = np.empty((M, n), np.int8)
    d = np.empty((M, n // 32), np.float32)
    s = np.empty((M, n // 32), np.int32)
    xn = np.empty((M, n), np.float32)
    self.L.orc_prep_rows(_p(x), n, M, n, _p(_as_f32(normw)), eps, block, perm[0], perm[1], perm[2], _p(_as_f32(signs)),
                         _p(xn), _p(q), _p(d), _p(s))
    return q, d, s, xn


Oracle.prep_rows = _oracle_prep_rows


class Reference:
    """libbtf_ref.so: the reference's own compiled code (see ref_shim.cpp)."""

    def __init__(self, path: str = REF_SO):
        L = ctypes.CDLL(path)
        sig = {
            "ref_f32_to_f16": (_u16, [_f32]),
            "ref_f16_to_f32": (_f32, [_u16]),
            "ref_ptq_quant_row": (None, [_vp, _vp, _i64]),
            "ref_ptq_trit": (_i32, [_vp, _i32]),
            "ref_repack_rows": (None, [_vp, _i64, _i64, _vp, _vp]),
            "ref_packed_code": (_i32, [_vp, _i64]),
            "ref_q8_block": (_i32, [_vp, _vp, _vp]),
            "ref_round_q8_0": (None, [_vp, _i64, _vp]),
            "ref_sub_dot": (_i32, [_u32, _u32, _vp]),
            "ref_pool_create": (_vp, [_i32]),
            "ref_pool_destroy": (None, [_vp]),
            "ref_pool_size": (_i32, [_vp]),
            "ref_gemv": (None, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _vp, _i64, _i32]),
            "ref_matvec_raw": (None, [_vp, _vp, _i64, _i64, _vp, _vp]),
            "ref_rmsnorm": (None, [_vp, _vp, _i64, _f32, _vp]),
            "ref_hadamard_input": (None, [_i32, _i32, _i32, _i32, _vp, _vp, _i64, _vp]),
            "ref_synth_write": (_i32, [ctypes.c_char_p, _i32, ctypes.c_uint64, _vp]),
            "ref_emu_open": (_vp, [ctypes.c_char_p, _i32, _i32, _i32]),
            "ref_emu_step": (_i32, [_vp, ctypes.c_int32, _vp]),
            "ref_emu_reset": (None, [_vp]),
            "ref_emu_close": (None, [_vp]),
            "ref_emu_hparams": (None, [_vp, _vp]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L
        self._pool = None

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def pool(self, threads: int):
        if self._pool is None or self.L.ref_pool_size(self._pool) != threads:
            if self._pool is not None:
                self.L.ref_pool_destroy(self._pool)
            self._pool = self.L.ref_pool_create(threads)
        return self._pool

    def ptq_quant_rows(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        N, K = w.shape
        out = np.empty((N, K // 128 * 28), dtype=np.uint8)
        for r in range(N):
            self.L.ref_ptq_quant_row(w[r].ctypes.data, out[r].ctypes.data, K)
        return out

    def repack_rows(self, src: np.ndarray, N: int, K: int):
        src = np.ascontiguousarray(src, dtype=np.uint8)
        codes = np.empty((N, K // 4), dtype=np.uint8)
        scales = np.empty((N, K // 128), dtype=np.uint16)
        self.L.ref_repack_rows(_p(src), N, K, _p(codes), _p(scales))
        return codes, scales

    def q8_rows(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M, K = x.shape
        q = np.empty((M, K), dtype=np.int8)
        d = np.empty((M, K // 32), dtype=np.float32)
        s = np.empty((M, K // 32), dtype=np.int32)
        for m in range(M):
            for b in range(K // 32):
                s[m, b] = self.L.ref_q8_block(x[m, b * 32:].ctypes.data, q[m, b * 32:].ctypes.data,
                                              d[m, b:].ctypes.data)
        return q, d, s

    def round_q8_0(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.L.ref_round_q8_0(_p(x), x.size, _p(out))
        return out

    def gemv(self, codes, scales, K: int, q, d, s, y: Optional[np.ndarray] = None, add: bool = False,
             threads: int = 1) -> np.ndarray:
        N = codes.shape[0]
        M = q.shape[0]
        if y is None:
            y = np.zeros((M, N), dtype=np.float32)
        pool = self.pool(threads) if threads > 1 else None
        self.L.ref_gemv(pool, _p(codes), _p(scales), N, K, _p(q), _p(d), _p(s), M, _p(y), y.shape[1],
                        1 if add else 0)
        return y

    def matvec_raw(self, src: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
        y = np.zeros(N, dtype=np.float32)
        self.L.ref_matvec_raw(None, _p(np.ascontiguousarray(src)), N, K, _p(np.ascontiguousarray(x, np.float32)),
                              _p(y))
        return y


class ReferenceGPU:
    """libbtf_ref_gpu.so: the reference's own CUDA launchers (src/cuda/kernels.cuh:17-56)
    over device pointers (ints) and a stream handle (int or None)."""

    def __init__(self, path: str = REF_GPU_SO):
        L = ctypes.CDLL(path)
        vpp, ip = ctypes.POINTER(_vp), ctypes.POINTER(_i32)
        sig = {
            "ref_gpu_last_error": (ctypes.c_char_p, []),
            "ref_gpu_init": (_i32, [_i32]),
            "ref_gpu_max_nb": (_i32, [_i32]),
            "ref_gpu_repack": (_i32, [_vp, ctypes.c_longlong, _vp, _vp, _vp]),
            "ref_gpu_quant": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
            "ref_gpu_gemv": (_i32, [vpp, vpp, ip, vpp, ip, _i32, _i32, _i32, _vp, _vp, _vp, _i32, _vp]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_GPU_SO)

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what}: {self.L.ref_gpu_last_error().decode()}")

    def init(self, device: int) -> None:
        self._check(self.L.ref_gpu_init(device), "kernels_init")

    def repack(self, src: int, nblocks: int, codes: int, scales: int, stream=None) -> None:
        self._check(self.L.ref_gpu_repack(src, nblocks, codes, scales, stream), "launch_repack")

    def quant(self, x: int, ldx: int, M: int, n: int, q: int, d: int, s: int, stream=None) -> None:
        self._check(self.L.ref_gpu_quant(x, ldx, M, n, q, d, s, stream), "launch_prep")

    def gemv(self, segs, K: int, M: int, q: int, d: int, s: int, mode: int, stream=None) -> None:
        """segs: [(codes, scales, N, y, ldy)] device pointers."""
        n = len(segs)
        codes = (_vp * 3)(*[sg[0] for sg in segs])
        scales = (_vp * 3)(*[sg[1] for sg in segs])
        Ns = (_i32 * 3)(*[sg[2] for sg in segs])
        ys = (_vp * 3)(*[sg[3] for sg in segs])
        lds = (_i32 * 3)(*[sg[4] for sg in segs])
        self._check(self.L.ref_gpu_gemv(codes, scales, Ns, ys, lds, n, K, M, q, d, s, mode, stream), "launch_gemv")


def panel_decode(panels: np.ndarray, N: int, K: int):
    """Independent numpy reader of the panel layout (include/btf_b200.h) -> T2 codes [N][K/4], scales [N][K/128].

    Written from the layout description, not from the library, so a test that
    compares it with the reference T2 checks the library's layout end to end.
    Returns the padded arrays too when N or K are not multiples of 8 / 1024."""
    S = (K + 1023) // 1024
    G = (N + 7) // 8
    p = np.asarray(panels, dtype=np.uint8).reshape(G, S, 2176)
    # codes: [G][S][quad h][half v][sub-block l][word i] uint32
    w = p[:, :, :2048].copy().view("<u4").reshape(G, S, 2, 2, 32, 4).astype(np.uint32)
    # code of row 4h+k, column 32l + 16v + 4i + c: (w >> (8c + 2k)) & 3
    c = np.arange(4, dtype=np.uint32)
    k = np.arange(4, dtype=np.uint32)
    codes = (w[..., None, None] >> (8 * c[None, :] + 2 * k[:, None])) & 3  # [..., k, c]
    # -> [G][h][k][S][l][v][i][c] = row (8G + 4h + k), column (1024 S + 32 l + 16 v + 4 i + c)
    codes = codes.transpose(0, 2, 6, 1, 4, 3, 5, 7).reshape(G * 8, S * 1024).astype(np.uint8)
    # back to T2 bytes: column e of a block at byte (e//32)*8 + ((e//16)%2)*4 + e%4, shift ((e//4)%4)*2
    e = np.arange(S * 1024)
    byte = (e // 128) * 32 + ((e % 128) // 32) * 8 + (((e % 128) // 16) % 2) * 4 + (e % 4)
    shift = (((e % 128) // 4) % 4) * 2
    t2 = np.zeros((G * 8, S * 256), dtype=np.uint8)
    for sh in range(0, 8, 2):
        sel = shift == sh
        np.bitwise_or.at(t2, (slice(None), byte[sel]), (codes[:, sel] << sh).astype(np.uint8))
    sc = p[:, :, 2048:].copy().view(np.uint16).reshape(G, S, 8, 8).transpose(0, 3, 1, 2).reshape(G * 8, S * 8)
    return np.ascontiguousarray(t2[:N, :K // 4]), np.ascontiguousarray(sc[:N, :K // 128])


Reference.rmsnorm, Reference.hadamard_input = _prep_methods("ref_")


# bd::SynthOptions defaults (ref/bonsai-decoder/include/bd/synth.hpp:17-30), in
# the order ref_synth_write takes them.
SYNTH_DEFAULTS = dict(n_embd=128, n_ff=256, n_head=4, n_head_kv=2, head_dim=32, n_rot=16, d_state=32, n_group=2,
                      dt_rank=4, hadamard_block=64, hadamard=1, explicit_signs=1, gdn_v_grouped=1, small_mat_type=30)


def synth_model(ref: "Reference", path: str, n_layer: int = 8, seed: int = 1, **over) -> None:
    """Writes the reference's synthetic qwen35 GGUF (bd::make_synth_qwen35)."""
    import numpy as np

    o = dict(SYNTH_DEFAULTS, **over)
    geom = np.array([o[k] for k in SYNTH_DEFAULTS], dtype=np.int32)
    if ref.L.ref_synth_write(path.encode(), n_layer, seed, geom.ctypes.data) != 0:
        raise RuntimeError("ref_synth_write failed")


class Emulator:
    """The reference's CPU emulator of its CUDA decode step (btf::make_emu_decoder)."""

    HP = ("n_layer", "n_embd", "n_ff", "n_vocab", "n_head", "n_head_kv", "head_dim", "n_rot", "d_state", "n_group",
          "dt_rank", "d_inner", "conv_kernel")

    def __init__(self, ref: "Reference", path: str, n_ctx: int = 64, round_q_f16: bool = True, threads: int = 8):
        import numpy as np

        self.ref = ref
        self.h = ref.L.ref_emu_open(path.encode(), n_ctx, int(round_q_f16), threads)
        if not self.h:
            raise RuntimeError("ref_emu_open failed")
        hp = np.zeros(13, dtype=np.int32)
        ref.L.ref_emu_hparams(self.h, hp.ctypes.data)
        self.hp = dict(zip(self.HP, (int(v) for v in hp)))

    def step(self, token: int):
        import numpy as np

        lg = np.empty(self.hp["n_vocab"], dtype=np.float32)
        nxt = self.ref.L.ref_emu_step(self.h, token, lg.ctypes.data)
        return nxt, lg

    def reset(self) -> None:
        self.ref.L.ref_emu_reset(self.h)

    def close(self) -> None:
        if self.h:
            self.ref.L.ref_emu_close(self.h)
            self.h = None
