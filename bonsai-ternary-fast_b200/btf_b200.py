"""Python host mirror of the btf_b200 C ABI (include/btf_b200.h).

This module is the Python face of the B200 ternary GEMV/GEMM library. It
mirrors the reference's launcher interface, ``btf::cuda`` in
src/cuda/kernels.cuh:17-56 (kernels_init, gemv_max_nb, launch_repack,
launch_gemv with GemvSeg / Q8Act / GemvMode), with the same argument meaning
and the same error behaviour: a bad argument or a failed launch raises
``RuntimeError`` (the reference throws ``std::runtime_error``).

Device memory is held in torch tensors (torch is only the allocator and the
stream source here); every kernel runs from ``libbtf_b200.so``, built in-tree
by ``make -C bonsai-ternary-fast_b200``. There is no CPU fallback: if the
library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
# BTF_B200_LIB selects another build of the library (e.g. a tuning variant)
LIB_PATH = os.environ.get("BTF_B200_LIB", os.path.join(HERE, "libbtf_b200.so"))

STORE, ADD, SWIGLU = 0, 1, 2  # GemvMode values (src/cuda/kernels.cuh:53)
PANEL_ROWS, PANEL_COLS, PANEL_BYTES = 8, 1024, 2176

# Every symbol include/btf_b200.h declares; tests check the library exports them.
EXPORTS = (
    "btf_status_string", "btf_last_error", "btf_version", "btf_init", "btf_gemv_max_nb",
    "btf_panel_bytes", "btf_t2_codes_bytes", "btf_t2_scales_bytes",
    "btf_repack_panels", "btf_repack_panels_host", "btf_repack_t2", "btf_t2_to_panels", "btf_panels_to_t2",
    "btf_quant_q8", "btf_gemv", "btf_gemv_f32", "btf_device_error", "btf_gemv_idot", "btf_gemm",
    "btf_gemv_gather", "btf_alloc", "btf_free", "btf_ipc_handle", "btf_ipc_open", "btf_ipc_close",
    "btf_gather_epoch_advance", "btf_gather_wait", "btf_gather_barrier", "btf_prep",
    "btf_gguf_open", "btf_gguf_close", "btf_gguf_tensor_count", "btf_gguf_find", "btf_gguf_tensor",
    "btf_gguf_load_panels", "btf_decoder_open", "btf_decoder_synthetic", "btf_decoder_step", "btf_decoder_run",
    "btf_decoder_reset", "btf_decoder_close", "btf_decoder_get_info", "btf_decoder_synthetic_tp",
    "btf_decoder_arena", "btf_decoder_connect", "btf_shard_rows", "btf_decoder_open_tp", "btf_gguf_load_panels_rows",
    "btf_plan_memory", "btf_plan_memory_synthetic", "btf_decoder_stats", "btf_decoder_reset_stats",
    "btf_gemm_f32_noalloc", "btf_chain_program_bytes", "btf_chain_encode", "btf_chain_run", "btf_stamp_next",
    "btf_gemm_idot", "btf_decoder_prefill", "btf_gemm_wm", "btf_gemm_wm_idot", "btf_gemv_mma", "btf_gemv_mma_idot",
)


class GemvSeg(ctypes.Structure):
    """btf_gemv_seg: one matrix of a multi-segment GEMV (GemvSeg, kernels.cuh:46-52)."""

    _fields_ = [("panels", ctypes.c_void_p), ("N", ctypes.c_int), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int)]


class Q8ActC(ctypes.Structure):
    """btf_q8act: Q8_0 activations (Q8Act, kernels.cuh:27-31)."""

    _fields_ = [("q", ctypes.c_void_p), ("d", ctypes.c_void_p), ("s", ctypes.c_void_p)]


class ChainOpC(ctypes.Structure):
    """btf_chain_op: one matmul call site of a persistent GEMV chain."""

    _fields_ = [("segs", GemvSeg * 3), ("nseg", ctypes.c_int), ("K", ctypes.c_int), ("mode", ctypes.c_int),
                ("x", ctypes.c_void_p), ("ldx", ctypes.c_int), ("normw", ctypes.c_void_p), ("eps", ctypes.c_float)]


class ChainC(ctypes.Structure):
    """btf_chain: an encoded chain (program buffer + launch shape)."""

    _fields_ = [("program", ctypes.c_void_p), ("n_ops", ctypes.c_int), ("M", ctypes.c_int), ("max_K", ctypes.c_int),
                ("grid", ctypes.c_int), ("depth", ctypes.c_int), ("smem", ctypes.c_int)]


_lib: Optional[ctypes.CDLL] = None


MAX_RANKS = 8


class HxC(ctypes.Structure):
    """btf_hx: input transform of a folded-Hadamard weight (kernels.cuh:34-38)."""

    _fields_ = [("block", ctypes.c_int), ("perm_hd", ctypes.c_int), ("perm_nk", ctypes.c_int),
                ("perm_rep", ctypes.c_int), ("signs", ctypes.c_void_p)]


class GgufTensorC(ctypes.Structure):
    """btf_gguf_tensor: one tensor of an open GGUF file."""

    _fields_ = [("name", ctypes.c_char_p), ("n_dims", ctypes.c_int), ("ne", ctypes.c_int64 * 4),
                ("type", ctypes.c_uint32), ("data", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class GatherC(ctypes.Structure):
    """btf_gather (include/btf_b200.h): N-sharded launch with the all-gather in the epilogue."""

    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("peer_y", (ctypes.c_void_p * MAX_RANKS) * 3), ("flags", ctypes.c_void_p * MAX_RANKS),
                ("expect", ctypes.c_void_p), ("done", ctypes.c_void_p),
                ("tagged", ctypes.c_int), ("site", ctypes.c_int), ("epoch", ctypes.c_void_p)]


class TaggedBufC(ctypes.Structure):
    """btf_tagged_buf: `words` 64-bit (value, tag) words at p, stored by the launch with `site`."""

    _fields_ = [("p", ctypes.c_void_p), ("words", ctypes.c_int64), ("site", ctypes.c_int)]


class DecoderOptsC(ctypes.Structure):
    _fields_ = [("n_ctx", ctypes.c_int), ("round_q_f16", ctypes.c_int), ("attn_splits", ctypes.c_int),
                ("cuda_graph", ctypes.c_int), ("staging_mb", ctypes.c_int), ("keep_page_cache", ctypes.c_int)]


DIM_FIELDS = ("n_layer", "n_embd", "n_ff", "n_vocab", "n_head", "n_head_kv", "head_dim", "n_rot", "d_state",
              "n_group", "dt_rank", "d_inner", "conv_kernel", "hadamard_block")


class DecoderDimsC(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int) for f in DIM_FIELDS] + [("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float)]


class DecoderInfoC(ctypes.Structure):
    _fields_ = [("dims", DecoderDimsC), ("pos", ctypes.c_int), ("stream", ctypes.c_void_p),
                ("weight_bytes", ctypes.c_uint64), ("state_bytes", ctypes.c_uint64),
                ("kv_bytes_per_token", ctypes.c_uint64), ("logits", ctypes.c_void_p), ("device_bytes", ctypes.c_uint64)]


class StepStatsC(ctypes.Structure):
    """btf_step_stats (StepStats, include/btf/fast.hpp:72-80)."""
    _fields_ = [("steps", ctypes.c_uint64), ("wall_s", ctypes.c_double), ("gpu_s", ctypes.c_double),
                ("weight_xfer_bytes", ctypes.c_uint64), ("weight_xfer_s", ctypes.c_double),
                ("mapped_read_bytes", ctypes.c_uint64)]


PLAN_FIELDS = ("panel_bytes", "vector_bytes", "kv_cache_bytes", "state_bytes", "work_bytes", "device_bytes",
               "pinned_bytes", "staging_bytes", "decode_bytes_fixed", "decode_bytes_per_ctx")


class MemoryPlanC(ctypes.Structure):
    """btf_memory_plan (btf::MemoryPlan, include/btf/fast.hpp:50-69, for the panel layout)."""
    _fields_ = [(f, ctypes.c_uint64) for f in PLAN_FIELDS] + [("n_matrices", ctypes.c_int), ("dims", DecoderDimsC)]


def lib() -> ctypes.CDLL:
    """Loads libbtf_b200.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    sig = {
        "btf_status_string": (ctypes.c_char_p, [i32]),
        "btf_last_error": (ctypes.c_char_p, []),
        "btf_version": (ctypes.c_char_p, []),
        "btf_init": (i32, [i32]),
        "btf_gemv_max_nb": (i32, [i32]),
        "btf_panel_bytes": (i64, [i64, i64]),
        "btf_t2_codes_bytes": (i64, [i64, i64]),
        "btf_t2_scales_bytes": (i64, [i64, i64]),
        "btf_repack_panels": (i32, [vp, i64, i64, vp, vp]),
        "btf_repack_panels_host": (i32, [vp, i64, i64, vp, i32]),
        "btf_repack_t2": (i32, [vp, i64, vp, vp, vp]),
        "btf_t2_to_panels": (i32, [vp, vp, i64, i64, vp, vp]),
        "btf_panels_to_t2": (i32, [vp, i64, i64, vp, vp, vp]),
        "btf_quant_q8": (i32, [vp, i32, i32, i32, Q8ActC, vp]),
        "btf_gemv": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, Q8ActC, i32, vp]),
        "btf_gemv_f32": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, vp, i32, i32, vp]),
        "btf_device_error": (i32, [i32]),
        "btf_gemv_idot": (i32, [vp, i32, i32, i32, Q8ActC, vp, vp]),
        "btf_gemm_idot": (i32, [vp, i32, i32, i32, Q8ActC, vp, vp]),
        "btf_gemm": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, Q8ActC, i32, vp]),
        "btf_gemm_wm": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, Q8ActC, i32, vp]),
        "btf_gemm_wm_idot": (i32, [vp, i32, i32, i32, Q8ActC, vp, vp]),
        "btf_gemv_mma": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, Q8ActC, i32, vp]),
        "btf_gemv_mma_idot": (i32, [vp, i32, i32, i32, Q8ActC, vp, vp]),
        "btf_gemm_f32_noalloc": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, vp, i32, i32, vp]),
        "btf_chain_program_bytes": (i64, [i32]),
        "btf_stamp_next": (i32, [vp]),
        "btf_chain_encode": (i32, [ctypes.POINTER(ChainOpC), i32, i32, vp, ctypes.POINTER(ChainC)]),
        "btf_chain_run": (i32, [ctypes.POINTER(ChainC), vp]),
        "btf_gemv_gather": (i32, [ctypes.POINTER(GemvSeg), i32, i32, i32, Q8ActC, i32, ctypes.POINTER(GatherC), vp]),
        "btf_alloc": (i32, [ctypes.c_size_t, ctypes.POINTER(vp)]),
        "btf_free": (i32, [vp]),
        "btf_ipc_handle": (i32, [vp, ctypes.c_char_p]),
        "btf_ipc_open": (i32, [ctypes.c_char_p, ctypes.POINTER(vp)]),
        "btf_ipc_close": (i32, [vp]),
        "btf_gather_epoch_advance": (i32, [vp, vp]),
        "btf_gather_wait": (i32, [ctypes.POINTER(TaggedBufC), i32, vp, vp]),
        "btf_gather_barrier": (i32, [ctypes.POINTER(GatherC), vp]),
        "btf_prep": (i32, [vp, i32, i32, i32, vp, ctypes.c_float, HxC, vp, i32, Q8ActC, vp]),
        "btf_gguf_open": (i32, [ctypes.c_char_p, ctypes.POINTER(vp)]),
        "btf_gguf_close": (i32, [vp]),
        "btf_gguf_tensor_count": (i64, [vp]),
        "btf_gguf_find": (i64, [vp, ctypes.c_char_p]),
        "btf_gguf_tensor": (i32, [vp, i64, ctypes.POINTER(GgufTensorC)]),
        "btf_gguf_load_panels": (i32, [vp, i64, vp, i64, vp]),
        "btf_decoder_open": (i32, [ctypes.c_char_p, ctypes.POINTER(DecoderOptsC), ctypes.POINTER(vp)]),
        "btf_decoder_synthetic": (i32, [ctypes.POINTER(DecoderDimsC), ctypes.c_uint64, ctypes.POINTER(DecoderOptsC),
                                        ctypes.POINTER(vp)]),
        "btf_decoder_step": (i32, [vp, ctypes.c_int32, vp, ctypes.POINTER(ctypes.c_int32)]),
        "btf_decoder_run": (i32, [vp, i32]),
        "btf_decoder_prefill": (i32, [vp, vp, i32, i32, vp, ctypes.POINTER(ctypes.c_int32)]),
        "btf_decoder_reset": (i32, [vp]),
        "btf_decoder_close": (i32, [vp]),
        "btf_decoder_get_info": (i32, [vp, ctypes.POINTER(DecoderInfoC)]),
        "btf_decoder_synthetic_tp": (i32, [ctypes.POINTER(DecoderDimsC), ctypes.c_uint64, ctypes.POINTER(DecoderOptsC),
                                           i32, i32, ctypes.POINTER(vp)]),
        "btf_decoder_arena": (i32, [vp, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64)]),
        "btf_decoder_connect": (i32, [vp, ctypes.POINTER(vp)]),
        "btf_shard_rows": (i32, [i32, i32, i32, ctypes.POINTER(i32), ctypes.POINTER(i32)]),
        "btf_decoder_open_tp": (i32, [ctypes.c_char_p, ctypes.POINTER(DecoderOptsC), i32, i32, ctypes.POINTER(vp)]),
        "btf_gguf_load_panels_rows": (i32, [vp, i64, i64, i64, vp, i64, vp]),
        "btf_decoder_stats": (i32, [vp, ctypes.POINTER(StepStatsC)]),
        "btf_decoder_reset_stats": (i32, [vp]),
        "btf_plan_memory": (i32, [ctypes.c_char_p, ctypes.POINTER(DecoderOptsC), i32, i32, ctypes.POINTER(MemoryPlanC)]),
        "btf_plan_memory_synthetic": (i32, [ctypes.POINTER(DecoderDimsC), ctypes.POINTER(DecoderOptsC), i32, i32,
                                            ctypes.POINTER(MemoryPlanC)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int, what: str) -> None:
    """Raises RuntimeError for a nonzero status, like the reference's check()."""
    if status != 0:
        L = lib()
        raise RuntimeError(f"{what}: {L.btf_status_string(status).decode()}: {L.btf_last_error().decode()}")


# ---------------------------------------------------------------- torch glue
def _torch():
    import torch  # imported lazily: the CPU-only paths do not need it

    return torch


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream) -> Optional[int]:
    if stream is None:
        return _torch().cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


_initialised = set()


def kernels_init(device: int = 0) -> None:
    """Per-device set-up (btf_init); kernels_init in src/cuda/kernels.cuh:17."""
    check(lib().btf_init(device), "btf_init")
    _initialised.add(device)


def ensure_init(device: int) -> None:
    if device not in _initialised:
        kernels_init(device)


def gemv_max_nb(K: int) -> int:
    """gemv_max_nb (kernels.cuh:20): activation rows per GEMV pass for width K."""
    return lib().btf_gemv_max_nb(K)


def panel_bytes(N: int, K: int) -> int:
    return lib().btf_panel_bytes(N, K)


def t2_codes_bytes(N: int, K: int) -> int:
    return lib().btf_t2_codes_bytes(N, K)


def t2_scales_bytes(N: int, K: int) -> int:
    return lib().btf_t2_scales_bytes(N, K)


@dataclass
class Q8Act:
    """Q8_0 activations on the device: q int8 [M][K], d fp32 [M][K/32], s int32 [M][K/32]."""

    q: object
    d: object
    s: object

    def c(self) -> Q8ActC:
        return Q8ActC(_ptr(self.q), _ptr(self.d), _ptr(self.s))

    @staticmethod
    def empty(M: int, K: int, device) -> "Q8Act":
        torch = _torch()
        return Q8Act(
            torch.empty((M, K), dtype=torch.int8, device=device),
            torch.empty((M, K // 32), dtype=torch.float32, device=device),
            torch.empty((M, K // 32), dtype=torch.int32, device=device),
        )


@dataclass
class PanelMatrix:
    """A ternary [N][K] matrix resident on the device in the panel layout."""

    panels: object  # uint8 tensor of panel_bytes(N, K)
    N: int
    K: int


def repack_panels(ptq_src, N: int, K: int, out=None, stream=None) -> PanelMatrix:
    """PTQ1_0 blocks (uint8 tensor, device or pinned-mapped) -> panel layout on the device.

    Replaces launch_repack (kernels.cuh:24) for the B200 resident layout."""
    torch = _torch()
    dev = ptq_src.device if ptq_src.is_cuda else torch.device("cuda", torch.cuda.current_device())
    ensure_init(dev.index)
    if out is None:
        out = torch.empty(panel_bytes(N, K), dtype=torch.uint8, device=dev)
    check(lib().btf_repack_panels(_ptr(ptq_src), N, K, _ptr(out), _stream(stream)), "btf_repack_panels")
    return PanelMatrix(out, N, K)


def repack_panels_host(ptq_src_np, N: int, K: int, threads: int = 0):
    """Host twin of repack_panels (numpy in, numpy out); btf::repack_rows/repack, src/repack.cpp:16-45."""
    import numpy as np

    src = np.ascontiguousarray(ptq_src_np, dtype=np.uint8)
    out = np.empty(panel_bytes(N, K), dtype=np.uint8)
    check(lib().btf_repack_panels_host(src.ctypes.data, N, K, out.ctypes.data, threads), "btf_repack_panels_host")
    return out


def launch_repack(src, nblocks: int, codes, scales, stream=None) -> None:
    """launch_repack (kernels.cuh:24): PTQ1_0 -> reference T2 codes/scales."""
    check(lib().btf_repack_t2(_ptr(src), nblocks, _ptr(codes), _ptr(scales), _stream(stream)), "btf_repack_t2")


def t2_to_panels(codes, scales, N: int, K: int, out=None, stream=None) -> PanelMatrix:
    torch = _torch()
    if out is None:
        out = torch.empty(panel_bytes(N, K), dtype=torch.uint8, device=codes.device)
    check(lib().btf_t2_to_panels(_ptr(codes), _ptr(scales), N, K, _ptr(out), _stream(stream)), "btf_t2_to_panels")
    return PanelMatrix(out, N, K)


def panels_to_t2(pm: PanelMatrix, stream=None):
    torch = _torch()
    codes = torch.empty(t2_codes_bytes(pm.N, pm.K), dtype=torch.uint8, device=pm.panels.device)
    scales = torch.empty(t2_scales_bytes(pm.N, pm.K) // 2, dtype=torch.int16, device=pm.panels.device)
    check(lib().btf_panels_to_t2(_ptr(pm.panels), pm.N, pm.K, _ptr(codes), _ptr(scales), _stream(stream)),
          "btf_panels_to_t2")
    return codes, scales


def quant_q8(x, act: Optional[Q8Act] = None, stream=None) -> Q8Act:
    """Q8_0 of fp32 rows x [M][K] (the quantising part of launch_prep, kernels.cuh:42-43)."""
    M, K = x.shape
    ensure_init(x.device.index)
    if act is None:
        act = Q8Act.empty(M, K, x.device)
    check(lib().btf_quant_q8(_ptr(x), x.stride(0), M, K, act.c(), _stream(stream)), "btf_quant_q8")
    return act


def launch_gemv(segs: Sequence[tuple], K: int, M: int, act: Q8Act, mode: int = STORE, stream=None) -> None:
    """launch_gemv (kernels.cuh:56). segs: (PanelMatrix, y tensor or None, ldy) per segment."""
    check(lib().btf_gemv(_segs(segs), len(segs), K, M, act.c(), mode, _stream(stream)), "btf_gemv")


def _segs(segs):
    arr = (GemvSeg * len(segs))()
    for i, (pm, y, ldy) in enumerate(segs):
        arr[i] = GemvSeg(_ptr(pm.panels), pm.N, _ptr(y), ldy)
    return arr


def launch_gemv_f32(segs: Sequence[tuple], K: int, M: int, x, mode: int = STORE, stream=None) -> None:
    """Fused quantise + GEMV from fp32 activations x [M][>=K] (btf_gemv_f32)."""
    check(lib().btf_gemv_f32(_segs(segs), len(segs), K, M, _ptr(x), x.stride(0), mode, _stream(stream)),
          "btf_gemv_f32")


def launch_gemm(segs: Sequence[tuple], K: int, M: int, act: Q8Act, mode: int = STORE, stream=None) -> None:
    """Prefill GEMM on the tcgen05 int8 tensor cores (btf_gemm), store / add modes; M <= 64 over
    large matrices runs on the weight-major kernel (btf_gemm_wm)."""
    check(lib().btf_gemm(_segs(segs), len(segs), K, M, act.c(), mode, _stream(stream)), "btf_gemm")


GEMM_WM_MAX_M = 64  # btf_gemm_wm takes 1 <= M <= this


def launch_gemm_wm(segs: Sequence[tuple], K: int, M: int, act: Q8Act, mode: int = STORE, stream=None) -> None:
    """Small-batch GEMM, weight-major on the tcgen05 tensor cores (btf_gemm_wm), 1 <= M <= 64."""
    check(lib().btf_gemm_wm(_segs(segs), len(segs), K, M, act.c(), mode, _stream(stream)), "btf_gemm_wm")


GEMV_MMA_MAX_M = 16  # btf_gemv_mma takes 1 <= M <= this and K <= GEMV_MMA_MAX_K
GEMV_MMA_MAX_K = 8192


def launch_gemv_mma(segs: Sequence[tuple], K: int, M: int, act: Q8Act, mode: int = STORE, stream=None) -> None:
    """Small-batch GEMM on warp-level int8 MMA (btf_gemv_mma), 1 <= M <= 16, K <= 8192, store / add modes."""
    check(lib().btf_gemv_mma(_segs(segs), len(segs), K, M, act.c(), mode, _stream(stream)), "btf_gemv_mma")


GEMM_NOALLOC_MAX_MK = 512 * 17408  # BTF_GEMM_NOALLOC_MAX_MK


def launch_gemm_f32_noalloc(segs: Sequence[tuple], K: int, M: int, x, mode: int = STORE, stream=None) -> None:
    """Prefill GEMM from fp32 activations x [M][>=K] with no allocation (btf_gemm_f32_noalloc): the Q8
    intermediate lives in the library's fixed device array, M * K <= GEMM_NOALLOC_MAX_MK."""
    check(lib().btf_gemm_f32_noalloc(_segs(segs), len(segs), K, M, _ptr(x), x.stride(0), mode, _stream(stream)),
          "btf_gemm_f32_noalloc")


@dataclass
class ChainOp:
    """One matmul call site of a GEMV chain: btf_gemv(segs, K, Q8(prep(x)), mode) with
    prep = RMSNorm with `normw` (None: no norm). segs: (PanelMatrix, y or None, ldy)."""

    segs: Sequence[tuple]
    K: int
    mode: int
    x: object
    normw: object = None
    eps: float = 1e-6


class Chain:
    """A persistent GEMV chain (btf_chain_encode / btf_chain_run): the ops run in
    order in one launch, each reading what the ops before it wrote. The program
    buffer is a device tensor held by this object; the tensors the ops name must
    stay alive (they are kept here)."""

    def __init__(self, ops: Sequence[ChainOp], M: int = 1):
        torch = _torch()
        n = len(ops)
        arr = (ChainOpC * n)()
        for i, op in enumerate(ops):
            c = ChainOpC()
            for k, (pm, y, ldy) in enumerate(op.segs):
                c.segs[k] = GemvSeg(_ptr(pm.panels), pm.N, _ptr(y), ldy)
            c.nseg, c.K, c.mode = len(op.segs), op.K, op.mode
            c.x, c.ldx = _ptr(op.x), op.x.stride(0)
            c.normw, c.eps = _ptr(op.normw), op.eps
            arr[i] = c
        dev = ops[0].x.device
        ensure_init(dev.index)
        nbytes = lib().btf_chain_program_bytes(n)
        self.program = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.c = ChainC()
        check(lib().btf_chain_encode(arr, n, M, _ptr(self.program), ctypes.byref(self.c)), "btf_chain_encode")
        self.ops = list(ops)

    @property
    def grid(self) -> int:
        return self.c.grid

    def run(self, stream=None) -> None:
        check(lib().btf_chain_run(ctypes.byref(self.c), _stream(stream)), "btf_chain_run")


def stamp_next(slot_ptr: Optional[int]) -> None:
    """The next quantiser / GEMV launch from this thread records its end time
    (global timer, ns; atomic max over its CTAs) at device address slot_ptr."""
    check(lib().btf_stamp_next(slot_ptr), "btf_stamp_next")


def device_error(clear: bool = False) -> int:
    """Device error word (nonzero after a bounded device-side wait timed out)."""
    return lib().btf_device_error(1 if clear else 0)


def gemv_idot(pm: PanelMatrix, M: int, act: Q8Act, stream=None):
    """Exact int32 trit dots idot[M][N][K/32] through the GEMV's decode path."""
    torch = _torch()
    out = torch.empty((M, pm.N, pm.K // 32), dtype=torch.int32, device=pm.panels.device)
    check(lib().btf_gemv_idot(_ptr(pm.panels), pm.N, pm.K, M, act.c(), _ptr(out), _stream(stream)), "btf_gemv_idot")
    return out


def gemm_idot(pm: PanelMatrix, M: int, act: Q8Act, stream=None):
    """Exact int32 accumulators idot[M][N][K/32] from the tcgen05 GEMM's tensor memory."""
    torch = _torch()
    out = torch.empty((M, pm.N, pm.K // 32), dtype=torch.int32, device=pm.panels.device)
    check(lib().btf_gemm_idot(_ptr(pm.panels), pm.N, pm.K, M, act.c(), _ptr(out), _stream(stream)), "btf_gemm_idot")
    return out


def gemm_wm_idot(pm: PanelMatrix, M: int, act: Q8Act, stream=None):
    """Exact int32 accumulators idot[M][N][K/32] from the weight-major GEMM's tensor memory (M <= 64)."""
    torch = _torch()
    out = torch.empty((M, pm.N, pm.K // 32), dtype=torch.int32, device=pm.panels.device)
    check(lib().btf_gemm_wm_idot(_ptr(pm.panels), pm.N, pm.K, M, act.c(), _ptr(out), _stream(stream)),
          "btf_gemm_wm_idot")
    return out


def gemv_mma_idot(pm: PanelMatrix, M: int, act: Q8Act, stream=None):
    """Exact int32 accumulators idot[M][N][K/32] from the warp-MMA small-batch GEMM's registers (M <= 16)."""
    torch = _torch()
    out = torch.empty((M, pm.N, pm.K // 32), dtype=torch.int32, device=pm.panels.device)
    check(lib().btf_gemv_mma_idot(_ptr(pm.panels), pm.N, pm.K, M, act.c(), _ptr(out), _stream(stream)),
          "btf_gemv_mma_idot")
    return out


def launch_gemv_gather(segs: Sequence[tuple], K: int, M: int, act: Q8Act, mode: int, gather: GatherC,
                       stream=None) -> None:
    """N-sharded launch_gemv whose epilogue all-gathers the outputs over NVLink (btf_gemv_gather)."""
    check(lib().btf_gemv_gather(_segs(segs), len(segs), K, M, act.c(), mode, ctypes.byref(gather), _stream(stream)),
          "btf_gemv_gather")


def alloc(nbytes: int) -> int:
    """cudaMalloc on the current device (a buffer whose IPC handle maps exactly it)."""
    p = ctypes.c_void_p()
    check(lib().btf_alloc(nbytes, ctypes.byref(p)), "btf_alloc")
    return p.value


def free(ptr: int) -> None:
    check(lib().btf_free(ptr), "btf_free")


def ipc_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(64)
    check(lib().btf_ipc_handle(ptr, buf), "btf_ipc_handle")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    p = ctypes.c_void_p()
    check(lib().btf_ipc_open(handle, ctypes.byref(p)), "btf_ipc_open")
    return p.value


def ipc_close(ptr: int) -> None:
    check(lib().btf_ipc_close(ptr), "btf_ipc_close")


def gather_epoch_advance(epoch_ptr: int, stream=None) -> None:
    """Starts a new tag epoch for tagged N-sharded launches (btf_gather_epoch_advance)."""
    check(lib().btf_gather_epoch_advance(epoch_ptr, _stream(stream)), "btf_gather_epoch_advance")


def gather_wait(bufs, epoch_ptr: int, stream=None) -> None:
    """Waits (bounded, on the device) for the tags of tagged output buffers: bufs = [(ptr, words, site)]."""
    arr = (TaggedBufC * len(bufs))()
    for i, (ptr, words, site) in enumerate(bufs):
        arr[i] = TaggedBufC(ptr, words, site)
    check(lib().btf_gather_wait(arr, len(bufs), epoch_ptr, _stream(stream)), "btf_gather_wait")


def gather_barrier(gather: GatherC, stream=None) -> None:
    """Cross-rank barrier in stream order on the arrival counters (btf_gather_barrier)."""
    check(lib().btf_gather_barrier(ctypes.byref(gather), _stream(stream)), "btf_gather_barrier")


def prep(x, normw=None, eps: float = 1e-6, block: int = 0, perm=(0, 0, 0), signs=None, xn_out=None,
         act: Optional[Q8Act] = None, stream=None) -> Q8Act:
    """launch_prep (kernels.cuh:42-43): RMSNorm -> permutation -> signs -> Hadamard -> Q8_0 (btf_prep)."""
    M, n = x.shape
    ensure_init(x.device.index)
    if act is None:
        act = Q8Act.empty(M, n, x.device)
    hx = HxC(block, perm[0], perm[1], perm[2], _ptr(signs))
    ldxn = xn_out.stride(0) if xn_out is not None else 0
    check(lib().btf_prep(_ptr(x), x.stride(0), M, n, _ptr(normw), eps, hx, _ptr(xn_out), ldxn, act.c(),
                         _stream(stream)), "btf_prep")
    return act


PTQ1_0 = 143


class GgufFile:
    """An open GGUF file (btf_gguf_*): tensor table and PTQ1_0 -> panel loading."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        check(lib().btf_gguf_open(path.encode(), ctypes.byref(h)), "btf_gguf_open")
        self.h = h.value

    def close(self) -> None:
        if self.h:
            lib().btf_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __len__(self) -> int:
        return int(lib().btf_gguf_tensor_count(self.h))

    def find(self, name: str) -> int:
        return int(lib().btf_gguf_find(self.h, name.encode()))

    def tensor(self, index: int) -> dict:
        t = GgufTensorC()
        check(lib().btf_gguf_tensor(self.h, index, ctypes.byref(t)), "btf_gguf_tensor")
        return {"name": t.name.decode(), "ne": list(t.ne)[:t.n_dims], "type": t.type, "data": t.data,
                "bytes": int(t.bytes)}

    def data(self, index: int):
        """The tensor's bytes as a read-only numpy view of the mapping."""
        import numpy as np

        t = self.tensor(index)
        buf = (ctypes.c_uint8 * t["bytes"]).from_address(t["data"])
        return np.frombuffer(buf, dtype=np.uint8)

    def load_panels(self, index: int, staging_bytes: int = 8 << 20, stream=None, rows=None) -> PanelMatrix:
        """A 2-D PTQ1_0 tensor -> resident panels on the current device; rows = (row0, n)
        loads only those rows (row0 a multiple of 8), as one rank's shard."""
        torch = _torch()
        t = self.tensor(index)
        K, N = t["ne"][0], t["ne"][1]
        row0, n = (0, N) if rows is None else rows
        dev = torch.device("cuda", torch.cuda.current_device())
        ensure_init(dev.index)
        out = torch.empty(panel_bytes(n, K), dtype=torch.uint8, device=dev)
        check(lib().btf_gguf_load_panels_rows(self.h, index, row0, n, _ptr(out), staging_bytes, _stream(stream)),
              "btf_gguf_load_panels")
        return PanelMatrix(out, n, K)


def _dims_c(dims: dict) -> DecoderDimsC:
    return DecoderDimsC(*[int(dims.get(f, 0)) for f in DIM_FIELDS], float(dims.get("rope_base", 1e4)),
                        float(dims.get("rms_eps", 1e-6)))


def plan_memory(path: Optional[str] = None, dims: Optional[dict] = None, n_ctx: int = 4096, attn_splits: int = 16,
                world: int = 1, rank: int = 0, staging_mb: int = 64) -> dict:
    """btf_plan_memory: the device and pinned memory a Decoder with these
    arguments would allocate on `rank`, and the bytes one decode step reads
    (btf::plan_memory, src/repack.cpp:142-204). Host only: needs no GPU."""
    o = DecoderOptsC(n_ctx, 1, attn_splits, 1, staging_mb, 0)
    p = MemoryPlanC()
    if path is not None:
        check(lib().btf_plan_memory(path.encode(), ctypes.byref(o), world, rank, ctypes.byref(p)), "btf_plan_memory")
    else:
        check(lib().btf_plan_memory_synthetic(ctypes.byref(_dims_c(dims)), ctypes.byref(o), world, rank,
                                              ctypes.byref(p)), "btf_plan_memory_synthetic")
    r = {f: int(getattr(p, f)) for f in PLAN_FIELDS}
    r["n_matrices"] = p.n_matrices
    r["dims"] = {f: getattr(p.dims, f) for f in DIM_FIELDS}
    return r


def plan_table(plan: dict) -> str:
    """Human-readable plan, one line per item (MemoryPlan::table, src/repack.cpp:125-140)."""
    rows = [(f"ternary matrices in panels ({plan['n_matrices']})", plan["panel_bytes"], "device"),
            ("f32 vectors (norms, ssm, conv1d, signs)", plan["vector_bytes"], "device"),
            ("KV cache fp16", plan["kv_cache_bytes"], "device"),
            ("delta-net + conv state", plan["state_bytes"], "device"),
            ("activations, partials, Q8, argmax", plan["work_bytes"], "device"),
            ("token in/out", plan["pinned_bytes"], "host"),
            ("load staging (peak, freed after load)", plan["staging_bytes"], "host")]
    out = [f"  {w:<44s} {k:<6s} {b:>14d} B  {b / 1048576.0:9.2f} MiB" for w, b, k in rows]
    dev = plan["device_bytes"]
    out.append(f"  {'total resident':<44s} {'device':<6s} {dev:>14d} B  {dev / 1048576.0:9.2f} MiB ({dev / 1e9:.3f} GB)")
    return "\n".join(out) + "\n"


class Decoder:
    """The batch-1 qwen35 decode step (btf_decoder_*): from a GGUF file or from
    seeded synthetic weights of a given geometry (a dict of DIM_FIELDS plus
    rope_base / rms_eps)."""

    def __init__(self, path: Optional[str] = None, dims: Optional[dict] = None, seed: int = 1, n_ctx: int = 4096,
                 round_q_f16: bool = True, attn_splits: int = 16, cuda_graph: bool = True, device: int = 0,
                 world: int = 1, rank: int = 0, staging_mb: int = 64, drop_page_cache: bool = True):
        torch = _torch()
        torch.cuda.set_device(device)
        ensure_init(device)
        o = DecoderOptsC(n_ctx, int(round_q_f16), attn_splits, int(cuda_graph), staging_mb, int(not drop_page_cache))
        h = ctypes.c_void_p()
        if path is not None:
            check(lib().btf_decoder_open_tp(path.encode(), ctypes.byref(o), world, rank, ctypes.byref(h)),
                  "btf_decoder_open")
        else:
            d = _dims_c(dims)
            check(lib().btf_decoder_synthetic_tp(ctypes.byref(d), seed, ctypes.byref(o), world, rank, ctypes.byref(h)),
                  "btf_decoder_synthetic")
        self.h = h.value
        self.world, self.rank, self._peers = world, rank, []

    def close(self) -> None:
        """Frees the decoder. Under tensor parallelism call it on every rank only
        after all ranks have synchronised (no rank still stores into another's arena)."""
        if self.h:
            lib().btf_decoder_close(self.h)
            self.h = None
        for p in self._peers:
            ipc_close(p)
        self._peers = []

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def connect_tp(self) -> None:
        """Tensor parallelism: exchanges the activation arenas' IPC handles over the
        default process group and connects the ranks (collective)."""
        import torch.distributed as dist

        base, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        check(lib().btf_decoder_arena(self.h, ctypes.byref(base), ctypes.byref(nbytes)), "btf_decoder_arena")
        handles = [None] * self.world
        dist.all_gather_object(handles, ipc_handle(base.value))
        arenas = [base.value if r == self.rank else ipc_open(handles[r]) for r in range(self.world)]
        self._peers = [a for r, a in enumerate(arenas) if r != self.rank]
        arr = (ctypes.c_void_p * self.world)(*arenas)
        check(lib().btf_decoder_connect(self.h, arr), "btf_decoder_connect")
        dist.barrier()

    def info(self) -> dict:
        i = DecoderInfoC()
        check(lib().btf_decoder_get_info(self.h, ctypes.byref(i)), "btf_decoder_get_info")
        r = {f: getattr(i.dims, f) for f in DIM_FIELDS}
        r.update(rope_base=i.dims.rope_base, rms_eps=i.dims.rms_eps, pos=i.pos, stream=i.stream,
                 weight_bytes=int(i.weight_bytes), state_bytes=int(i.state_bytes),
                 kv_bytes_per_token=int(i.kv_bytes_per_token), logits=i.logits, device_bytes=int(i.device_bytes))
        return r

    def step(self, token: int, logits: bool = False):
        """One token -> (greedy next token, logits as a numpy array or None)."""
        import numpy as np

        out = np.empty(self.info()["n_vocab"], dtype=np.float32) if logits else None
        nxt = ctypes.c_int32()
        check(lib().btf_decoder_step(self.h, token, out.ctypes.data if logits else None, ctypes.byref(nxt)),
              "btf_decoder_step")
        return nxt.value, out

    def prefill(self, tokens, max_chunk: int = 0, logits: bool = False):
        """The prompt in chunks of up to max_chunk (0: 8) tokens -> (greedy next token,
        logits of the last prompt token or None) (btf_decoder_prefill)."""
        import numpy as np

        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.empty(self.info()["n_vocab"], dtype=np.float32) if logits else None
        nxt = ctypes.c_int32()
        check(lib().btf_decoder_prefill(self.h, toks.ctypes.data, len(toks), max_chunk,
                                        out.ctypes.data if logits else None, ctypes.byref(nxt)), "btf_decoder_prefill")
        return nxt.value, out

    def run(self, steps: int) -> None:
        """`steps` greedy steps on the device (asynchronous on the decoder's stream)."""
        check(lib().btf_decoder_run(self.h, steps), "btf_decoder_run")

    def reset(self) -> None:
        check(lib().btf_decoder_reset(self.h), "btf_decoder_reset")

    def stats(self) -> dict:
        """Steps since reset_stats with their host wall time and device time
        (FastDecoder::stats); waits for a pending run()."""
        s = StepStatsC()
        check(lib().btf_decoder_stats(self.h, ctypes.byref(s)), "btf_decoder_stats")
        return {f: getattr(s, f) for f, _ in StepStatsC._fields_}

    def reset_stats(self) -> None:
        check(lib().btf_decoder_reset_stats(self.h), "btf_decoder_reset_stats")
