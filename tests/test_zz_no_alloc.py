"""btf_gemm_f32_noalloc: the prefill GEMM for callers that cannot allocate.

Some hosts cannot give this library device memory for the Q8 intermediate
between the fp32 activations and the GEMM: an engine that reserves the whole
device up front and hands a plugin only its operand tensors, or a serving loop
that may not call cudaMalloc between steps. For them the library keeps that
intermediate in a fixed device array of its own (M * K <= 512 x 17408).

These tests call the entry point through the C ABI and check it against the
two-call route it replaces (btf_quant_q8 into a caller buffer, then btf_gemm),
with the GEMM tests' tolerance (rel-RMS 1e-5), on two calls in a row: the second
is smaller than the first, so a stale Q8 activation left in the shared array
would show. The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

import synth
from conftest import rel_rms

TOL = 1e-5


def _noalloc(btf, segs, K, M, x, mode):
    """One call of the new entry point through the C ABI (ctypes), on torch's current stream."""
    import torch

    L = btf.lib()
    rc = L.btf_gemm_f32_noalloc(btf._segs(segs), len(segs), K, M, ctypes.c_void_p(x.data_ptr()), x.stride(0), mode,
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, (rc, L.btf_last_error().decode())


def _two_routes(btf, cuda, M, K, N, seed, mode):
    import torch

    src = synth.ternary_ptq(N, K, seed=seed)
    pm = btf.repack_panels(torch.from_numpy(src).to(cuda), N, K)
    x_np = synth.activations(M, K, seed=seed + 1)
    x = torch.from_numpy(x_np).to(cuda)
    y0 = torch.from_numpy(np.random.default_rng(seed).standard_normal((M, N)).astype(np.float32)).to(cuda)
    y_two = y0.clone() if mode == btf.ADD else torch.full((M, N), 7.0, device=cuda)
    y_one = y0.clone() if mode == btf.ADD else torch.full((M, N), -3.0, device=cuda)
    act = btf.quant_q8(x)  # the existing route: a caller-allocated Q8 activation
    btf.launch_gemm([(pm, y_two, N)], K, M, act, mode)
    _noalloc(btf, [(pm, y_one, N)], K, M, x, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    return src, x_np, y0.cpu().numpy(), y_two.cpu().numpy(), y_one.cpu().numpy()


@pytest.mark.gpu
def test_gemm_noalloc_matches_two_call_route(cuda, btf, orc):
    # call 1: the larger case, store mode
    M, K, N = 192, 5120, 200
    _, _, _, y_two, y_one = _two_routes(btf, cuda, M, K, N, seed=31, mode=btf.STORE)
    assert rel_rms(y_one, y_two) <= TOL, rel_rms(y_one, y_two)

    # call 2: smaller, add mode; the array still holds call 1's activation
    M, K, N = 64, 2048, 72
    src, x_np, y0, y_two, y_one = _two_routes(btf, cuda, M, K, N, seed=47, mode=btf.ADD)
    assert rel_rms(y_one, y_two) <= TOL, rel_rms(y_one, y_two)
    codes, scales = orc.repack_t2(src, N, K)
    q, d, s = orc.q8_rows(x_np)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8) + y0
    assert rel_rms(y_one, want) <= TOL, rel_rms(y_one, want)


@pytest.mark.gpu
def test_gemm_noalloc_strided_and_unaligned_x(cuda, btf):
    """x as a strided view (ldx = K + 4) and x at a base pointer 4 bytes past a
    16-byte boundary: both take the quantiser's scalar-load path. Each call is
    compared with the two-call route on the same view, two calls in a row."""
    import torch

    M, K, N = 80, 1024, 96
    src = synth.ternary_ptq(N, K, seed=61)
    pm = btf.repack_panels(torch.from_numpy(src).to(cuda), N, K)
    wide = torch.from_numpy(synth.activations(M, K + 4, seed=62)).to(cuda)
    flat = torch.from_numpy(synth.activations(1, M * K + 4, seed=63).reshape(-1)).to(cuda)
    views = {"strided": wide[:, :K], "offset": flat[1:1 + M * K].view(M, K)}
    assert views["strided"].stride(0) == K + 4 and views["offset"].data_ptr() % 16 == 4
    for name, x in views.items():
        act = btf.Q8Act.empty(M, K, cuda)
        L = btf.lib()
        import ctypes as C

        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = L.btf_quant_q8(C.c_void_p(x.data_ptr()), x.stride(0), M, K, act.c(), st)
        assert rc == 0, L.btf_last_error().decode()
        y_two = torch.full((M, N), 5.0, device=cuda)
        y_one = torch.full((M, N), -5.0, device=cuda)
        btf.launch_gemm([(pm, y_two, N)], K, M, act, btf.STORE)
        _noalloc(btf, [(pm, y_one, N)], K, M, x, btf.STORE)
        torch.cuda.synchronize()
        assert btf.device_error() == 0
        assert rel_rms(y_one.cpu().numpy(), y_two.cpu().numpy()) <= TOL, name


def test_gemm_noalloc_rejects_sizes_beyond_its_array(btf):
    """M * K above the array's size is refused before any CUDA call (runs without a GPU)."""
    L = btf.lib()
    seg = (btf.GemvSeg * 1)()
    K = 17408
    M = btf.GEMM_NOALLOC_MAX_MK // K + 1
    rc = L.btf_gemm_f32_noalloc(seg, 1, K, M, ctypes.c_void_p(16), K, btf.STORE, None)
    assert rc == 1  # BTF_ERR_ARG
    assert "exceeds the static scratch" in L.btf_last_error().decode()
    assert L.btf_gemm_f32_noalloc(seg, 1, 1000, 64, ctypes.c_void_p(16), 1000, btf.STORE, None) == 1  # K % 128
    # a segment without panels is refused before anything is launched
    assert L.btf_gemm_f32_noalloc(seg, 1, 1024, 64, ctypes.c_void_p(16), 1024, btf.STORE, None) == 1
    assert "segment 0" in L.btf_last_error().decode()
