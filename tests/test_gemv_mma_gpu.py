"""GPU parity of the warp-MMA small-batch GEMM (btf_gemv_mma) against the oracle.

The reference serves a batch of M rows as repeated launch_gemv passes
(src/cuda/kernels.cu:805-821) of the math the oracle restates
(src/emu_decoder.cpp:143-165). btf_gemv_mma computes the same outputs for
1 <= M <= 16 and K <= 8192 with int8 warp MMAs. The bar is the GEMM's: every 32-column integer
accumulator equal to the oracle's idot, and fp32 outputs within rel-RMS 1e-5 of
the oracle. Shapes cover M = 1 .. 16 (rows past M masked), row counts that
leave the last 32-row unit with one to four panels or a partial panel, K with
a partial last 512-column stage, warps that walk several units, add mode,
strided outputs, activation scales of 2^18 and more, and the batch-16 lm_head
on a subset of rows.
"""
import numpy as np
import pytest

import synth
from conftest import rel_rms

TOL = 1e-5


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _case(btf, orc, cuda, M, K, N, seed, mode=0, rows=None, ldy=None):
    import torch

    src = synth.ternary_ptq(N, K, seed=seed)
    x = synth.activations(M, K, seed=seed + 1)
    ldy = ldy or N
    y0 = np.random.default_rng(seed).standard_normal((M, ldy)).astype(np.float32)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    act = btf.quant_q8(_dev(x, cuda))
    y = _dev(y0, cuda)
    btf.launch_gemv_mma([(pm, y, ldy)], K, M, act, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    got = y.cpu().numpy()
    assert np.array_equal(got[:, N:], y0[:, N:])  # columns past N untouched
    q, d, s = orc.q8_rows(x)
    sel = slice(None) if rows is None else rows
    codes, scales = orc.repack_t2(src[sel], src[sel].shape[0], K)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    if mode == btf.ADD:
        want = want + y0[:, :N][:, sel]
    g = got[:, :N][:, sel]
    assert rel_rms(g, want) <= TOL, rel_rms(g, want)
    return got


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [
    (1, 1024, 64),     # one activation row, two units
    (5, 1024, 200),    # rows past M masked; the last unit has one panel
    (16, 5120, 300),   # the batch-16 width; a partial last panel (300 = 37 * 8 + 4)
    (16, 640, 130),    # K = 5 blocks: a second stage with one block
    (8, 1152, 72),     # a second slice with one block
    (12, 384, 1000),   # 3 blocks
    (9, 8192, 136),    # the largest K
    (15, 6144, 40),    # the o projection's K
])
def test_gemv_mma_matches_oracle(cuda, btf, orc, M, K, N):
    _case(btf, orc, cuda, M, K, N, seed=M + K + N)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [3, 11, 16])
def test_gemv_mma_add_mode_and_strided_output(cuda, btf, orc, M):
    _case(btf, orc, cuda, M, 1024, 264, seed=50 + M, mode=btf.ADD, ldy=264 + 7)


@pytest.mark.gpu
def test_gemv_mma_many_units_per_warp(cuda, btf, orc):
    # more 32-row units than warps (148 CTAs x 8): every warp walks several units
    # and its ring crosses unit boundaries; rows from the first, middle and last units
    M, K = 16, 512
    N = 148 * 8 * 32 * 3 + 77
    rows = np.r_[0:256, N // 2 - 128:N // 2 + 128, N - 333:N]
    _case(btf, orc, cuda, M, K, N, seed=71, rows=rows)


@pytest.mark.gpu
def test_gemv_mma_lm_head_batch16(cuda, btf, orc):
    # configuration 4's lm_head at batch 16 on rows of the first, a middle and the last units
    M, K, N = 16, 5120, 248320
    sel = np.r_[0:512, N // 2:N // 2 + 256, N - 256:N]
    _case(btf, orc, cuda, M, K, N, seed=3, rows=sel)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(16, 1024, 200), (13, 640, 136), (16, 2048, 130), (7, 384, 64), (1, 5120, 96)])
def test_gemv_mma_integer_accumulators_bit_exact(cuda, btf, orc, M, K, N):
    # the dump form writes each 32-column step's int32 accumulator from the MMA's
    # registers (less its bias); every one must equal the oracle's idot
    # (src/emu_decoder.cpp:154-157)
    src = synth.ternary_ptq(N, K, seed=M)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=M + 1)
    act = btf.quant_q8(_dev(x, cuda))
    got = btf.gemv_mma_idot(pm, M, act).cpu().numpy()
    codes, _ = orc.repack_t2(src, N, K)
    q, d, s = orc.q8_rows(x)
    assert np.array_equal(got, orc.idot(codes, K, q, s))


@pytest.mark.gpu
def test_gemv_mma_matches_weight_major_and_gemv(cuda, btf):
    # the same Q8 input through the warp-MMA GEMM, the weight-major GEMM and
    # 4-row GEMV passes: all three agree
    import torch

    M, K, N = 16, 2048, 192
    src = synth.ternary_ptq(N, K, seed=9)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    act = btf.quant_q8(_dev(synth.activations(M, K, seed=10), cuda))
    ys = [torch.empty((M, N), device=cuda) for _ in range(3)]
    btf.launch_gemv_mma([(pm, ys[0], N)], K, M, act, btf.STORE)
    btf.launch_gemm_wm([(pm, ys[1], N)], K, M, act, btf.STORE)
    for m0 in range(0, M, 4):
        sub = btf.Q8Act(act.q[m0:m0 + 4], act.d[m0:m0 + 4], act.s[m0:m0 + 4])
        btf.launch_gemv([(pm, ys[2][m0:m0 + 4], N)], K, 4, sub, btf.STORE)
    torch.cuda.synchronize()
    a, b, c = (y.cpu().numpy() for y in ys)
    assert rel_rms(a, b) <= TOL and rel_rms(a, c) <= TOL


@pytest.mark.gpu
def test_gemv_mma_large_activation_scales(cuda, btf, orc):
    # scales of 2^18 and above beside ordinary ones: the epilogue multiplies by d
    # itself, so any finite d takes the same path; the oracle gets the same scales
    import torch

    M, K, N = 16, 1024, 136
    src = synth.ternary_ptq(N, K, seed=81)
    x = synth.activations(M, K, seed=82)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    act = btf.quant_q8(_dev(x, cuda))
    act.d[3, 0:4] *= np.float32(2.0 ** 26)
    act.d[13, 9:11] *= np.float32(2.0 ** 34)
    y = torch.empty((M, N), device=cuda)
    btf.launch_gemv_mma([(pm, y, N)], K, M, act, btf.STORE)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    q, _, s = orc.q8_rows(x)
    d = act.d.cpu().numpy()
    assert d[3, 0] >= 2.0 ** 18 and d[13, 9] >= 2.0 ** 18
    codes, scales = orc.repack_t2(src, N, K)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    for r in range(M):
        assert rel_rms(got[r], want[r]) <= TOL, (r, rel_rms(got[r], want[r]))


@pytest.mark.gpu
def test_gemv_mma_segments(cuda, btf, orc):
    # three segments sharing K and the activation (one launch each)
    import torch

    M, K = 16, 1024
    Ns = (300, 128, 77)
    x = synth.activations(M, K, seed=131)
    act = btf.quant_q8(_dev(x, cuda))
    q, d, s = orc.q8_rows(x)
    segs, srcs, ys = [], [], []
    for i, N in enumerate(Ns):
        src = synth.ternary_ptq(N, K, seed=132 + i)
        y = torch.zeros((M, N), device=cuda)
        segs.append((btf.repack_panels(_dev(src, cuda), N, K), y, N))
        srcs.append(src)
        ys.append(y)
    btf.launch_gemv_mma(segs, K, M, act, btf.STORE)
    torch.cuda.synchronize()
    for src, y, N in zip(srcs, ys, Ns):
        codes, scales = orc.repack_t2(src, N, K)
        assert rel_rms(y.cpu().numpy(), orc.gemv(codes, scales, K, q, d, s, threads=8)) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(3, 2 * 148 * 8 * 32), (8, 2 * 148 * 8 * 32), (16, 2 * 148 * 8 * 32),
                                 (6, 2 * 148 * 32), (12, 148 * 32), (16, 17408)])
def test_gemv_and_gemm_route_to_warp_mma(cuda, btf, orc, M, N):
    # btf_gemv and btf_gemm hand the warp-MMA kernel 9 <= M <= 16 rows over
    # (SM count) 32-row units or more, 5 <= M <= 8 over 2 x (SM count) units or
    # more, 3 <= M <= 4 over 8 x (SM count) units or more: bit for bit its
    # output, and within the bar of the oracle on a subset of rows
    import torch

    K = 1024
    src = synth.ternary_ptq(N, K, seed=190 + M)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=191 + M)
    act = btf.quant_q8(_dev(x, cuda))
    ys = [torch.full((M, N), 3.0, device=cuda) for _ in range(3)]
    btf.launch_gemv_mma([(pm, ys[0], N)], K, M, act, btf.STORE)
    btf.launch_gemv([(pm, ys[1], N)], K, M, act, btf.STORE)
    btf.launch_gemm([(pm, ys[2], N)], K, M, act, btf.STORE)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    a, b, c = (y.cpu().numpy() for y in ys)
    assert np.array_equal(a, b) and np.array_equal(a, c)
    rows = np.r_[0:min(200, N // 2), N - min(200, N // 2):N]
    codes, scales = orc.repack_t2(src[rows], len(rows), K)
    q, d, s = orc.q8_rows(x)
    assert rel_rms(a[:, rows], orc.gemv(codes, scales, K, q, d, s, threads=8)) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,mode", [(24, 0), (32, 1)])
def test_gemv_and_gemm_run_two_passes_of_16_rows(cuda, btf, orc, M, mode):
    # 17 <= M <= 32 rows over a matrix of 8 x (SM count) 32-row units or more:
    # btf_gemv and btf_gemm run two warp-MMA passes (rows 0..15, then the rest),
    # bit for bit those two direct calls, and within the bar of the oracle
    import torch

    K, N = 1024, 148 * 8 * 32
    src = synth.ternary_ptq(N, K, seed=300 + M)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=301 + M)
    act = btf.quant_q8(_dev(x, cuda))
    y0 = np.random.default_rng(M).standard_normal((M, N)).astype(np.float32)
    ys = [_dev(y0, cuda) for _ in range(3)]
    for m0 in (0, 16):
        mm = min(16, M - m0)
        sub = btf.Q8Act(act.q[m0:m0 + mm], act.d[m0:m0 + mm], act.s[m0:m0 + mm])
        btf.launch_gemv_mma([(pm, ys[0][m0:m0 + mm], N)], K, mm, sub, mode)
    btf.launch_gemv([(pm, ys[1], N)], K, M, act, mode)
    btf.launch_gemm([(pm, ys[2], N)], K, M, act, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    a, b, c = (y.cpu().numpy() for y in ys)
    assert np.array_equal(a, b) and np.array_equal(a, c)
    rows = np.r_[0:200, N - 200:N]
    codes, scales = orc.repack_t2(src[rows], len(rows), K)
    q, d, s = orc.q8_rows(x)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8) + (y0[:, rows] if mode == btf.ADD else 0)
    assert rel_rms(a[:, rows], want) <= TOL


def test_gemv_mma_rejects_bad_arguments(btf):
    """Refused before any CUDA call (runs without a GPU)."""
    import ctypes

    L = btf.lib()
    seg = (btf.GemvSeg * 1)()
    act = btf.Q8ActC(16, 16, 16)
    assert L.btf_gemv_mma(seg, 1, 1024, 17, act, btf.STORE, None) == 1  # M > 16
    assert "M <= 16" in L.btf_last_error().decode()
    assert L.btf_gemv_mma(seg, 1, 1000, 16, act, btf.STORE, None) == 1  # K % 128
    assert L.btf_gemv_mma(seg, 1, 8320, 16, act, btf.STORE, None) == 1  # K > 8192
    assert L.btf_gemv_mma(seg, 1, 1024, 16, act, btf.SWIGLU, None) == 1  # no SwiGLU mode
    assert L.btf_gemv_mma(seg, 1, 1024, 16, act, btf.STORE, None) == 1  # segment without panels
    assert "segment 0" in L.btf_last_error().decode()
    assert L.btf_gemv_mma(seg, 1, 1024, 0, act, btf.STORE, None) == 0  # nothing to do
    assert L.btf_gemv_mma_idot(None, 64, 1024, 16, act, ctypes.c_void_p(16), None) == 1
