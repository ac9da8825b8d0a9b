"""GPU parity of the weight-major small-batch GEMM (btf_gemm_wm) against the oracle.

The reference serves a batch of M rows as repeated launch_gemv passes
(src/cuda/kernels.cu:805-821) of the math the oracle restates
(src/emu_decoder.cpp:143-165). btf_gemm_wm computes the same outputs for
1 <= M <= 64 with the weights as the tensor core's 128-row operand. The bar is
the GEMM's: every 32-column integer accumulator equal to the oracle's idot, and
fp32 outputs within rel-RMS 1e-5 of the oracle. Shapes cover every padded
batch width (16, 32, 64), tiles with fewer than 128 rows, K whose block count
leaves the last tensor-memory slot partly empty, CTAs that walk several weight
tiles, add mode, activation scales of 2^18 and more, and the batch-16
lm_head and M = 64 prefill shapes on a subset of rows.
"""
import numpy as np
import pytest

import synth
from conftest import rel_rms

TOL = 1e-5


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _run(btf, cuda, src, x, M, K, N, mode, y0=None, scale_rows=None):
    import torch

    pm = btf.repack_panels(_dev(src, cuda), N, K)
    act = btf.quant_q8(_dev(x, cuda))
    if scale_rows is not None:  # raise some activation scales far above what the quantiser writes
        for r, blocks, f in scale_rows:
            act.d[r, blocks] *= f
    y = _dev(y0, cuda) if mode == btf.ADD else torch.full((M, N), 7.0, device=cuda)
    btf.launch_gemm_wm([(pm, y, N)], K, M, act, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    return y.cpu().numpy(), act


def _case(btf, orc, cuda, M, K, N, seed, mode=0, rows=None):
    src = synth.ternary_ptq(N, K, seed=seed)
    x = synth.activations(M, K, seed=seed + 1)
    y0 = np.random.default_rng(seed).standard_normal((M, N)).astype(np.float32)
    got, _ = _run(btf, cuda, src, x, M, K, N, mode, y0)
    q, d, s = orc.q8_rows(x)
    sel = slice(None) if rows is None else rows
    codes, scales = orc.repack_t2(src[sel], src[sel].shape[0], K)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    if mode == btf.ADD:
        want = want + y0[:, sel]
    g = got[:, sel]
    assert rel_rms(g, want) <= TOL, rel_rms(g, want)
    return got


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [
    (1, 1024, 64),     # one row, a tile of 64 weight rows
    (5, 1024, 200),    # padded to 16, a partial second tile
    (16, 5120, 300),   # the batch-16 width
    (17, 640, 130),    # padded to 32; 5 blocks: the last slot holds one of two
    (32, 2048, 256),
    (40, 1152, 72),    # padded to 64; a column group with no live rows
    (64, 5120, 200),
    (16, 384, 1000),   # 3 blocks: the last slot holds three of four
    (9, 17408, 136),   # the down projection's K
])
def test_gemm_wm_matches_oracle(cuda, btf, orc, M, K, N):
    _case(btf, orc, cuda, M, K, N, seed=M + K + N)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [3, 16, 24, 64])
def test_gemm_wm_add_mode(cuda, btf, orc, M):
    _case(btf, orc, cuda, M, 1024, 264, seed=50 + M, mode=btf.ADD)


@pytest.mark.gpu
def test_gemm_wm_persistent_tiles(cuda, btf, orc):
    # more 128-row tiles than SMs: every CTA walks two or three tiles and its
    # pipelines cross tile boundaries; rows from the first, middle and last tiles
    M, K = 16, 512
    N = 148 * 128 * 2 + 77
    rows = np.r_[0:256, N // 2 - 128:N // 2 + 128, N - 333:N]
    _case(btf, orc, cuda, M, K, N, seed=71, rows=rows)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,rows", [(16, 5120, 248320, 1024), (64, 5120, 17408, 512), (64, 17408, 5120, 256)])
def test_gemm_wm_benchmark_shapes(cuda, btf, orc, M, K, N, rows):
    # the batch-16 lm_head (configuration 4) and configuration 2's M = 64 prefill;
    # rows from the first, a middle and the last tiles so the CPU oracle stays quick
    sel = np.r_[0:rows // 2, N // 2:N // 2 + rows // 4, N - rows // 4:N]
    _case(btf, orc, cuda, M, K, N, seed=3, rows=sel)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(16, 1024, 200), (29, 640, 136), (64, 2048, 130), (7, 384, 64)])
def test_gemm_wm_integer_accumulators_bit_exact(cuda, btf, orc, M, K, N):
    # the kernel's dump form writes each 32-column step's int32 accumulator read
    # from tensor memory; every one must equal the oracle's idot
    # (src/emu_decoder.cpp:154-157)
    src = synth.ternary_ptq(N, K, seed=M)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=M + 1)
    act = btf.quant_q8(_dev(x, cuda))
    got = btf.gemm_wm_idot(pm, M, act).cpu().numpy()
    codes, _ = orc.repack_t2(src, N, K)
    q, d, s = orc.q8_rows(x)
    assert np.array_equal(got, orc.idot(codes, K, q, s))


@pytest.mark.gpu
def test_gemm_wm_matches_gemm_and_gemv(cuda, btf):
    # the same Q8 input through the weight-major GEMM, the 128-row GEMM and the
    # GEMV passes: all three agree
    import torch

    M, K, N = 64, 2048, 192
    src = synth.ternary_ptq(N, K, seed=9)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    act = btf.quant_q8(_dev(synth.activations(M, K, seed=10), cuda))
    ys = [torch.empty((M, N), device=cuda) for _ in range(3)]
    btf.launch_gemm_wm([(pm, ys[0], N)], K, M, act, btf.STORE)
    btf.launch_gemm([(pm, ys[1], N)], K, M, act, btf.STORE)
    for m0 in range(0, M, 8):  # 8-row GEMV passes on row views of the activation
        sub = btf.Q8Act(act.q[m0:m0 + 8], act.d[m0:m0 + 8], act.s[m0:m0 + 8])
        btf.launch_gemv([(pm, ys[2][m0:m0 + 8], N)], K, 8, sub, btf.STORE)
    torch.cuda.synchronize()
    a, b, c = (y.cpu().numpy() for y in ys)
    assert rel_rms(a, b) <= TOL and rel_rms(a, c) <= TOL


@pytest.mark.gpu
def test_gemm_wm_large_activation_scales(cuda, btf, orc):
    # scales of 2^18 and above (a caller's own Q8 data; the library's quantiser
    # writes fp16 values) beside ordinary ones: the epilogue multiplies by d
    # itself, so any finite d takes the same path; the oracle gets the same scales
    M, K, N = 24, 1024, 136
    src = synth.ternary_ptq(N, K, seed=81)
    x = synth.activations(M, K, seed=82)
    boost = [(3, slice(0, 4), np.float32(2.0 ** 26)), (17, slice(9, 11), np.float32(2.0 ** 34))]
    got, act = _run(btf, cuda, src, x, M, K, N, btf.STORE, scale_rows=boost)
    q, _, s = orc.q8_rows(x)
    d = act.d.cpu().numpy()
    assert d[3, 0] >= 2.0 ** 18 and d[17, 9] >= 2.0 ** 18
    codes, scales = orc.repack_t2(src, N, K)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    for r in range(M):
        assert rel_rms(got[r], want[r]) <= TOL, (r, rel_rms(got[r], want[r]))


def test_gemm_wm_rejects_bad_arguments(btf):
    """Refused before any CUDA call (runs without a GPU)."""
    import ctypes

    L = btf.lib()
    seg = (btf.GemvSeg * 1)()
    act = btf.Q8ActC(16, 16, 16)
    assert L.btf_gemm_wm(seg, 1, 1024, 65, act, btf.STORE, None) == 1  # M > 64
    assert "at most 64" in L.btf_last_error().decode()
    assert L.btf_gemm_wm(seg, 1, 1000, 16, act, btf.STORE, None) == 1  # K % 128
    assert L.btf_gemm_wm(seg, 1, 1024, 16, act, btf.SWIGLU, None) == 1  # no SwiGLU mode
    assert L.btf_gemm_wm(seg, 1, 1024, 16, act, btf.STORE, None) == 1  # segment without panels
    assert "segment 0" in L.btf_last_error().decode()
    assert L.btf_gemm_wm(seg, 1, 1024, 0, act, btf.STORE, None) == 0  # nothing to do
    assert L.btf_gemm_wm_idot(None, 64, 1024, 16, act, ctypes.c_void_p(16), None) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("M", [17, 24, 40, 64])
def test_gemv_and_gemm_route_small_batches_here(cuda, btf, orc, M):
    # btf_gemv and btf_gemm hand 17 <= M <= 64 rows (9..16 go to the warp-MMA
    # kernel) over a matrix with an SM's worth of 128-row tiles to the
    # weight-major kernel: bit for bit its output,
    # and within the bar of the oracle on a subset of rows
    import torch

    K, N = 1024, 148 * 128
    src = synth.ternary_ptq(N, K, seed=90 + M)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=91 + M)
    act = btf.quant_q8(_dev(x, cuda))
    ys = [torch.full((M, N), 3.0, device=cuda) for _ in range(3)]
    btf.launch_gemm_wm([(pm, ys[0], N)], K, M, act, btf.STORE)
    btf.launch_gemv([(pm, ys[1], N)], K, M, act, btf.STORE)
    btf.launch_gemm([(pm, ys[2], N)], K, M, act, btf.STORE)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    a, b, c = (y.cpu().numpy() for y in ys)
    assert np.array_equal(a, b) and np.array_equal(a, c)
    rows = np.r_[0:200, N - 200:N]
    codes, scales = orc.repack_t2(src[rows], len(rows), K)
    q, d, s = orc.q8_rows(x)
    assert rel_rms(a[:, rows], orc.gemv(codes, scales, K, q, d, s, threads=8)) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1])
def test_gemm_wm_segments_and_strided_output(cuda, btf, orc, mode):
    # three segments sharing K and the activation (one launch each), outputs with
    # ldy > N, in store and add mode
    import torch

    M, K = 24, 1024
    Ns = (300, 128, 77)
    x = synth.activations(M, K, seed=121 + mode)
    act = btf.quant_q8(_dev(x, cuda))
    q, d, s = orc.q8_rows(x)
    segs, srcs, ys, y0s = [], [], [], []
    for i, N in enumerate(Ns):
        src = synth.ternary_ptq(N, K, seed=122 + i)
        y0 = np.random.default_rng(i).standard_normal((M, N + 5)).astype(np.float32)
        y = _dev(y0, cuda)
        segs.append((btf.repack_panels(_dev(src, cuda), N, K), y, N + 5))
        srcs.append(src)
        ys.append(y)
        y0s.append(y0)
    btf.launch_gemm_wm(segs, K, M, act, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    for src, y, y0, N in zip(srcs, ys, y0s, Ns):
        got = y.cpu().numpy()
        codes, scales = orc.repack_t2(src, N, K)
        want = orc.gemv(codes, scales, K, q, d, s, threads=8) + (y0[:, :N] if mode == btf.ADD else 0)
        assert rel_rms(got[:, :N], want) <= TOL, rel_rms(got[:, :N], want)
        assert np.array_equal(got[:, N:], y0[:, N:])  # the columns past N are untouched
