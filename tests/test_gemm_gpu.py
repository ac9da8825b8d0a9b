"""GPU parity of the tcgen05 prefill GEMM (btf_gemm) against the oracle.

The reference has no GEMM: prefill runs as repeated 8-row GEMV passes
(src/cuda/kernels.cu:805-821), whose math the oracle restates
(src/emu_decoder.cpp:143-165). The bar is the GEMV's: exact int32 partials
(the MMA computes each 32-column idot exactly in int32) and fp32 outputs within
rel-RMS 1e-5 of the oracle and of the double reference. Shapes cover partial M
and N tiles, add mode, and the benchmark's prefill configurations (M = 64 and
512 with K=5120 -> N=17408 and K=17408 -> N=5120), the latter checked on a
subset of output rows so the CPU oracle stays quick.
"""
import numpy as np
import pytest

import synth
from conftest import rel_rms

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _case(btf, orc, cuda, M, K, N, seed, mode=0, rows=None):
    import torch

    src = synth.ternary_ptq(N, K, seed=seed)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=seed + 1)
    act = btf.quant_q8(_dev(x, cuda))
    y0 = np.random.default_rng(seed).standard_normal((M, N)).astype(np.float32)
    y = _dev(y0, cuda) if mode == btf.ADD else torch.full((M, N), 7.0, device=cuda)
    btf.launch_gemm([(pm, y, N)], K, M, act, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    got = y.cpu().numpy()
    q, d, s = orc.q8_rows(x)
    sel = slice(None) if rows is None else rows
    codes, scales = orc.repack_t2(src[sel], src[sel].shape[0], K)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    want64 = orc.gemv_f64(codes, scales, K, q, d) if rows is None and N * K * M <= 64 * 5120 * 260 else None
    g = got[:, sel]
    if mode == btf.ADD:
        want = want + y0[:, sel]
        if want64 is not None:
            want64 = want64 + y0[:, sel]
    assert rel_rms(g, want) <= TOL, rel_rms(g, want)
    if want64 is not None:
        assert rel_rms(g, want64) <= TOL
    return got


@pytest.mark.parametrize("M,K,N", [(64, 1024, 64), (128, 1024, 37), (130, 2048, 130), (64, 5120, 200),
                                   (200, 1152, 72)])
def test_gemm_matches_oracle(cuda, btf, orc, M, K, N):
    _case(btf, orc, cuda, M, K, N, seed=M + K + N)


def test_gemm_add_mode(cuda, btf, orc):
    _case(btf, orc, cuda, 96, 1024, 80, seed=5, mode=btf.ADD)


def test_gemm_equals_gemv_passes(cuda, btf, orc):
    # same Q8 input through both paths: the GEMM and the 4-row GEMV passes agree
    import torch

    M, K, N = 64, 2048, 96
    src = synth.ternary_ptq(N, K, seed=9)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    act = btf.quant_q8(_dev(synth.activations(M, K, seed=10), cuda))
    y1 = torch.empty((M, N), device=cuda)
    y2 = torch.empty((M, N), device=cuda)
    btf.launch_gemm([(pm, y1, N)], K, M, act, btf.STORE)
    btf.launch_gemv([(pm, y2, N)], K, M, act, btf.STORE)
    torch.cuda.synchronize()
    assert rel_rms(y1.cpu().numpy(), y2.cpu().numpy()) <= TOL


@pytest.mark.parametrize("M,K,N", [(64, 5120, 17408), (512, 5120, 17408), (64, 17408, 5120), (512, 17408, 5120)])
def test_gemm_prefill_configs(cuda, btf, orc, M, K, N):
    # benchmark configuration 2 shapes; rows from the first, a middle and the last N tile
    rows = np.r_[0:64, N // 2 - 32:N // 2 + 32, N - 64:N]
    _case(btf, orc, cuda, M, K, N, seed=0, rows=rows)


def test_gemm_three_segments_qkv_shapes(cuda, btf, orc):
    # q/k/v in one call (3 segments sharing K and the activation), prefill M=64
    import torch

    K, M = 5120, 64
    Ns = (6144, 1024, 1024)
    x = synth.activations(M, K, seed=41)
    act = btf.quant_q8(_dev(x, cuda))
    q, d, s = orc.q8_rows(x)
    segs, srcs, ys = [], [], []
    for i, N in enumerate(Ns):
        src = synth.ternary_ptq(N, K, seed=42 + i)
        y = torch.empty((M, N + 3), device=cuda)  # ldy > N
        segs.append((btf.repack_panels(_dev(src, cuda), N, K), y, N + 3))
        srcs.append(src)
        ys.append(y)
    btf.launch_gemm(segs, K, M, act, btf.STORE)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    for src, y, N in zip(srcs, ys, Ns):
        rows = np.r_[0:32, N - 32:N]
        codes, scales = orc.repack_t2(src[rows], len(rows), K)
        want = orc.gemv(codes, scales, K, q, d, s, threads=8)
        assert rel_rms(y.cpu().numpy()[:, :N][:, rows], want) <= TOL


def test_gemm_extreme_activation_scales(cuda, btf, orc):
    # rows whose Q8 scale d = fp16(amax/127) is near the fp16 maximum, a
    # subnormal fp16 value, or zero, beside ordinary rows; each row is checked
    # on its own since the rows differ by 12 orders of magnitude
    import torch

    M, K, N = 96, 2048, 136
    src = synth.ternary_ptq(N, K, seed=61)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=62)
    x[3] *= np.float32(2e6)
    x[5] *= np.float32(1e-5)
    x[7] = 0.0
    x[70, 256:512] *= np.float32(2e6)  # two 128-column blocks of row 70
    act = btf.quant_q8(_dev(x, cuda))
    y = torch.full((M, N), 7.0, device=cuda)
    btf.launch_gemm([(pm, y, N)], K, M, act, btf.STORE)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    got = y.cpu().numpy()
    q, d, s = orc.q8_rows(x)
    assert 2.0 ** 14 < d[3].max() < 65504 and 0 < d[5].max() < 2.0 ** -14
    codes, scales = orc.repack_t2(src, N, K)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    assert np.all(got[7] == 0.0)
    for r in range(M):
        if r != 7:
            assert rel_rms(got[r], want[r]) <= TOL, (r, rel_rms(got[r], want[r]))


@pytest.mark.parametrize("M,K,N,rows", [(64, 5120, 17408, 2048), (64, 17408, 5120, 640), (77, 1152, 200, 200)])
def test_gemm_integer_accumulators_bit_exact(cuda, btf, orc, M, K, N, rows):
    # the GEMM kernel itself (its dump form, btf_gemm_idot) writes each 32-column
    # region's int32 accumulator from tensor memory; every one must equal the
    # oracle's idot (the integer of src/emu_decoder.cpp:154-157). Configuration
    # 2's shapes on their first `rows` weight rows (the oracle stays quick).
    src = synth.ternary_ptq(N, K, seed=0)[:rows]
    pm = btf.repack_panels(_dev(src, cuda), rows, K)
    x = synth.activations(M, K, seed=2)
    act = btf.quant_q8(_dev(x, cuda))
    got = btf.gemm_idot(pm, M, act).cpu().numpy()
    codes, _ = orc.repack_t2(src, rows, K)
    q, d, s = orc.q8_rows(x)
    assert np.array_equal(got, orc.idot(codes, K, q, s))
