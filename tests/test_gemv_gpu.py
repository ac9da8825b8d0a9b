"""GPU parity of the ternary GEMV against the oracle, through the C ABI.

Follows the reference's test_gemv (tests/test_gpu_kernels.cpp:203-276): random
q in [-127, 127], d in U(0.001, 0.05), s = sum(q); three segments N = {37, 64, 9}
stored with ldy = N + 3; add and swiglu modes; shapes K=1024 M in {1,3,8,13},
K=5120 M=1, K=17408 M=2 (:562-564). The bar, written in each test:
  * idot (per row, sub-block, activation row) bit-exact;
  * fp32 y within rel-RMS 1e-5 of the oracle (and of the double reference),
    the reference's tolerance, plus a per-element bound
    |y - y64| <= 1e-5 * sum |terms| + 1e-30 so near-zero outputs are judged fairly.
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


class Mat:
    def __init__(self, btf, orc, N, K, seed, device):
        self.N, self.K = N, K
        self.src = synth.ternary_ptq(N, K, seed=seed)
        self.codes, self.scales = orc.repack_t2(self.src, N, K)
        self.pm = btf.repack_panels(_dev(self.src, device), N, K)


def _random_act(M, K, rng):
    q = rng.integers(-127, 128, size=(M, K)).astype(np.int8)
    d = rng.uniform(0.001, 0.05, size=(M, K // 32)).astype(np.float32)
    s = q.reshape(M, -1, 32).astype(np.int32).sum(-1).astype(np.int32)
    return q, d, s


def _act_dev(btf, q, d, s, device):
    return btf.Q8Act(_dev(q, device), _dev(d, device), _dev(s, device))


def _abs_terms(orc, mat, q, d, s):
    idot = orc.idot(mat.codes, mat.K, q, s).astype(np.float64)  # [M][N][K/32]
    sc = np.array([orc.L.orc_f16_to_f32(int(v)) for v in mat.scales.reshape(-1)], dtype=np.float64)
    sc = np.repeat(sc.reshape(mat.N, -1), 4, axis=1)  # per sub-block
    return np.abs(idot * sc[None] * d.astype(np.float64)[:, None, :]).sum(-1)


def _check(y, y_orc, y64, bound, label):
    assert rel_rms(y, y_orc) <= TOL, (label, rel_rms(y, y_orc))
    assert rel_rms(y, y64) <= TOL, (label, rel_rms(y, y64))
    err = np.abs(y.astype(np.float64) - y64)
    assert np.all(err <= TOL * bound + 1e-30), (label, float((err - TOL * bound).max()))


@pytest.mark.parametrize("K,M", [(1024, 1), (1024, 3), (1024, 8), (1024, 13), (5120, 1), (17408, 2)])
def test_gemv_segments_store_add_swiglu(cuda, btf, orc, K, M):
    import torch

    rng = np.random.default_rng(K * 17 + M)
    q, d, s = _random_act(M, K, rng)
    act = _act_dev(btf, q, d, s, cuda)
    Ns = [37, 64, 9]
    mats = [Mat(btf, orc, n, K, seed=100 + i + K, device=cuda) for i, n in enumerate(Ns)]
    ys = [torch.full((M, n + 3), 7.0, device=cuda) for n in Ns]  # ldy = N + 3
    btf.launch_gemv([(m.pm, y, m.N + 3) for m, y in zip(mats, ys)], K, M, act, btf.STORE)
    for i, (m, y) in enumerate(zip(mats, ys)):
        g = y.cpu().numpy()
        assert np.all(g[:, m.N:] == 7.0), "wrote past N"
        y_orc = orc.gemv(m.codes, m.scales, K, q, d, s)
        y64 = orc.gemv_f64(m.codes, m.scales, K, q, d)
        _check(g[:, :m.N], y_orc, y64, _abs_terms(orc, m, q, d, s), f"store seg{i}")
    # add: y = y0 + W x
    y0 = rng.standard_normal((M, Ns[0])).astype(np.float32)
    ya = _dev(y0, cuda)
    btf.launch_gemv([(mats[0].pm, ya, Ns[0])], K, M, act, btf.ADD)
    y64 = orc.gemv_f64(mats[0].codes, mats[0].scales, K, q, d) + y0
    y_orc = orc.gemv(mats[0].codes, mats[0].scales, K, q, d, s, y=y0.copy(), add=True)
    bound = _abs_terms(orc, mats[0], q, d, s) + np.abs(y0)
    _check(ya.cpu().numpy(), y_orc, y64, bound, "add")
    # swiglu: gate = segment 1, up = a fresh N=64 matrix
    up = Mat(btf, orc, Ns[1], K, seed=999 + K, device=cuda)
    yg = torch.zeros((M, Ns[1]), device=cuda)
    btf.launch_gemv([(mats[1].pm, yg, Ns[1]), (up.pm, None, 0)], K, M, act, btf.SWIGLU)
    g64 = orc.gemv_f64(mats[1].codes, mats[1].scales, K, q, d)
    u64 = orc.gemv_f64(up.codes, up.scales, K, q, d)
    want = g64 / (1 + np.exp(-g64)) * u64
    y_orc = orc.gemv_swiglu((mats[1].codes, mats[1].scales), (up.codes, up.scales), K, q, d, s)
    got = yg.cpu().numpy()
    assert rel_rms(got, want) <= TOL and rel_rms(got, y_orc) <= TOL


@pytest.mark.parametrize("N,K,M", [(37, 1024, 1), (64, 1024, 3), (9, 5120, 2), (33, 17408, 1), (16, 1152, 2)])
def test_idot_bit_exact(cuda, btf, orc, N, K, M):
    rng = np.random.default_rng(N + K + M)
    q, d, s = _random_act(M, K, rng)
    mat = Mat(btf, orc, N, K, seed=N * K, device=cuda)
    got = btf.gemv_idot(mat.pm, M, _act_dev(btf, q, d, s, cuda)).cpu().numpy()
    assert np.array_equal(got, orc.idot(mat.codes, K, q, s))


@pytest.mark.parametrize("name,K,N", [s for s in synth.LAYER_SHAPES])
def test_config1_shapes_quantised_end_to_end(cuda, btf, orc, name, K, N):
    # seeded weights/activations of the benchmark configurations; activation
    # quantised on the device, then the GEMV; compared with the oracle path
    mat = Mat(btf, orc, N, K, seed=0, device=cuda)
    x = synth.activations(1, K, seed=2)
    act = btf.quant_q8(_dev(x, cuda))
    q, d, s = orc.q8_rows(x)
    assert np.array_equal(act.q.cpu().numpy(), q)
    import torch

    y = torch.empty((1, N), device=cuda)
    btf.launch_gemv([(mat.pm, y, N)], K, 1, act, btf.STORE)
    y_orc = orc.gemv(mat.codes, mat.scales, K, q, d, s, threads=8)
    y64 = orc.gemv_f64(mat.codes, mat.scales, K, q, d) if N * K <= 6144 * 5120 else None
    g = y.cpu().numpy()
    assert rel_rms(g, y_orc) <= TOL, name
    if y64 is not None:
        assert rel_rms(g, y64) <= TOL, name
    # integer partials of the first rows are exact
    rows = slice(0, 48)
    idot_gpu = btf.gemv_idot(mat.pm, 1, act).cpu().numpy()[:, rows]
    assert np.array_equal(idot_gpu, orc.idot(mat.codes[rows], K, q, s))


@pytest.mark.parametrize("K,M,mode", [(5120, 1, 0), (6144, 2, 1), (17408, 1, 0), (1152, 3, 2), (5120, 4, 2),
                                      (2048, 9, 1)])
def test_fused_quantise_gemv_equals_two_step(cuda, btf, orc, K, M, mode):
    # btf_gemv_f32 quantises inside the GEMV with the same bit-exact rule:
    # its output must equal quantiser + GEMV bit for bit, and match the oracle
    import torch

    x = _dev(synth.activations(M, K, seed=K + M), cuda)
    a = Mat(btf, orc, 45, K, seed=K, device=cuda)
    b = Mat(btf, orc, 45, K, seed=K + 1, device=cuda)
    segs2 = [(a.pm, None, 0), (b.pm, None, 0)]
    y1 = torch.randn((M, 45), device=cuda)
    y2 = y1.clone()
    if mode == btf.SWIGLU:
        segs_a, segs_b = [(a.pm, y1, 45), segs2[1]], [(a.pm, y2, 45), segs2[1]]
    else:
        segs_a, segs_b = [(a.pm, y1, 45)], [(a.pm, y2, 45)]
    act = btf.quant_q8(x)
    btf.launch_gemv(segs_a, K, M, act, mode)
    btf.launch_gemv_f32(segs_b, K, M, x, mode)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    q, d, s = orc.q8_rows(x.cpu().numpy())
    if mode == btf.STORE:
        assert rel_rms(y2.cpu().numpy(), orc.gemv(a.codes, a.scales, K, q, d, s)) <= TOL
    assert btf.device_error() == 0


def test_gemv_in_cuda_graph_matches_eager(cuda, btf, orc):
    # the reference captures the whole decode step in one CUDA graph
    # (src/cuda/gpu_decoder.cu:459-486); graph replay must equal eager bit for bit
    import torch

    K, N = 5120, 1024
    mat = Mat(btf, orc, N, K, seed=4, device=cuda)
    x = _dev(synth.activations(1, K, seed=5), cuda)
    act = btf.Q8Act.empty(1, K, cuda)
    y_e = torch.empty((1, N), device=cuda)
    y_g = torch.empty((1, N), device=cuda)
    btf.quant_q8(x, act)
    btf.launch_gemv([(mat.pm, y_e, N)], K, 1, act)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        btf.quant_q8(x, act, stream=s)
        btf.launch_gemv([(mat.pm, y_g, N)], K, 1, act, stream=s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_e, y_g)


def test_gemv_rejects_bad_arguments(cuda, btf):
    import torch

    act = btf.Q8Act.empty(1, 1024, cuda)
    pm = btf.PanelMatrix(torch.zeros(btf.panel_bytes(16, 1024), dtype=torch.uint8, device=cuda), 16, 1024)
    y = torch.zeros((1, 16), device=cuda)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        btf.launch_gemv([(pm, y, 16)], 1000, 1, act)
    with pytest.raises(RuntimeError, match="swiglu"):
        btf.launch_gemv([(pm, y, 16)], 1024, 1, act, btf.SWIGLU)
    with pytest.raises(RuntimeError, match="segments"):
        btf.launch_gemv([(pm, y, 16)] * 4, 1024, 1, act)


@pytest.mark.parametrize("M", [1, 16])
def test_lm_head_shape_row_subsets(cuda, btf, orc, M):
    # benchmark configuration 4's lm_head, 5120 -> 248320 (31040 row groups; M=16 runs as
    # four 4-row passes), checked on rows from the first, a middle and the last row groups
    import torch

    N, K = synth.LM_HEAD[2], synth.LM_HEAD[1]
    # random digit bytes are valid PTQ1_0 (every byte decodes to trits, types.hpp:70-78);
    # bytes 26-27 of each block get a proper fp16 scale
    rng = np.random.default_rng(5)
    src = rng.integers(0, 256, size=(N, K // 128, 28), dtype=np.uint8)
    src[:, :, 26:28] = synth.block_scales(N, K, seed=6).view(np.uint8).reshape(N, K // 128, 2)
    src = src.reshape(N, K // 128 * 28)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=6)
    act = btf.quant_q8(_dev(x, cuda))
    y = torch.empty((M, N), device=cuda)
    btf.launch_gemv([(pm, y, N)], K, M, act, btf.STORE)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    rows = np.r_[0:64, N // 2 - 32:N // 2 + 32, N - 64:N]
    codes, scales = orc.repack_t2(src[rows], len(rows), K)
    q, d, s = orc.q8_rows(x)
    want = orc.gemv(codes, scales, K, q, d, s, threads=8)
    assert rel_rms(y.cpu().numpy()[:, rows], want) <= TOL


@pytest.mark.parametrize("M,mode", [(64, 0), (96, 1)])
def test_gemv_prefill_batch_runs_on_the_gemm(cuda, btf, orc, M, mode):
    # launch_gemv with a prefill batch (M >= 64, store / add) is the tcgen05 GEMM:
    # bit for bit btf_gemm's output, and within the GEMV bar of the oracle
    import torch

    K = 2048
    rng = np.random.default_rng(M + mode)
    q, d, s = _random_act(M, K, rng)
    act = _act_dev(btf, q, d, s, cuda)
    mats = [Mat(btf, orc, n, K, seed=500 + n, device=cuda) for n in (72, 40)]
    y0 = [rng.standard_normal((M, m.N)).astype(np.float32) for m in mats]
    yv = [_dev(y, cuda) for y in y0]
    yg = [_dev(y, cuda) for y in y0]
    btf.launch_gemv([(m.pm, y, m.N) for m, y in zip(mats, yv)], K, M, act, mode)
    btf.launch_gemm([(m.pm, y, m.N) for m, y in zip(mats, yg)], K, M, act, mode)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    for m, a, b, y_init in zip(mats, yv, yg, y0):
        a, b = a.cpu().numpy(), b.cpu().numpy()
        assert np.array_equal(a, b)
        add = mode == btf.ADD
        y_orc = orc.gemv(m.codes, m.scales, K, q, d, s, y=y_init.copy() if add else None, add=add)
        y64 = orc.gemv_f64(m.codes, m.scales, K, q, d) + (y_init if add else 0)
        _check(a, y_orc, y64, _abs_terms(orc, m, q, d, s) + (np.abs(y_init) if add else 0), f"M={M}")


@pytest.mark.parametrize("M,K,N", [(1, 5120, 17408), (4, 17408, 5120), (3, 1152, 44)])
def test_gemv_kernel_integer_dots_bit_exact(cuda, btf, orc, M, K, N):
    # btf_gemv_idot runs the shipped GEMV kernel in its dump form: every
    # (m, row, sub-block) value is the fp32 operand its epilogue multiplies
    # ((float) of the biased dp4a integer), written as int32. Configuration 0's
    # full 5120 -> 17408 matrix, a 4-row pass at K = 17408 and a ragged case.
    src = synth.ternary_ptq(N, K, seed=0)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    x = synth.activations(M, K, seed=2)
    act = btf.quant_q8(_dev(x, cuda))
    got = btf.gemv_idot(pm, M, act).cpu().numpy()
    codes, _ = orc.repack_t2(src, N, K)
    q, d, s = orc.q8_rows(x)
    assert np.array_equal(got, orc.idot(codes, K, q, s))
