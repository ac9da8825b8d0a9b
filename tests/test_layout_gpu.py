"""GPU tests of the load-time repack and the Q8 quantiser, through the C ABI.

Mirrors the reference's test_gpu_kernels.cpp test_repack (:74-97, mapped host
source, 0 mismatches) and test_prep's Q8 part (:100-161), tightened to
bit-exact since the raw-input quantiser has no WHT/norm rounding in front."""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("N,K", [(41, 1024), (37, 1152), (16, 128), (130, 5120), (17, 17408)])
def test_repack_panels_device_matches_host_twin(cuda, btf, orc, N, K):
    import oracle

    src = synth.ternary_ptq(N, K, seed=N * 7 + K)
    pm = btf.repack_panels(_dev(src, cuda), N, K)
    got = pm.panels.cpu().numpy()
    assert np.array_equal(got, btf.repack_panels_host(src, N, K))
    codes, scales = oracle.panel_decode(got, N, K)
    c_ref, s_ref = orc.repack_t2(src, N, K)
    assert np.array_equal(codes, c_ref) and np.array_equal(scales, s_ref)


def test_repack_from_mapped_host_memory(cuda, btf):
    # the reference's test_repack reads the PTQ1_0 source from mapped host
    # memory (cudaHostAlloc(cudaHostAllocMapped) + cudaHostGetDevicePointer,
    # tests/test_gpu_kernels.cpp:78-83); do the same through the runtime
    import ctypes

    import torch

    rt = ctypes.CDLL("libcudart.so.12")
    N, K = 41, 1024
    src = synth.ternary_ptq(N, K, seed=3)
    hptr, dptr = ctypes.c_void_p(), ctypes.c_void_p()
    assert rt.cudaHostAlloc(ctypes.byref(hptr), ctypes.c_size_t(src.nbytes), ctypes.c_uint(2)) == 0  # Mapped
    try:
        ctypes.memmove(hptr, src.ctypes.data, src.nbytes)
        assert rt.cudaHostGetDevicePointer(ctypes.byref(dptr), hptr, ctypes.c_uint(0)) == 0
        out = torch.empty(btf.panel_bytes(N, K), dtype=torch.uint8, device=cuda)
        btf.check(btf.lib().btf_repack_panels(dptr.value, N, K, out.data_ptr(), None), "repack")
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), btf.repack_panels_host(src, N, K))
    finally:
        rt.cudaFreeHost(hptr)


def test_repack_t2_and_roundtrip(cuda, btf, orc):
    import torch

    N, K = 37, 2048
    src = synth.ternary_ptq(N, K, seed=9)
    codes = torch.empty(N * K // 4, dtype=torch.uint8, device=cuda)
    scales = torch.empty(N * K // 128, dtype=torch.int16, device=cuda)
    btf.launch_repack(_dev(src, cuda), N * K // 128, codes, scales)
    c_ref, s_ref = orc.repack_t2(src, N, K)
    assert np.array_equal(codes.cpu().numpy().reshape(N, -1), c_ref)
    assert np.array_equal(scales.cpu().numpy().view(np.uint16).reshape(N, -1), s_ref)
    pm = btf.t2_to_panels(codes, scales, N, K)
    assert np.array_equal(pm.panels.cpu().numpy(), btf.repack_panels_host(src, N, K))
    c2, s2 = btf.panels_to_t2(pm)
    assert np.array_equal(c2.cpu().numpy().reshape(N, -1), c_ref)
    assert np.array_equal(s2.cpu().numpy().view(np.uint16).reshape(N, -1), s_ref)


@pytest.mark.parametrize("M,K", [(1, 1024), (3, 5120), (8, 2048), (2, 256), (1, 17408), (5, 6144)])
def test_quant_q8_bit_exact(cuda, btf, orc, M, K):
    rng = np.random.default_rng(M * 131 + K)
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    x[0, 64:96] = 0.0
    if K >= 256:
        x[-1, 128:160] = -0.0
        x[-1, 192:224] = 0.0
        x[-1, 223] = -0.0
        x[0, 160:192] = 1e-30  # tiny amax (127/amax still finite)
    act = btf.quant_q8(_dev(x, cuda))
    q, d, s = orc.q8_rows(x)
    assert np.array_equal(act.q.cpu().numpy(), q)
    assert act.d.cpu().numpy().tobytes() == d.tobytes()
    assert np.array_equal(act.s.cpu().numpy(), s)


def test_quant_q8_row_stride(cuda, btf, orc):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, 1024 + 96)).astype(np.float32)
    act = btf.quant_q8(_dev(x, cuda)[:, :1024])
    q, d, s = orc.q8_rows(x[:, :1024])
    assert np.array_equal(act.q.cpu().numpy(), q) and np.array_equal(act.s.cpu().numpy(), s)


def test_bad_arguments_raise(cuda, btf):
    import torch

    x = torch.zeros((1, 100), device=cuda)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        btf.quant_q8(x)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        btf.repack_panels(torch.zeros(28, dtype=torch.uint8, device=cuda), 1, 100)
