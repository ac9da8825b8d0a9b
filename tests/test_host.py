"""CPU tests of the product library's host side: exports, layout sizes, the
host repack twin, argument checking. No kernel is launched here."""
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, PKG


def _declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "btf_b200.h")).read()
    return sorted(set(re.findall(r"\b(btf_[a-z0-9_]+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol(btf):
    names = _declared_symbols()
    assert len(names) >= 15
    L = btf.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(btf.EXPORTS) == set(names)
    out = subprocess.run(["nm", "-D", "--defined-only", btf.LIB_PATH], capture_output=True, text=True).stdout
    for n in names:
        assert re.search(rf"\bT {n}$", out, re.M), n


def test_layout_sizes(btf):
    assert btf.panel_bytes(17408, 5120) == 17408 * 5120 // 4 + 17408 * 40 * 2  # no padding at the config-0 shape
    assert btf.panel_bytes(37, 1024) == 5 * 1 * 2176
    assert btf.panel_bytes(16, 1152) == 2 * 2 * 2176
    assert btf.t2_codes_bytes(37, 1024) == 37 * 256
    assert btf.t2_scales_bytes(37, 1024) == 37 * 8 * 2
    assert btf.gemv_max_nb(5120) == 4 and btf.gemv_max_nb(100) == 0


@pytest.mark.parametrize("N,K,random_bytes,threads", [(37, 1024, 0, 3), (41, 1152, 0, 3), (16, 128, 0, 3),
                                                      (1, 5120, 0, 3), (33, 3072, 0, 3), (41, 1152, 1, 1),
                                                      (300, 1280, 1, 4)])
def test_host_repack_matches_reference_t2(btf, orc, N, K, random_bytes, threads):
    import oracle
    import synth

    src = synth.ternary_ptq(N, K, seed=N + K)
    if random_bytes:  # every byte value decodes to five digits, 243..255 included
        src = np.random.default_rng(N * K).integers(0, 256, size=src.shape, dtype=np.uint8)
    pan = btf.repack_panels_host(src, N, K, threads=threads)
    assert pan.size == btf.panel_bytes(N, K)
    codes, scales = oracle.panel_decode(pan, N, K)
    c_ref, s_ref = orc.repack_t2(src, N, K)
    assert np.array_equal(codes, c_ref) and np.array_equal(scales, s_ref)
    # padding: rows >= N and columns >= K hold code 1 (trit 0) and scale 0
    G, S = (N + 7) // 8, (K + 1023) // 1024
    full_codes, full_scales = oracle.panel_decode(pan, G * 8, S * 1024)
    assert np.all(full_codes[N:] == 0x55) and np.all(full_codes[:, K // 4:] == 0x55)
    assert np.all(full_scales[N:] == 0) and np.all(full_scales[:, K // 128:] == 0)


def test_host_repack_rejects_bad_shape(btf):
    src = np.zeros(28, dtype=np.uint8)
    with pytest.raises(RuntimeError, match="invalid argument"):
        btf.repack_panels_host(src, 1, 100)


def test_init_without_gpu_reports_error(btf):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc = btf.lib().btf_init(0)
    assert rc != 0
    assert btf.lib().btf_last_error().decode()


def test_cpp_shim_header_compiles():
    # the C++17 mirror of the reference launchers (include/btf_b200.hpp) must
    # compile as a drop-in for src/cuda/kernels.cuh call sites
    src = os.path.join(ROOT, "tests", "shim_compile.cpp")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                        "-I", "/usr/local/cuda/include", src], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def _seg(btf, ptr=16, N=8, y=64, ldy=8):
    arr = (btf.GemvSeg * 1)()
    arr[0] = btf.GemvSeg(ptr, N, y, ldy)
    return arr


def test_gather_entry_points_reject_bad_arguments(btf):
    # argument checks run before any device access, so they are testable without a GPU
    import ctypes

    L = btf.lib()
    act = btf.Q8ActC(256, 256, 256)
    g = btf.GatherC()
    g.world, g.rank = 1, 0  # world must be >= 2
    rc = L.btf_gemv_gather(_seg(btf), 1, 1024, 1, act, btf.STORE, ctypes.byref(g), None)
    assert rc == 1 and "world" in L.btf_last_error().decode()
    g.world, g.rank = 2, 0
    g.tagged, g.site = 1, 2000  # site >= 1024
    rc = L.btf_gemv_gather(_seg(btf), 1, 1024, 1, act, btf.STORE, ctypes.byref(g), None)
    assert rc == 1 and "site" in L.btf_last_error().decode()
    g.site, g.epoch = 3, 4096
    rc = L.btf_gemv_gather(_seg(btf), 1, 1024, 1, act, btf.STORE, ctypes.byref(g), None)
    assert rc == 1 and "peer_y" in L.btf_last_error().decode()  # peer pointers not set
    rc = L.btf_gemv_gather(_seg(btf), 1, 1000, 1, act, btf.STORE, ctypes.byref(g), None)
    assert rc == 1 and "multiple of 128" in L.btf_last_error().decode()
    bufs = (btf.TaggedBufC * 1)()
    assert L.btf_gather_wait(bufs, 0, 4096, None) == 1
    bufs[0] = btf.TaggedBufC(0, 10, 1)
    assert L.btf_gather_wait(bufs, 1, 4096, None) == 1  # null buffer
    assert L.btf_gather_epoch_advance(None, None) == 1
    assert L.btf_gather_barrier(ctypes.byref(btf.GatherC()), None) == 1
    assert L.btf_alloc(0, ctypes.byref(ctypes.c_void_p())) == 1
    assert L.btf_ipc_handle(None, ctypes.create_string_buffer(64)) == 1


def test_decoder_entry_points_reject_bad_arguments(btf):
    # argument checks run before any device access, so they are testable without a GPU
    import ctypes

    L = btf.lib()
    h = ctypes.c_void_p()
    assert L.btf_decoder_open(None, None, ctypes.byref(h)) == 1
    dims = btf.DecoderDimsC(*([4, 256, 512, 300, 3, 2, 128, 32, 32, 2, 4, 0, 4, 128]), 1e7, 1e-6)  # 3 % 2 heads
    assert L.btf_decoder_synthetic(ctypes.byref(dims), 1, None, ctypes.byref(h)) == 1
    assert "dims" in L.btf_last_error().decode()
    dims.n_head = 4
    assert L.btf_decoder_synthetic_tp(ctypes.byref(dims), 1, None, 9, 0, ctypes.byref(h)) == 1  # world > 8
    assert L.btf_decoder_synthetic_tp(ctypes.byref(dims), 1, None, 2, 2, ctypes.byref(h)) == 1  # rank >= world
    dims.hadamard_block = 96  # not a power of two
    assert L.btf_decoder_synthetic(ctypes.byref(dims), 1, None, ctypes.byref(h)) == 1
    nxt = ctypes.c_int32()
    assert L.btf_decoder_step(None, 1, None, ctypes.byref(nxt)) == 1
    assert L.btf_decoder_run(None, 1) == 1
    assert L.btf_decoder_connect(None, None) == 1
    info = btf.DecoderInfoC()
    assert L.btf_decoder_get_info(None, ctypes.byref(info)) == 1


def test_decoder_stats_reject_null_handles(btf):
    import ctypes

    L = btf.lib()
    s = btf.StepStatsC()
    assert L.btf_decoder_stats(None, ctypes.byref(s)) == 1
    assert L.btf_decoder_reset_stats(None) == 1


def test_cpp_shim_host_repack_equals_the_c_abi(btf, tmp_path):
    # btf::cuda::repack_panels_host (include/btf_b200.hpp) linked against the library, no GPU
    import synth

    exe = str(tmp_path / "shim_repack")
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                        os.path.join(ROOT, "tests", "shim_repack.cpp"), "-o", exe, "-L", PKG, "-lbtf_b200",
                        f"-Wl,-rpath,{PKG}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    N, K = 41, 1152
    src = synth.ternary_ptq(N, K, seed=5)
    (tmp_path / "src.bin").write_bytes(src.tobytes())
    r = subprocess.run([exe, str(N), str(K), str(tmp_path / "src.bin"), str(tmp_path / "pan.bin")],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    got = np.frombuffer((tmp_path / "pan.bin").read_bytes(), dtype=np.uint8)
    assert np.array_equal(got, btf.repack_panels_host(src, N, K, threads=1))
