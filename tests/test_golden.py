"""Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py from
the reference's own compiled code) checked against the oracle, the host repack
twin and, with `-m gpu`, the CUDA path through the C ABI.

Bar: repack codes/scales, Q8 q/d/s and the int32 idot bit-exact; the oracle's
GEMV bit-exact (same loop order as the reference emulator); the GPU's fp32
outputs within rel-RMS 1e-5 (the reference's tolerance, tests/test_gpu_kernels.cpp
ref_gemv comparisons).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_rms

TOL = 1e-5
MANIFEST = json.load(open(os.path.join(GOLDEN, "MANIFEST.json")))
CASES = sorted(MANIFEST["cases"])


def _load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def _silu_mul(g, u):
    g = g.astype(np.float64)
    with np.errstate(over="ignore"):  # exp(-g) = inf for very negative g gives silu(g) = -0
        return g / (1.0 + np.exp(-g)) * u.astype(np.float64)


@pytest.mark.parametrize("name", CASES)
def test_fixture_checksums(name):
    meta = MANIFEST["cases"][name]
    digest = hashlib.sha256(open(os.path.join(GOLDEN, f"{name}.npz"), "rb").read()).hexdigest()
    assert digest == meta["sha256"]
    g = _load(name)
    assert (int(g["N"]), int(g["K"]), int(g["M"])) == (meta["N"], meta["K"], meta["M"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_reproduces_golden(orc, name):
    g = _load(name)
    N, K = int(g["N"]), int(g["K"])
    codes, scales = orc.repack_t2(g["src"], N, K)
    assert np.array_equal(codes, g["codes"]) and np.array_equal(scales, g["scales"])
    q, d, s = orc.q8_rows(g["x"])
    assert np.array_equal(q, g["q"]) and np.array_equal(d.view(np.uint32), g["d"].view(np.uint32))
    assert np.array_equal(s, g["s"])
    assert np.array_equal(orc.idot(codes, K, q, s), g["idot"])
    y = orc.gemv(codes, scales, K, q, d, s)
    assert np.array_equal(y.view(np.uint32), g["y_store"].view(np.uint32))
    ya = orc.gemv(codes, scales, K, q, d, s, y=g["y0"].copy(), add=True)
    assert np.array_equal(ya.view(np.uint32), g["y_add"].view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_host_repack_twin_matches_golden(btf, name):
    import oracle

    g = _load(name)
    N, K = int(g["N"]), int(g["K"])
    panels = btf.repack_panels_host(g["src"], N, K)
    codes, scales = oracle.panel_decode(panels, N, K)[:2]
    assert np.array_equal(codes[:N, :K // 4], g["codes"])
    assert np.array_equal(scales[:N, :K // 128], g["scales"])


def test_generator_is_deterministic(ref):
    import sys

    sys.path.insert(0, GOLDEN)
    import make_golden

    N, K, M, seed = make_golden.CASES["small"]
    fresh = make_golden.make_case(ref, N, K, M, seed)
    g = _load("small")
    for k, v in fresh.items():
        assert np.array_equal(np.asarray(v), g[k]), k


# ---------------------------------------------------------------- GPU (C ABI)
def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_gpu_repack_and_quant_bit_exact(cuda, btf, name):
    import oracle

    g = _load(name)
    N, K = int(g["N"]), int(g["K"])
    pm = btf.repack_panels(_dev(g["src"], cuda), N, K)
    codes, scales = btf.panels_to_t2(pm)
    assert np.array_equal(codes.cpu().numpy().reshape(N, K // 4), g["codes"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint16).reshape(N, K // 128), g["scales"])
    pc, ps = oracle.panel_decode(pm.panels.cpu().numpy(), N, K)[:2]
    assert np.array_equal(pc[:N, :K // 4], g["codes"]) and np.array_equal(ps[:N, :K // 128], g["scales"])
    act = btf.quant_q8(_dev(g["x"], cuda))
    assert np.array_equal(act.q.cpu().numpy(), g["q"])
    assert np.array_equal(act.d.cpu().numpy().view(np.uint32), g["d"].view(np.uint32))
    assert np.array_equal(act.s.cpu().numpy(), g["s"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_gpu_idot_and_gemv_match_golden(cuda, btf, name):
    import torch

    g = _load(name)
    N, K, M = int(g["N"]), int(g["K"]), int(g["M"])
    pm = btf.repack_panels(_dev(g["src"], cuda), N, K)
    up = btf.repack_panels(_dev(g["up_src"], cuda), N, K)
    act = btf.Q8Act(_dev(g["q"], cuda), _dev(g["d"], cuda), _dev(g["s"], cuda))
    assert np.array_equal(btf.gemv_idot(pm, M, act).cpu().numpy(), g["idot"])
    y = torch.full((M, N), 3.0, device=cuda)
    btf.launch_gemv([(pm, y, N)], K, M, act, btf.STORE)
    ya = _dev(g["y0"], cuda)
    btf.launch_gemv([(pm, ya, N)], K, M, act, btf.ADD)
    ys = torch.empty((M, N), device=cuda)
    btf.launch_gemv([(pm, ys, N), (up, None, 0)], K, M, act, btf.SWIGLU)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    assert rel_rms(y.cpu().numpy(), g["y_store"]) <= TOL
    assert rel_rms(ya.cpu().numpy(), g["y_add"]) <= TOL
    assert rel_rms(ys.cpu().numpy(), _silu_mul(g["y_store"], g["up_y"])) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_gpu_gemm_matches_golden(cuda, btf, name):
    import torch

    g = _load(name)
    N, K, M = int(g["N"]), int(g["K"]), int(g["M"])
    pm = btf.repack_panels(_dev(g["src"], cuda), N, K)
    act = btf.Q8Act(_dev(g["q"], cuda), _dev(g["d"], cuda), _dev(g["s"], cuda))
    y = torch.full((M, N), 3.0, device=cuda)
    btf.launch_gemm([(pm, y, N)], K, M, act, btf.STORE)
    ya = _dev(g["y0"], cuda)
    btf.launch_gemm([(pm, ya, N)], K, M, act, btf.ADD)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    assert rel_rms(y.cpu().numpy(), g["y_store"]) <= TOL
    assert rel_rms(ya.cpu().numpy(), g["y_add"]) <= TOL
