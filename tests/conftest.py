"""Shared test set-up: import paths, the `gpu` marker, oracle fixtures.

Test layout mirrors the reference's CTest split (CMakeLists.txt:68-96 of the
reference): CPU tests pin the oracle and the host logic; `-m gpu` tests run the
CUDA kernels through the C ABI against the oracle.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "bonsai-ternary-fast_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# the reference's decoder-test prompt (tests/test_common.hpp:67-70)
DECODER_PROMPT = [259, 272, 44, 32, 259, 261, 103, 97, 264]

# synthetic qwen35 models (bd::make_synth_qwen35 options over the defaults):
# the Hadamard variants the binding distinguishes, f32 alpha/beta, and the real
# model's head geometry (head_dim 256, d_state 128, block 1024)
DECODER_CONFIGS = {
    "default (block 64)": dict(),
    "identity signs": dict(explicit_signs=0),
    "no hadamard": dict(hadamard=0),
    "gdn v tiled": dict(gdn_v_grouped=0),
    "f32 alpha/beta": dict(small_mat_type=0),
    "real head geometry": dict(n_layer=4, n_embd=1024, n_ff=2048, n_head=4, n_head_kv=1, head_dim=256, n_rot=64,
                               d_state=128, n_group=2, dt_rank=8, hadamard_block=1024),
}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    import oracle

    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle

    if not oracle.Reference.available():
        pytest.skip("oracle/_ref/libbtf_ref.so not built (reference tree absent)")
    return oracle.Reference()


@pytest.fixture(scope="session")
def btf():
    import btf_b200

    btf_b200.lib()
    return btf_b200


@pytest.fixture(scope="session")
def cuda(btf):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    btf.kernels_init(0)
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def rel_rms(a, ref):
    """sqrt(sum (a-ref)^2 / sum ref^2): the reference's tolerance metric
    (tests/test_common.hpp:36-44, test_gpu_kernels.cpp:194-201)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    num = float(np.sum((a - ref) ** 2))
    den = float(np.sum(ref ** 2))
    return np.sqrt(num / den) if den > 0 else np.sqrt(num)
