"""Failure detection on the GPU without a fault: a bounded device-side wait that
runs out.

Every device-side wait of the library (the tagged and counted all-gather
completions, the cross-rank barrier, the TMA/mbarrier waits) gives up after a
time limit, records a time-out in the device error word and returns, so the
context stays usable and the host learns of it from btf_device_error. Here the
tag check of the tagged all-gather (btf_gather_wait) waits for tags that no
launch ever stores, on one GPU: the wait must end after its 2 s limit with the
error word set to the time-out code, the word must clear, and a GEMV launched
afterwards must still match the oracle. Nothing faults, traps or hangs. The
file is named to run after the other GPU tests."""
import time

import numpy as np
import pytest

import synth
from conftest import rel_rms

pytestmark = pytest.mark.gpu

ERR_WAIT_TIMEOUT = 1  # the device error word's time-out code


def test_tag_wait_that_runs_out_reports_a_timeout_and_the_context_stays_usable(cuda, btf, orc):
    import torch

    assert btf.device_error() == 0
    words = torch.zeros(3000, dtype=torch.int64, device=cuda)  # tag half 0: never epoch * 1024 + site
    epoch = torch.ones(1, dtype=torch.int32, device=cuda)
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        btf.gather_wait([(words.data_ptr(), words.numel(), 5)], epoch.data_ptr())
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert btf.device_error() == ERR_WAIT_TIMEOUT
        assert btf.device_error(clear=True) == ERR_WAIT_TIMEOUT
        assert btf.device_error() == 0
        assert waited >= 1.0, waited  # it gave up at its limit, not at once
    finally:
        btf.device_error(clear=True)

    # the context still runs kernels correctly
    K, N = 1024, 40
    src = synth.ternary_ptq(N, K, seed=21)
    pm = btf.repack_panels(torch.from_numpy(src).to(cuda), N, K)
    x = synth.activations(1, K, seed=22)
    act = btf.quant_q8(torch.from_numpy(x).to(cuda))
    y = torch.empty((1, N), device=cuda)
    btf.launch_gemv([(pm, y, N)], K, 1, act, btf.STORE)
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    codes, scales = orc.repack_t2(src, N, K)
    q, d, s = orc.q8_rows(x)
    assert rel_rms(y.cpu().numpy(), orc.gemv(codes, scales, K, q, d, s)) <= 1e-5
