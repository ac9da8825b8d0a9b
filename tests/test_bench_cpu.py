"""CPU legs of bench.py: the reference-arm GEMV sample and the CPU emulator's
decode-step sample, run on small cases (the full-size runs belong to the bench)."""
import os
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)


def _bench():
    import bench

    return bench


def test_cpu_decode_reference_extrapolates_per_token_time(ref):
    bench = _bench()
    small = dict(bench.CONFIG3, n_layer=16, n_embd=512, n_ff=1024, n_vocab=1000, n_head=4, n_head_kv=2,
                 head_dim=128, n_rot=64, d_state=64, n_group=2, dt_rank=4, d_inner=256, hadamard_block=128)
    out = bench.cpu_decode_reference(2, steps=2, geometry=small)
    assert out["kind"] == "reference" and out["unit"] == "tok/s" and out["cores"] == 2
    assert out["value"] > 0 and abs(out["value"] * out["s_per_token"] - 1.0) < 1e-9
    assert "to 16 layers" in out["sample"]
    dirs = [d for d in (os.environ.get("TMPDIR"), "/dev/shm", "/tmp", ROOT) if d and os.path.isdir(d)]
    assert not [f for d in dirs for f in os.listdir(d) if f.startswith(f"btf_cpu_decode_{os.getpid()}_")]


def test_cpu_reference_gemv_line(ref):
    bench = _bench()
    out = bench.cpu_reference(2, reps=1)
    assert out["kind"] == "reference" and out["unit"] == "GB/s" and out["value"] > 0 and out["cores"] == 2
