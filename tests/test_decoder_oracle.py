"""CPU checks of the whole-decoder oracle and of the GGUF metadata the decoder binds.

The decoder's oracle is the reference's CPU emulator of its CUDA decode step
(src/emu_decoder.cpp, btf::make_emu_decoder) on the reference's synthetic
qwen35 model (ref/bonsai-decoder/src/synth.cpp), both compiled from the
reference's sources into oracle/_ref/libbtf_ref.so.
"""
import os

import numpy as np
import pytest

import oracle

# the reference's decoder-test prompt (tests/test_common.hpp:67-70)
PROMPT = [259, 272, 44, 32, 259, 261, 103, 97, 264]


def test_emulator_runs_and_is_deterministic(ref, tmp_path):
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=8, seed=1)
    emu = oracle.Emulator(ref, path, n_ctx=64)
    assert emu.hp["n_layer"] == 8 and emu.hp["n_embd"] == 128 and emu.hp["d_inner"] == 128
    toks, logs = [], []
    for t in PROMPT:
        nxt, lg = emu.step(t)
        toks.append(nxt)
        logs.append(lg)
        assert np.all(np.isfinite(lg)) and nxt == int(np.argmax(lg))
    emu.reset()
    for t, want_tok, want_lg in zip(PROMPT, toks, logs):
        nxt, lg = emu.step(t)
        assert nxt == want_tok and np.array_equal(lg, want_lg)
    emu.close()


def test_gguf_metadata_of_the_synthetic_model(ref, btf, tmp_path):
    # the library's GGUF reader sees the reference writer's tensors (the
    # metadata itself is bound by the decoder, checked on the GPU)
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=4, seed=3)
    with btf.GgufFile(path) as g:
        assert g.find("token_embd.weight") >= 0 and g.find("blk.3.attn_q.weight") >= 0
        t = g.tensor(g.find("blk.0.ssm_alpha.weight"))
        assert t["type"] == 30 and t["ne"] == [128, 4]  # BF16 [dt_rank][n_embd]
        t = g.tensor(g.find("blk.0.ffn_gate.weight"))
        assert t["type"] == btf.PTQ1_0 and t["ne"] == [128, 256]
