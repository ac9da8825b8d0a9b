"""CPU checks of the whole-decoder oracles and of the GGUF metadata the decoder binds.

Two oracles for the decode step:
- the reference's CPU emulator of its CUDA decode step (src/emu_decoder.cpp,
  btf::make_emu_decoder), compiled from the reference's sources into
  oracle/_ref/libbtf_ref.so with its synthetic qwen35 writer
  (ref/bonsai-decoder/src/synth.cpp);
- oracle/decode.py, a restatement of that step over the plain-C oracle and
  numpy, pinned here to the emulator's logits on every synthetic model the GPU
  decoder is tested on.
"""
import numpy as np
import pytest

import decode
import oracle
from conftest import DECODER_CONFIGS, DECODER_PROMPT, rel_rms

PROMPT = DECODER_PROMPT


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


@pytest.mark.parametrize("label", list(DECODER_CONFIGS))
def test_restated_decode_step_matches_the_emulator(orc, ref, tmp_path, label):
    # prompt, then 15 greedy steps fed back: the restatement reproduces the
    # emulator's logits bit for bit (same C library transcendentals, same
    # float32 summation order, the pinned C oracle for prep, Q8 and GEMV)
    cfg = dict(DECODER_CONFIGS[label])
    n_layer = cfg.pop("n_layer", 8)
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=n_layer, seed=1, **cfg)
    emu = oracle.Emulator(ref, path, n_ctx=32, threads=1)
    dec = decode.DecodeOracle(orc, path, n_ctx=32)
    assert dec.V == emu.hp["n_vocab"] and dec.L == n_layer and dec.DI == emu.hp["d_inner"]
    tok, first = None, None
    for i in range(len(PROMPT) + 15):
        t = PROMPT[i] if i < len(PROMPT) else tok
        ne, le = emu.step(t)
        nd, ld = dec.step(t)
        first = ld if first is None else first
        assert np.array_equal(ld, le), f"step {i}: logits differ, rel-rms {rel_rms(ld, le):.3e}"
        assert nd == ne
        tok = ne
    emu.close()
    # reset clears the conv, delta-rule and KV state: the first step repeats
    dec.reset()
    assert np.array_equal(dec.step(PROMPT[0])[1], first)


@pytest.mark.parametrize("plant", ["no q rounding", "no bf16 alpha/beta", "no v regrouping"])
def test_pin_detects_a_planted_mistake(orc, ref, tmp_path, plant):
    # the bit-exact pin is sensitive: one planted deviation in the restatement
    # (never in the product) shows up in the logits within the prompt
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=8, seed=1)
    emu = oracle.Emulator(ref, path, n_ctx=16, threads=1)
    dec = decode.DecodeOracle(orc, path, n_ctx=16, round_q_f16=plant != "no q rounding")
    for lay in dec.layers:
        if plant == "no bf16 alpha/beta" and lay["rec"]:
            lay["ab_bf16"] = False
        if plant == "no v regrouping" and lay["rec"]:
            block, perm, signs = lay["out"].hx
            lay["out"].hx = (block, (0, 0, 0), signs)
    differs = [not np.array_equal(dec.step(t)[1], emu.step(t)[1]) for t in PROMPT]
    emu.close()
    assert any(differs)


def test_restated_decode_step_rejects_like_the_emulator(orc, ref, tmp_path):
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=4, seed=2)
    dec = decode.DecodeOracle(orc, path, n_ctx=2)
    with pytest.raises(ValueError):
        dec.step(dec.V)
    dec.step(1)
    dec.step(2)
    with pytest.raises(RuntimeError):
        dec.step(3)  # context full


def test_restated_gguf_reader_agrees_with_the_library(btf, ref, tmp_path):
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=4, seed=3)
    kv, ts = decode.read_gguf(path)
    assert kv["general.architecture"] == "qwen35" and kv["qwen35.block_count"] == 4
    with btf.GgufFile(path) as g:
        for name, (t, ne, raw) in ts.items():
            info = g.tensor(g.find(name))
            assert info["type"] == t and info["ne"] == ne, name
