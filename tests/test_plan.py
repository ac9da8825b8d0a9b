"""Memory plan of the decoder (btf_plan_memory), checked on the CPU.

The plan replaces btf::plan_memory / MemoryPlan (src/repack.cpp:142-204,
include/btf/fast.hpp:50-69) for the panel layout. It runs the decoder's own
binding with every device call skipped. These tests recompute each figure
independently from the GGUF's tensor shapes (oracle/decode.py's reader):
- panel sizes;
- vector sizes;
- KV cache and recurrent state;
- the reference's bytes-per-step definition, restated for panels.

A GPU test checks the opened decoder's allocation total against the plan.
"""
import numpy as np
import pytest

import decode
import oracle
from conftest import DECODER_CONFIGS

CONFIG3 = dict(n_layer=64, n_embd=5120, n_ff=17408, n_vocab=248320, n_head=24, n_head_kv=4, head_dim=256, n_rot=64,
               d_state=128, n_group=16, dt_rank=48, d_inner=6144, conv_kernel=4, hadamard_block=1024, rope_base=1e7,
               rms_eps=1e-6)


def panel_bytes(N, K):
    return -(-N // 8) * -(-K // 1024) * 2176


def shard(N, world, rank):
    groups = -(-N // 8)
    per = -(-groups // world) * 8
    r0 = min(N, rank * per)
    return r0, max(0, min(N, r0 + per) - r0)


def expected_from_gguf(path, n_ctx, world=1, rank=0, chunk=64 << 20):
    """The plan recomputed from the file's tensor table."""
    kv, ts = decode.read_gguf(path)
    p = "qwen35."
    L = kv[p + "block_count"] - kv.get(p + "nextn_predict_layers", 0)
    E, V = kv[p + "embedding_length"], ts["token_embd.weight"][1][1]
    HK, HD = kv[p + "attention.head_count_kv"], kv.get(p + "attention.key_length")
    KC, DK, NK, NV, DI = (kv[p + k] for k in ("ssm.conv_kernel", "ssm.state_size", "ssm.group_count",
                                               "ssm.time_step_rank", "ssm.inner_size"))
    C = 2 * DK * NK + DI
    interval = kv.get(p + "full_attention_interval", 4)
    n_gdn = sum(((il + 1) % interval) != 0 for il in range(L))
    n_attn = L - n_gdn
    mats = [n for n, (t, ne, _) in ts.items() if t == decode.T_PTQ1_0 and n != "token_embd.weight"]
    mats = [n for n in mats if not n.startswith("blk.") or int(n.split(".")[1]) < L]
    panels, staging, read = 0, 0, 0
    for n in mats + ([] if "output.weight" in ts else ["token_embd.weight"]):
        K, N = ts[n][1]
        r0, rows = shard(N, world, rank) if world > 1 else (0, N)
        panels += panel_bytes(rows, K)
        read += panel_bytes(rows, K)
        staging = max(staging, 2 * min(-(-rows // 8) * 8, max(8, chunk // (K // 128 * 28) // 8 * 8)) * (K // 128 * 28))
    K, N = ts["token_embd.weight"][1]
    panels += panel_bytes(N, K)  # the whole table, on every rank
    staging = max(staging, 2 * min(-(-N // 8) * 8, max(8, chunk // (K // 128 * 28) // 8 * 8)) * (K // 128 * 28))
    read += E // 4 + E // 64  # one embedding row per step
    vec_names = [n for n, (t, ne, _) in ts.items() if t != decode.T_PTQ1_0 and
                 (not n.startswith("blk.") or int(n.split(".")[1]) < L)]
    vectors = sum(int(np.prod(ts[n][1])) * 4 for n in vec_names)
    signs = 0
    if kv.get("prism.hadamard.version", 0) and kv["prism.hadamard.sign_mode"] == "explicit":
        signs = sum(kv["prism.hadamard.sign_widths"]) * 4
    state_alloc = n_gdn * (KC * C + NV * (DI // NV) * DK) * 4
    state_rw = 2 * n_gdn * ((KC - 1) * C + NV * (DI // NV) * DK) * 4
    return dict(panel_bytes=panels, vector_bytes=vectors + signs, kv_cache_bytes=n_attn * 2 * n_ctx * HK * HD * 2,
                state_bytes=state_alloc, staging_bytes=staging, decode_bytes_per_ctx=n_attn * 2 * HK * HD * 2,
                decode_bytes_fixed=read + vectors + signs + state_rw + 2 * V * 4,
                n_matrices=len(mats) + 1 + (0 if "output.weight" in ts else 1))


@pytest.mark.parametrize("label", list(DECODER_CONFIGS))
def test_plan_of_a_gguf_matches_its_tensor_table(btf, ref, tmp_path, label):
    cfg = dict(DECODER_CONFIGS[label])
    n_layer = cfg.pop("n_layer", 8)
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=n_layer, seed=1, **cfg)
    plan = btf.plan_memory(path, n_ctx=64)
    want = expected_from_gguf(path, 64)
    for k, v in want.items():
        assert plan[k] == v, (k, plan[k], v)
    parts = ("panel_bytes", "vector_bytes", "kv_cache_bytes", "state_bytes", "work_bytes")
    assert plan["device_bytes"] == sum(plan[k] for k in parts)
    assert plan["work_bytes"] > 0 and plan["pinned_bytes"] == 16
    assert plan["dims"]["n_layer"] == n_layer
    assert "total resident" in btf.plan_table(plan)


@pytest.mark.parametrize("world", [2, 4])
def test_plan_per_rank_under_tensor_parallelism(btf, ref, tmp_path, world):
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=8, seed=1)
    one = btf.plan_memory(path, n_ctx=64)
    plans = [btf.plan_memory(path, n_ctx=64, world=world, rank=r) for r in range(world)]
    for r, p in enumerate(plans):
        want = expected_from_gguf(path, 64, world, r)
        for k, v in want.items():
            assert p[k] == v, (r, k, p[k], v)
        # everything but the matrices is replicated
        for k in ("vector_bytes", "kv_cache_bytes", "state_bytes", "work_bytes", "decode_bytes_per_ctx"):
            assert p[k] == one[k]
    # the ranks' row shards add up to the whole matrices (the embedding table is on every rank)
    kv, ts = decode.read_gguf(path)
    K, N = ts["token_embd.weight"][1]
    table = panel_bytes(N, K)
    assert sum(p["panel_bytes"] - table for p in plans) == one["panel_bytes"] - table


def test_plan_of_the_synthetic_config3_decoder(btf):
    # config 3: the 64-layer decoder the decode benchmark runs (every matmul ternary, f32 alpha/beta)
    d = CONFIG3
    plan = btf.plan_memory(dims=d, n_ctx=4096)
    E, F, V, H, HK, HD = d["n_embd"], d["n_ff"], d["n_vocab"], d["n_head"], d["n_head_kv"], d["head_dim"]
    NV, DK, NK, DI, KC = d["dt_rank"], d["d_state"], d["n_group"], d["d_inner"], d["conv_kernel"]
    C = 2 * DK * NK + DI
    n_gdn = sum((il + 1) % 4 != 0 for il in range(d["n_layer"]))
    n_attn = d["n_layer"] - n_gdn
    ffn = 2 * panel_bytes(F, E) + panel_bytes(E, F)
    gdn = panel_bytes(C, E) + panel_bytes(DI, E) + panel_bytes(E, DI)
    att = panel_bytes(2 * H * HD, E) + 2 * panel_bytes(HK * HD, E) + panel_bytes(E, H * HD)
    mats = d["n_layer"] * ffn + n_gdn * gdn + n_attn * att + panel_bytes(V, E)  # + lm_head
    assert plan["panel_bytes"] == mats + panel_bytes(V, E)
    assert plan["n_matrices"] == 3 * d["n_layer"] + 3 * n_gdn + 4 * n_attn + 2
    vectors = E + d["n_layer"] * 2 * E + n_gdn * (2 * NV * E + 2 * NV + KC * C + DI // NV) + n_attn * 2 * HD
    assert plan["vector_bytes"] == vectors * 4
    assert plan["kv_cache_bytes"] == n_attn * 2 * 4096 * HK * HD * 2
    assert plan["decode_bytes_per_ctx"] == n_attn * 2 * HK * HD * 2 == 65536
    state_rw = 2 * n_gdn * ((KC - 1) * C + NV * (DI // NV) * DK) * 4
    assert plan["decode_bytes_fixed"] == mats + E // 4 + E // 64 + vectors * 4 + state_rw + 2 * V * 4
    assert plan["staging_bytes"] == 0  # synthetic weights are generated on the device
    # fits one B200 many times over
    assert plan["device_bytes"] < 8e9


def test_plan_follows_the_staging_size(btf, ref, tmp_path):
    # FastOptions::staging_mb: smaller chunks, smaller pinned staging; the device plan is unchanged
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=4, seed=1)
    a = btf.plan_memory(path, n_ctx=64, staging_mb=64)
    b = btf.plan_memory(path, n_ctx=64, staging_mb=1)
    assert b["staging_bytes"] == expected_from_gguf(path, 64, chunk=1 << 20)["staging_bytes"]
    assert a["device_bytes"] == b["device_bytes"]
    with pytest.raises(RuntimeError):
        btf.plan_memory(path, staging_mb=5000)


def test_plan_rejects_bad_arguments(btf, ref, tmp_path):
    with pytest.raises(RuntimeError):
        btf.plan_memory(str(tmp_path / "missing.gguf"))
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=4, seed=1)
    with pytest.raises(RuntimeError):
        btf.plan_memory(path, world=2, rank=2)
    with pytest.raises(RuntimeError):
        btf.plan_memory(path, n_ctx=0)
    with pytest.raises(RuntimeError):
        btf.plan_memory(dims=dict(CONFIG3, n_head_kv=5))  # n_head % n_head_kv
    with pytest.raises(RuntimeError):
        btf.plan_memory(dims=dict(CONFIG3, head_dim=512, n_rot=64))  # beyond the attention kernels


def test_cpp_shim_plan_runs_without_a_gpu(btf, ref, tmp_path):
    # btf::cuda::plan_memory (include/btf_b200.hpp) linked against the library
    import os
    import subprocess

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    pkg = os.path.join(root, "bonsai-ternary-fast_b200")
    exe = str(tmp_path / "shim_plan")
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(root, "include"), "-I", "/usr/local/cuda/include",
                        os.path.join(root, "tests", "shim_plan.cpp"), "-o", exe, "-L", pkg, "-lbtf_b200",
                        f"-Wl,-rpath,{pkg}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    path = str(tmp_path / "synth.gguf")
    oracle.synth_model(ref, path, n_layer=4, seed=2)
    r = subprocess.run([exe, path], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    dev, host, fixed, per_ctx = (int(v) for v in r.stdout.splitlines()[0].split())
    plan = btf.plan_memory(path, n_ctx=64)
    assert (dev, host, fixed, per_ctx) == (plan["device_bytes"], plan["pinned_bytes"] + plan["staging_bytes"],
                                           plan["decode_bytes_fixed"], plan["decode_bytes_per_ctx"])
    assert "total resident" in r.stdout
    r = subprocess.run([exe, str(tmp_path / "missing.gguf")], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "btf_plan_memory" in r.stderr


SMALL = dict(n_layer=8, n_embd=256, n_ff=512, n_vocab=300, n_head=2, n_head_kv=1, head_dim=128, n_rot=32, d_state=32,
             n_group=2, dt_rank=4, d_inner=128, conv_kernel=4, hadamard_block=0, rope_base=1e7, rms_eps=1e-6)


def test_written_gguf_plans_like_the_synthetic_decoder(btf, tmp_path):
    # synth.write_qwen35_gguf (the load benchmark's model file) binds to the same
    # allocations as the synthetic decoder of that geometry; only the load's
    # staging differs (synthetic weights are generated on the device)
    import synth

    path = str(tmp_path / "w.gguf")
    size = synth.write_qwen35_gguf(path, SMALL, seed=3)
    assert size == __import__("os").path.getsize(path)
    a = btf.plan_memory(path, n_ctx=64)
    b = btf.plan_memory(dims=SMALL, n_ctx=64)
    assert a["staging_bytes"] > 0 == b["staging_bytes"]
    for k in a:
        if k not in ("staging_bytes", "dims"):
            assert a[k] == b[k], (k, a[k], b[k])
    want = expected_from_gguf(path, 64)
    for k, v in want.items():
        assert a[k] == v, (k, a[k], v)


def test_written_gguf_decodes_like_the_reference_emulator(orc, ref, tmp_path):
    # the reference's own binding accepts the file, and the restated decode
    # step reproduces its emulator bit for bit on it
    import synth

    path = str(tmp_path / "w.gguf")
    synth.write_qwen35_gguf(path, SMALL, seed=5)
    emu = oracle.Emulator(ref, path, n_ctx=16, threads=1)
    assert emu.hp["n_layer"] == 8 and emu.hp["n_vocab"] == 300 and emu.hp["d_inner"] == 128
    dec = decode.DecodeOracle(orc, path, n_ctx=16)
    for t in (1, 5, 9, 200, 33, 7):
        ne, le = emu.step(t)
        nd, ld = dec.step(t)
        assert np.array_equal(ld, le) and nd == ne and np.all(np.isfinite(le))
    emu.close()
