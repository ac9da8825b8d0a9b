"""Pins the C oracle (oracle/oracle.c) to the reference's own compiled code.

Every check here compares the restatement with oracle/_ref/libbtf_ref.so,
built from the reference's sources, on the same seeded inputs. The cases follow
the reference's tests/test_packed.cpp (seed-generated, 30 % zero weights,
N=37, K=1024) plus the edge cases the GEMV path meets (all-zero and negative
zero Q8 blocks, subnormal fp16 scales, odd row counts).
"""
import numpy as np
import pytest

from conftest import rel_rms


def _test_packed_weights(rng, N, K):
    # tests/test_packed.cpp:16-20: N(0,1) weights, ~30 % forced to zero
    w = rng.standard_normal((N, K)).astype(np.float32)
    w *= (rng.random((N, K)) < 0.3) == 0
    return w


def test_fp16_rounding_matches_reference(orc, ref):
    rng = np.random.default_rng(11)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 0.02,
        (rng.random(20000).astype(np.float32) * 2e-4),  # around the fp16 subnormal range
        np.array([0.0, -0.0, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08, 65504.0, 65519.0, 65520.0, 1e9,
                  -1e-9, np.inf, -np.inf], dtype=np.float32),
        np.frombuffer(rng.integers(0, 2**32, 20000, dtype=np.uint32).astype(np.uint32).tobytes(), dtype=np.float32),
    ])
    for v in vals:
        if np.isnan(v):
            continue
        h = ref.L.ref_f32_to_f16(float(v))
        assert orc.L.orc_f32_to_f16(float(v)) == h, v
        a, b = orc.L.orc_f16_to_f32(h), ref.L.ref_f16_to_f32(h)
        assert np.float32(a).tobytes() == np.float32(b).tobytes()


def test_ptq_quant_row_matches_reference(orc, ref):
    rng = np.random.default_rng(7)
    w = _test_packed_weights(rng, 37, 1024)
    assert np.array_equal(orc.ptq_quant_rows(w), ref.ptq_quant_rows(w))


def test_ptq_encode_roundtrip(orc, ref):
    import synth

    t = synth.trits(9, 512, seed=5)
    sc = synth.block_scales(9, 512, seed=6)
    src = orc.ptq_encode(t, sc)
    assert np.array_equal(src, synth.encode_ptq1_0(t, sc))  # numpy encoder == C oracle
    assert np.array_equal(orc.ptq_trits(src, 512), t)
    # the reference's trit reader sees the same trits
    blk = src.reshape(-1, 28)
    for b in range(0, blk.shape[0], 7):
        for e in range(128):
            assert ref.L.ref_ptq_trit(blk[b].ctypes.data, e) == t.reshape(-1, 128)[b, e]


@pytest.mark.parametrize("N,K", [(37, 1024), (41, 1152), (1, 128), (16, 5120)])
def test_repack_t2_matches_reference(orc, ref, N, K):
    rng = np.random.default_rng(N * 1000 + K)
    src = ref.ptq_quant_rows(_test_packed_weights(rng, N, K))
    c1, s1 = orc.repack_t2(src, N, K)
    c2, s2 = ref.repack_rows(src, N, K)
    assert np.array_equal(c1, c2) and np.array_equal(s1, s2)
    # test_packed.cpp:24-42: every code is trit + 1 and every scale the block's bytes
    tr = orc.ptq_trits(src, K)
    codes = np.array([[orc.L.orc_t2_code(c1[r].ctypes.data, e) for e in range(K)] for r in range(min(N, 4))])
    assert np.array_equal(codes, tr[: codes.shape[0]] + 1)


def test_q8_matches_reference_and_round_q8_0(orc, ref):
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((3, 1024)) * 3).astype(np.float32)
    x[0, 64:96] = 0.0     # all-zero block (test_packed.cpp:47)
    x[1, 0:32] = -0.0     # all negative zero
    x[2, 32:64] = 0.0
    x[2, 63] = -0.0       # zeros ending in -0.0: d keeps the sign
    x[1, 96:128] = 1e-30  # tiny values
    q1, d1, s1 = orc.q8_rows(x)
    q2, d2, s2 = ref.q8_rows(x)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2)
    assert d1.tobytes() == d2.tobytes()
    assert np.array_equal(s1, q1.reshape(3, -1, 32).astype(np.int32).sum(-1))
    # test_packed.cpp:44-61: q * d reproduces bd::round_q8_0 exactly
    r = ref.round_q8_0(x)
    assert np.array_equal((q1.astype(np.float32).reshape(3, -1, 32) * d1[..., None]).reshape(3, -1), r)
    assert np.array_equal(orc.round_q8_0(x), r)


@pytest.mark.parametrize("N,K,M", [(37, 1024, 1), (64, 1024, 3), (9, 2048, 8), (130, 5120, 2)])
def test_gemv_bit_exact_vs_reference(orc, ref, N, K, M):
    rng = np.random.default_rng(N + K + M)
    src = ref.ptq_quant_rows(_test_packed_weights(rng, N, K))
    codes, scales = ref.repack_rows(src, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q, d, s = ref.q8_rows(x)
    y_ref = ref.gemv(codes, scales, K, q, d, s)
    y_orc = orc.gemv(codes, scales, K, q, d, s)
    assert y_orc.tobytes() == y_ref.tobytes()
    # add mode, and the multithreaded reference split
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    a1 = orc.gemv(codes, scales, K, q, d, s, y=y0.copy(), add=True, threads=3)
    a2 = ref.gemv(codes, scales, K, q, d, s, y=y0.copy(), add=True, threads=3)
    assert a1.tobytes() == a2.tobytes()
    # integer partials are exact: the double reference agrees to 1e-5
    assert rel_rms(y_orc, orc.gemv_f64(codes, scales, K, q, d)) < 1e-5


def test_packed_dot_vs_matvec_raw(orc, ref):
    # test_packed.cpp:63-87: T2 integer dot vs the raw PTQ1_0 matvec with ggml activation rounding
    rng = np.random.default_rng(7)
    N, K = 37, 1024
    src = ref.ptq_quant_rows(_test_packed_weights(rng, N, K))
    x = (rng.standard_normal(K) * 3).astype(np.float32)
    codes, scales = orc.repack_t2(src, N, K)
    q, d, s = orc.q8_rows(x[None])
    y = orc.gemv(codes, scales, K, q, d, s)[0]
    assert rel_rms(y, ref.matvec_raw(src, N, K, x)) < 1e-5


def test_idot_is_code_dot_minus_sum(orc, ref):
    rng = np.random.default_rng(3)
    N, K, M = 12, 512, 2
    src = ref.ptq_quant_rows(_test_packed_weights(rng, N, K))
    codes, _ = ref.repack_rows(src, N, K)
    q, d, s = ref.q8_rows(rng.standard_normal((M, K)).astype(np.float32))
    idot = orc.idot(codes, K, q, s)
    tr = orc.ptq_trits(src, K).astype(np.int64)
    want = np.einsum("nsk,msk->mns", tr.reshape(N, K // 32, 32), q.astype(np.int64).reshape(M, K // 32, 32))
    assert np.array_equal(idot, want)
    # and the reference's own sub-block dot gives the same code dots
    aw = q[0].view(np.uint32)
    cw = codes[0].view(np.uint32)
    for sb in range(K // 32):
        cd = ref.L.ref_sub_dot(int(cw[2 * sb]), int(cw[2 * sb + 1]), aw[sb * 8:].ctypes.data)
        assert cd - s[0, sb] == idot[0, 0, sb]


@pytest.mark.parametrize("n,block,perm,signs", [(1024, 64, False, True), (5120, 1024, False, True),
                                                (2048, 128, True, True), (256, 0, False, False),
                                                (17408, 1024, False, True), (64, 32, True, False)])
def test_prep_transform_matches_reference(orc, ref, n, block, perm, signs):
    # bd::rmsnorm and bd::hadamard_input (cpu_ops.cpp:90-127) against the restatement,
    # bit for bit, on the shapes of the reference's test_prep (test_gpu_kernels.cpp:557-561)
    rng = np.random.default_rng(n + block)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    assert np.array_equal(orc.rmsnorm(x, w, 1e-6).view(np.uint32), ref.rmsnorm(x, w, 1e-6).view(np.uint32))
    assert np.array_equal(orc.rmsnorm(x, None, 1e-6).view(np.uint32), ref.rmsnorm(x, None, 1e-6).view(np.uint32))
    sg = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float32) if signs else None
    pm = (32, n // 64, 2) if perm else (0, 0, 0)
    a = orc.hadamard_input(x, block, pm, sg)
    b = ref.hadamard_input(x, block, pm, sg)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
