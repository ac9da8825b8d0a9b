"""GPU parity of the persistent GEMV chain (btf_chain_encode / btf_chain_run).

The chain replaces the reference decoder's per-matmul launch_prep + launch_gemv
pairs (src/cuda/gpu_decoder.cu:401-450) with one launch in which op i+1 reads
what op i wrote. The bar, written in each test:
  * every op's fp32 output within rel-RMS 1e-5 of the oracle GEMV (the
    reference's tolerance, tests/test_gpu_kernels.cpp:194-201) given the op's
    actual input buffer after the run, plus the per-element bound
    |y - y64| <= 1e-5 * sum |terms| of the GEMV tests; the Q8 activation the op
    used is the oracle's Q8 of (RMSNorm of) that input, so a single flipped q
    would fail the bound;
  * the RMSNorm sum of squares follows the kernel's fixed parallel order,
    restated by `chain_norm_scale` below; the resulting scale is also within
    1 ulp of the reference's sequential bd::rmsnorm scale;
  * ordering: a multi-op chain (in-place residual adds) equals the same ops run
    as one-op chains in sequence, bit for bit; a second run and a graph replay
    reproduce the first, bit for bit.
"""
import numpy as np
import pytest

import synth
from conftest import rel_rms

pytestmark = pytest.mark.gpu

TOL = 1e-5
EPS = 1e-6


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


class Mat:
    def __init__(self, btf, orc, N, K, seed, device):
        self.N, self.K = N, K
        src = synth.ternary_ptq(N, K, seed=seed)
        self.codes, self.scales = orc.repack_t2(src, N, K)
        self.pm = btf.repack_panels(_dev(src, device), N, K)


def chain_norm_scale(x, eps):
    """Per-row RMSNorm scale 1/sqrt(mean(x^2) + eps) with the chain kernel's
    sum-of-squares order: items (row, 32-column block) of the padded activation
    are split over 4 CTAs in contiguous quarters; thread t of a CTA sums its items
    t, t + 256, ... (each item's 32 squares in column order, double); a lane
    butterfly (xor 16..1) per warp; warps, then CTAs, in order."""
    M, K = x.shape
    NB = 1 if M == 1 else 2
    nsp, nsub = -(-K // 1024) * 32, K // 32
    total = NB * nsp
    blk = np.cumsum((x.astype(np.float64) ** 2).reshape(M, nsub, 32), axis=2)[..., -1]
    tot = np.zeros(NB)
    for r in range(4):
        lo, hi = r * total // 4, (r + 1) * total // 4
        part = np.zeros((256, NB))
        for i in range(lo, hi):
            m, b = divmod(i, nsp)
            if m < M and b < nsub:
                part[(i - lo) % 256, m] += blk[m, b]
        cta = np.zeros(NB)
        for w in range(8):
            v = part[32 * w:32 * w + 32].copy()
            for o in (16, 8, 4, 2, 1):
                v = v + v[np.arange(32) ^ o]
            cta = cta + v[0]
        tot = tot + cta
    mean = (tot[:M] / np.float64(K)).astype(np.float32)
    return (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)


def _q8_input(orc, x, normw):
    """The Q8 activation a chain op quantises from input x (after RMSNorm when normw is given)."""
    if normw is not None:
        sc = chain_norm_scale(x, EPS)
        x = (x * sc[:, None]).astype(np.float32) * normw[None, :].astype(np.float32)
        x = x.astype(np.float32)
    return orc.q8_rows(np.ascontiguousarray(x, dtype=np.float32))


def _abs_terms(orc, mat, q, d, s):
    idot = orc.idot(mat.codes, mat.K, q, s).astype(np.float64)
    sc = np.array([orc.L.orc_f16_to_f32(int(v)) for v in mat.scales.reshape(-1)], dtype=np.float64)
    sc = np.repeat(sc.reshape(mat.N, -1), 4, axis=1)
    return np.abs(idot * sc[None] * d.astype(np.float64)[:, None, :]).sum(-1)


def _check_op(orc, mats, mode, x, normw, y_before, y_after, label):
    """One op's outputs against the oracle given its actual input x."""
    q, d, s = _q8_input(orc, x, normw)
    if mode == 2:  # swiglu
        g, u = mats
        want = orc.gemv_swiglu((g.codes, g.scales), (u.codes, u.scales), g.K, q, d, s)
        g64 = orc.gemv_f64(g.codes, g.scales, g.K, q, d)
        u64 = orc.gemv_f64(u.codes, u.scales, u.K, q, d)
        assert rel_rms(y_after[0], want) <= TOL, (label, rel_rms(y_after[0], want))
        assert rel_rms(y_after[0], g64 / (1 + np.exp(-g64)) * u64) <= TOL, label
        return
    for k, m in enumerate(mats):
        y0 = y_before[k] if mode == 1 else None
        want = orc.gemv(m.codes, m.scales, m.K, q, d, s, y=None if y0 is None else y0.copy(), add=mode == 1)
        y64 = orc.gemv_f64(m.codes, m.scales, m.K, q, d) + (y0 if mode == 1 else 0)
        bound = _abs_terms(orc, m, q, d, s) + (np.abs(y0) if mode == 1 else 0)
        got = y_after[k]
        assert rel_rms(got, want) <= TOL, (label, k, rel_rms(got, want))
        err = np.abs(got.astype(np.float64) - y64)
        assert np.all(err <= TOL * bound + 1e-30), (label, k, float((err - TOL * bound).max()))


@pytest.mark.parametrize("K,Ns,mode,M,norm", [
    (1024, [37, 64, 9], 0, 1, False),   # three segments, few units per CTA (slice-split warps)
    (1152, [40, 24], 0, 2, True),       # a partial second slice, two activation rows, RMSNorm
    (5120, [6144, 1024, 1024], 0, 1, True),  # the q/k/v call site of configuration 1
    (6144, [5120], 1, 1, False),        # o + residual add
    (5120, [17408, 17408], 2, 1, True),  # gate/up swiglu with RMSNorm
    (17408, [5120], 1, 2, False),       # down + residual add, two rows
    (2048, [264, 264], 2, 2, False),    # swiglu, ragged rows
])
def test_chain_single_op_vs_oracle(cuda, btf, orc, K, Ns, mode, M, norm):
    import torch

    rng = np.random.default_rng(K + sum(Ns) + 7 * mode + M)
    mats = [Mat(btf, orc, n, K, seed=K * 3 + i + mode, device=cuda) for i, n in enumerate(Ns)]
    x = synth.activations(M, K, seed=K + M).astype(np.float32) * np.float32(3.0)
    normw = rng.uniform(0.5, 1.5, size=K).astype(np.float32) if norm else None
    ld_pad = 3
    ys0 = [rng.standard_normal((M, n + ld_pad)).astype(np.float32) for n in Ns]
    ys = [_dev(y, cuda) for y in ys0]
    segs = [(m.pm, ys[i] if not (mode == 2 and i == 1) else None, (m.N + ld_pad) if not (mode == 2 and i == 1) else 0)
            for i, m in enumerate(mats)]
    op = btf.ChainOp(segs, K, mode, _dev(x, cuda), None if normw is None else _dev(normw, cuda), EPS)
    ch = btf.Chain([op], M=M)
    ch.run()
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    after = [y.cpu().numpy() for y in ys]
    for i, n in enumerate(Ns):
        if mode == 2 and i == 1:
            continue
        assert np.array_equal(after[i][:, n:], ys0[i][:, n:]), "wrote past N"
    _check_op(orc, mats, mode, x, normw, [y[:, :n] for y, n in zip(ys0, Ns)],
              [y[:, :n] for y, n in zip(after, Ns)], f"K={K} mode={mode} M={M}")


def test_chain_norm_scale_vs_reference_rmsnorm(orc):
    # the kernel's parallel sum order moves the RMSNorm scale by at most 1 ulp
    # from bd::rmsnorm's sequential double sum (cpu_ops.cpp:113-127)
    for K, M, seed in ((5120, 1, 1), (17408, 1, 2), (1152, 2, 3)):
        x = synth.activations(M, K, seed=seed).astype(np.float32)
        got = chain_norm_scale(x, EPS)
        ss = np.array([np.cumsum(x[m].astype(np.float64) ** 2)[-1] for m in range(M)])
        want = (np.float32(1.0) / np.sqrt((ss / K).astype(np.float32) + np.float32(EPS))).astype(np.float32)
        ulp = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
        assert np.all(ulp <= 1), ulp


def _layer_chain_ops(btf, mats, bufs, norms, K_e):
    """One decoder layer's matmul call sites in the reference's order
    (gpu_decoder.cu:411-416, :437-450) on an in-place residual stream h."""
    h, q, k, v, f = bufs["h"], bufs["q"], bufs["k"], bufs["v"], bufs["f"]
    return [
        btf.ChainOp([(mats["q"].pm, q, q.shape[1]), (mats["k"].pm, k, k.shape[1]), (mats["v"].pm, v, v.shape[1])],
                    K_e, btf.STORE, h, norms[0], EPS),
        btf.ChainOp([(mats["o"].pm, h, h.shape[1])], q.shape[1], btf.ADD, q),
        btf.ChainOp([(mats["gate"].pm, f, f.shape[1]), (mats["up"].pm, None, 0)], K_e, btf.SWIGLU, h, norms[1], EPS),
        btf.ChainOp([(mats["down"].pm, h, h.shape[1])], f.shape[1], btf.ADD, f),
    ]


def test_chain_ordering_bit_exact(cuda, btf, orc):
    import torch

    E, Q, KV, F, L = 1024, 1536, 256, 2048, 2
    rng = np.random.default_rng(5)
    layers = []
    for li in range(L):
        shapes = {"q": (E, Q), "k": (E, KV), "v": (E, KV), "o": (Q, E), "gate": (E, F), "up": (E, F), "down": (F, E)}
        layers.append({n: Mat(btf, orc, N, K, seed=100 * li + j, device=cuda)
                       for j, (n, (K, N)) in enumerate(shapes.items())})
    norms = [[_dev(rng.uniform(0.5, 1.5, size=E).astype(np.float32), cuda) for _ in range(2)] for _ in range(L)]
    h0 = synth.activations(1, E, seed=9).astype(np.float32)
    bufs = {"h": _dev(h0, cuda), "q": torch.zeros((1, Q), device=cuda), "k": torch.zeros((1, KV), device=cuda),
            "v": torch.zeros((1, KV), device=cuda), "f": torch.zeros((1, F), device=cuda)}
    ops = [op for li in range(L) for op in _layer_chain_ops(btf, layers[li], bufs, norms[li], E)]
    whole = btf.Chain(ops)
    singles = [btf.Chain([op]) for op in ops]

    def reset():
        bufs["h"].copy_(_dev(h0, cuda))
        for n in ("q", "k", "v", "f"):
            bufs[n].zero_()

    def snap():
        torch.cuda.synchronize()
        return {n: t.cpu().numpy().copy() for n, t in bufs.items()}

    reset()
    whole.run()
    a = snap()
    reset()
    whole.run()  # the program's counters carry over from the first run
    b = snap()
    reset()
    for c in singles:
        c.run()
    c1 = snap()
    assert btf.device_error() == 0
    for n in bufs:
        assert np.array_equal(a[n], b[n]), n
        if all(s.grid == whole.grid for s in singles):
            assert np.array_equal(a[n], c1[n]), n  # same unit split: bit-exact
        else:
            assert rel_rms(a[n], c1[n]) <= 1e-4, n
    # graph capture: one replay == eager
    st = torch.cuda.Stream(device=cuda)
    g = torch.cuda.CUDAGraph()
    reset()
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=st):
        whole.run(stream=st)
    reset()
    torch.cuda.synchronize()
    g.replay()
    gr = snap()
    for n in bufs:
        assert np.array_equal(a[n], gr[n]), n
    # the last layer's down op against the oracle from the buffers it read
    reset()
    for c in singles[:-1]:
        c.run()
    pre = snap()
    singles[-1].run()
    post = snap()
    _check_op(orc, [layers[-1]["down"]], btf.ADD, pre["f"], None, [pre["h"]], [post["h"]], "last down")


def test_chain_config1_layer_vs_oracle(cuda, btf, orc):
    # configuration 1's shapes, each op reading the previous op's output; the
    # residual targets are separate preset buffers so that every op can be
    # checked against the oracle from the buffers it read
    import torch

    shapes = {n: (K, N) for n, K, N in synth.LAYER_SHAPES}
    mats = {n: Mat(btf, orc, N, K, seed=0, device=cuda) for n, (K, N) in shapes.items()}
    rng = np.random.default_rng(11)
    E, Q, KV, F = 5120, shapes["q"][1], shapes["k"][1], shapes["gate"][1]
    A = synth.activations(1, E, seed=2).astype(np.float32)
    B0 = rng.standard_normal((1, E)).astype(np.float32)
    C0 = rng.standard_normal((1, E)).astype(np.float32)
    wa, wf = (rng.uniform(0.5, 1.5, size=E).astype(np.float32) for _ in range(2))
    t = {"A": _dev(A, cuda), "B": _dev(B0, cuda), "C": _dev(C0, cuda), "q": torch.zeros((1, Q), device=cuda),
         "k": torch.zeros((1, KV), device=cuda), "v": torch.zeros((1, KV), device=cuda),
         "f": torch.zeros((1, F), device=cuda)}
    ops = [
        btf.ChainOp([(mats["q"].pm, t["q"], Q), (mats["k"].pm, t["k"], KV), (mats["v"].pm, t["v"], KV)], E, btf.STORE,
                    t["A"], _dev(wa, cuda), EPS),
        btf.ChainOp([(mats["o"].pm, t["B"], E)], Q, btf.ADD, t["q"]),
        btf.ChainOp([(mats["gate"].pm, t["f"], F), (mats["up"].pm, None, 0)], E, btf.SWIGLU, t["B"], _dev(wf, cuda),
                    EPS),
        btf.ChainOp([(mats["down"].pm, t["C"], E)], F, btf.ADD, t["f"]),
    ]
    btf.Chain(ops).run()
    torch.cuda.synchronize()
    assert btf.device_error() == 0
    r = {n: v.cpu().numpy() for n, v in t.items()}
    _check_op(orc, [mats["q"], mats["k"], mats["v"]], 0, A, wa, None, [r["q"], r["k"], r["v"]], "qkv")
    _check_op(orc, [mats["o"]], 1, r["q"], None, [B0], [r["B"]], "o")
    _check_op(orc, [mats["gate"], mats["up"]], 2, r["B"], wf, None, [r["f"]], "gate/up")
    _check_op(orc, [mats["down"]], 1, r["f"], None, [C0], [r["C"]], "down")


def test_chain_rejects_bad_arguments(cuda, btf):
    import torch

    x = torch.zeros((1, 1024), device=cuda)
    y = torch.zeros((1, 8), device=cuda)
    pm = btf.repack_panels(_dev(synth.ternary_ptq(8, 1024, seed=1), cuda), 8, 1024)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        btf.Chain([btf.ChainOp([(pm, y, 8)], 1000, btf.STORE, x)])
    with pytest.raises(RuntimeError, match="M <="):
        btf.Chain([btf.ChainOp([(pm, y, 8)], 1024, btf.STORE, x)], M=3)
    with pytest.raises(RuntimeError, match="swiglu"):
        btf.Chain([btf.ChainOp([(pm, y, 8)], 1024, btf.SWIGLU, x)])
