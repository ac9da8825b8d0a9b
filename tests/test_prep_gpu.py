"""GPU parity of the fused prep (btf_prep: RMSNorm -> permutation -> signs ->
Hadamard -> Q8_0) against the host form the reference's own test builds
(tests/test_gpu_kernels.cpp:100-160: bd::rmsnorm + bd::hadamard_input +
q8_block_host, restated in oracle/oracle.c and pinned to those functions).

Bar, as the reference's test_prep: q may differ by at most 1 on at most 1e-3 of
the values (a value within float rounding of a .5 boundary may round the other
way, because the double sum of squares is summed in another order); d within
rel-RMS 1e-4; the normalised rows within rel-RMS 1e-6. Without norm and
transform the prep is bit-exact to btf_quant_q8."""
import numpy as np
import pytest

from conftest import rel_rms

pytestmark = pytest.mark.gpu

# (n, block, norm, perm, signs, M): the reference's cases (test_gpu_kernels.cpp:557-561) + more. perm is
# False, True (head dim 32, two repeats) or an explicit (hd, nk, rep). Rows of n = 1024 k run the
# register-span kernel: k <= 8 in one CTA (norm summed from registers), k > 8 over several CTAs (every
# CTA sums the row); a head dim that is not a multiple of 4 takes its scalar gathers; n = 256 and
# 2560 (span 512) run the shared-memory kernel.
CASES = [(1024, 64, True, False, True, 1), (5120, 1024, True, False, True, 3), (2048, 128, False, True, True, 8),
         (256, 0, True, False, False, 2), (17408, 1024, False, False, True, 1), (6144, 256, True, True, True, 4),
         (5120, 16, True, False, True, 2), (17408, 1024, True, False, True, 2), (9216, 512, True, True, True, 1),
         (6144, 1024, True, (6, 512, 2), True, 2), (8192, 2, False, False, False, 3), (2560, 512, True, True, True, 2)]


@pytest.mark.parametrize("n,block,norm,perm,signs,M", CASES)
def test_prep_matches_host(cuda, btf, orc, n, block, norm, perm, signs, M):
    import torch

    rng = np.random.default_rng(n + block + M)
    x = (rng.standard_normal((M, n)) * 3).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    sg = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float32) if signs else None
    pm = perm if isinstance(perm, tuple) else (32, n // 64, 2) if perm else (0, 0, 0)
    eps = 1e-6
    q, d, s, xn = orc.prep_rows(x, w if norm else None, eps, block, pm, sg)
    dx = torch.from_numpy(x).to(cuda)
    xn_dev = torch.empty((M, n), device=cuda)
    act = btf.prep(dx, torch.from_numpy(w).to(cuda) if norm else None, eps, block, pm,
                   torch.from_numpy(sg).to(cuda) if signs else None, xn_dev)
    torch.cuda.synchronize()
    gq = act.q.cpu().numpy()
    diff = np.abs(gq.astype(np.int32) - q.astype(np.int32))
    assert diff.max() <= 1 and (diff != 0).mean() <= 1e-3, (diff.max(), (diff != 0).mean())
    assert rel_rms(act.d.cpu().numpy(), d) <= 1e-4
    assert rel_rms(xn_dev.cpu().numpy(), xn) <= 1e-6
    # s is the sum of the returned q
    assert np.array_equal(act.s.cpu().numpy(), gq.reshape(M, -1, 32).astype(np.int32).sum(-1))


@pytest.mark.parametrize("n,block", [(5120, 1024), (17408, 256)])
def test_prep_strided_rows(cuda, btf, orc, n, block):
    """Rows with a stride of n + 3 floats (not 16-byte aligned): the scalar loads
    and the unaligned norm sum of the register-span kernel."""
    import torch

    M = 3
    rng = np.random.default_rng(n + 7)
    x = (rng.standard_normal((M, n)) * 2).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    sg = np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float32)
    pm = (32, n // 64, 2)
    q, d, s, xn = orc.prep_rows(x, w, 1e-6, block, pm, sg)
    big = torch.zeros((M, n + 3), device=cuda)
    big[:, :n] = torch.from_numpy(x).to(cuda)
    xn_dev = torch.zeros((M, n + 1), device=cuda)
    act = btf.prep(big[:, :n], torch.from_numpy(w).to(cuda), 1e-6, block, pm, torch.from_numpy(sg).to(cuda),
                   xn_dev[:, :n])
    torch.cuda.synchronize()
    gq = act.q.cpu().numpy()
    diff = np.abs(gq.astype(np.int32) - q.astype(np.int32))
    assert diff.max() <= 1 and (diff != 0).mean() <= 1e-3, (diff.max(), (diff != 0).mean())
    assert rel_rms(act.d.cpu().numpy(), d) <= 1e-4
    assert rel_rms(xn_dev[:, :n].cpu().numpy(), xn) <= 1e-6
    assert np.array_equal(act.s.cpu().numpy(), gq.reshape(M, -1, 32).astype(np.int32).sum(-1))


def test_prep_without_transform_equals_quant_q8(cuda, btf):
    import torch

    x = torch.from_numpy((np.random.default_rng(3).standard_normal((5, 17408)) * 2).astype(np.float32)).to(cuda)
    a = btf.prep(x)
    b = btf.quant_q8(x)
    torch.cuda.synchronize()
    assert np.array_equal(a.q.cpu().numpy(), b.q.cpu().numpy())
    assert np.array_equal(a.d.cpu().numpy().view(np.uint32), b.d.cpu().numpy().view(np.uint32))
    assert np.array_equal(a.s.cpu().numpy(), b.s.cpu().numpy())


def test_prep_rejects_bad_transform(cuda, btf):
    import torch

    x = torch.zeros((1, 5120), device=cuda)
    with pytest.raises(RuntimeError, match="invalid argument"):
        btf.prep(x, block=2048)  # larger than the span (1024)
    with pytest.raises(RuntimeError, match="invalid argument"):
        btf.prep(x, block=24)    # not a power of two
    with pytest.raises(RuntimeError, match="invalid argument"):
        btf.prep(x, block=64, perm=(32, 7, 2))  # hd*nk*rep != n
