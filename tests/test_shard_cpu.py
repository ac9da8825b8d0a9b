"""N-sharding host logic on CPU: partition properties, and a world_size-2 gloo
run in which each rank computes its row shard with the oracle, all-gathers the
fp32 slices and checks the result bit for bit against the unsharded oracle
GEMV (the partition must not change a single output bit: every row's sum is
computed the same way whichever rank owns it)."""
import os
import socket

import numpy as np
import pytest

import shard
import synth


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("N", [1, 7, 8, 37, 1024, 5120, 17408, 248320])
def test_shard_rows_partition(N, world):
    covered = np.zeros(N, dtype=np.int32)
    pers = set()
    for r in range(world):
        s = shard.shard_rows(N, world, r)
        pers.add(s.per)
        assert s.per % 8 == 0 and 0 <= s.n <= s.per
        assert s.r0 % 8 == 0 or s.n == 0
        covered[s.r0:s.r0 + s.n] += 1
    assert len(pers) == 1 and np.all(covered == 1)
    assert shard.gathered_rows(N, world) >= N


def test_shard_rows_rejects_bad_arguments():
    for args in [(0, 2, 0), (8, 0, 0), (8, 2, 2), (8, 2, -1)]:
        with pytest.raises(ValueError):
            shard.shard_rows(*args)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, N, K, M, out_dir):
    import sys

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle

        orc = oracle.Oracle()
        src = synth.ternary_ptq(N, K, seed=3)
        x = synth.activations(M, K, seed=4)
        q, d, s = orc.q8_rows(x)  # replicated activation: same bits on every rank
        sh = shard.shard_rows(N, world, rank)
        y_local = torch.zeros((M, sh.per), dtype=torch.float32)
        if sh.n:
            codes, scales = orc.repack_t2(src[sh.r0:sh.r0 + sh.n], sh.n, K)
            y_local[:, :sh.n] = torch.from_numpy(orc.gemv(codes, scales, K, q, d, s))
        y_full = torch.empty((M, sh.per * world), dtype=torch.float32)
        shard.all_gather_rows(y_local, y_full)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), shard.unpad(y_full, N).numpy())
    finally:
        dist.destroy_process_group()
    sys.stdout.flush()


@pytest.mark.parametrize("N,K,M", [(37, 256, 1), (64, 1152, 3)])
def test_gloo_world2_sharded_gemv_bit_exact(orc, tmp_path, N, K, M):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), N, K, M, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    codes, scales = orc.repack_t2(synth.ternary_ptq(N, K, seed=3), N, K)
    q, d, s = orc.q8_rows(synth.activations(M, K, seed=4))
    want = orc.gemv(codes, scales, K, q, d, s)
    for r in range(world):
        got = np.load(tmp_path / f"y{r}.npy")
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), r


def test_decoder_shard_rule_equals_shard_rows(btf):
    # the tensor-parallel decoder (C++) splits every matrix exactly as shard.shard_rows
    import ctypes

    L = btf.lib()
    r0, n = ctypes.c_int(), ctypes.c_int()
    for N in (8, 37, 256, 1000, 1024, 5120, 6144, 10240, 17408, 248320):
        for world in (1, 2, 3, 4, 8):
            for rank in range(world):
                assert L.btf_shard_rows(N, world, rank, ctypes.byref(r0), ctypes.byref(n)) == 0
                want = shard.shard_rows(N, world, rank)
                assert (r0.value, n.value) == (want.r0, want.n), (N, world, rank)
    assert L.btf_shard_rows(0, 2, 0, ctypes.byref(r0), ctypes.byref(n)) == 1
