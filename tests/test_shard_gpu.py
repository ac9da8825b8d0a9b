"""N-sharded GEMV on 2+ GPUs: each rank (one process per GPU, NCCL) repacks and
runs only its row shard through the C ABI, the fp32 slices are all-gathered, and
every rank's gathered output must match the unsharded oracle within rel-RMS
1e-5 (the GEMV's own tolerance; a shard's CTA split differs from the
unsharded launch's, so the fp32 summation order of a row may differ). Run
three times: all-gather by NCCL after the GEMV; fused into the GEMV epilogue
(btf_gemv_gather: NVLink stores into every rank's buffer + arrival counters);
and the tagged form (64-bit (value, tag) words checked by btf_gather_wait),
which also runs a batch of 24 over large shards on the weight-major tcgen05
GEMM and a batch of 8 over lm_head-size shards on the warp-MMA GEMM. Skipped
with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

import shard
import synth
from conftest import rel_rms

pytestmark = pytest.mark.gpu

CASES = [(17408, 5120, 1, 0), (5120, 17408, 1, 1), (1000, 1024, 3, 1), (37, 256, 2, 2)]  # N, K, M, mode
# tagged form only: a batch of 24 over shards of 148 128-row tiles, which
# btf_gemv_gather runs on the weight-major tcgen05 GEMM, and a batch of 8 over
# shards of 148 x 8 32-row units, which it runs on the warp-MMA GEMM (one weight
# pass each)
TAGGED_EXTRA = [(2 * 148 * 128, 1024, 24, 0), (2 * 148 * 8 * 32, 1024, 8, 0)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import btf_b200 as btf

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        btf.kernels_init(rank)
        for ci, (N, K, M, mode) in enumerate(CASES):
            src = synth.ternary_ptq(N, K, seed=10 + ci)
            x = torch.from_numpy(synth.activations(M, K, seed=20 + ci)).to(dev)
            act = btf.quant_q8(x)
            mats = [shard.ShardedMatrix(btf, src, N, K, world, rank, dev)]
            if mode == btf.SWIGLU:
                mats.append(shard.ShardedMatrix(btf, synth.ternary_ptq(N, K, seed=30 + ci), N, K, world, rank, dev))
            sh = mats[0].shard
            y0 = torch.from_numpy(np.random.default_rng(ci).standard_normal((M, N)).astype(np.float32)).to(dev)
            y_local = torch.zeros((M, sh.per), device=dev)
            if mode == btf.ADD:
                y_local[:, :sh.n] = y0[:, sh.r0:sh.r0 + sh.n]
            if sh.n:
                segs = [mats[0].segment(y_local)]
                if mode == btf.SWIGLU:
                    segs.append((mats[1].pm, None, 0))
                btf.launch_gemv(segs, K, M, act, mode)
            y_full = torch.empty((M, sh.per * world), device=dev)
            shard.all_gather_rows(y_local, y_full)
            torch.cuda.synchronize()
            assert btf.device_error() == 0
            np.save(os.path.join(out_dir, f"c{ci}_r{rank}.npy"), shard.unpad(y_full, N).cpu().numpy())
        dist.barrier()
        # the same cases with the all-gather fused into the GEMV epilogue (NVLink stores)
        arena = shard.GatherArena(btf, sum(M * N * 12 + 512 for N, K, M, _ in CASES + TAGGED_EXTRA), world, rank,
                                  dev)
        for ci, (N, K, M, mode) in enumerate(CASES):
            src = synth.ternary_ptq(N, K, seed=10 + ci)
            act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=20 + ci)).to(dev))
            gate = shard.ShardedMatrix(btf, src, N, K, world, rank, dev)
            up = shard.ShardedMatrix(btf, synth.ternary_ptq(N, K, seed=30 + ci), N, K, world, rank, dev) \
                if mode == btf.SWIGLU else None
            sh = gate.shard
            off, y_full = arena.buffer((M, N))
            y_full.copy_(torch.from_numpy(np.random.default_rng(ci).standard_normal((M, N)).astype(np.float32)))
            torch.cuda.synchronize()
            dist.barrier()  # every rank's buffer holds y0 before anyone stores into it
            if sh.n:
                segs = [(gate.pm, y_full[:, sh.r0:], N)]
                if up is not None:
                    segs.append((up.pm, None, 0))
                btf.launch_gemv_gather(segs, K, M, act, mode, arena.gather_desc([off + 4 * sh.r0]))
            torch.cuda.synchronize()
            assert btf.device_error() == 0
            np.save(os.path.join(out_dir, f"g{ci}_r{rank}.npy"), y_full.cpu().numpy())
        dist.barrier()
        # tagged form: (value, tag) words, no counters; a bounded device wait checks the tags
        btf.gather_epoch_advance(arena.epoch_ptr)
        for ci, (N, K, M, mode) in enumerate(CASES + TAGGED_EXTRA):
            src = synth.ternary_ptq(N, K, seed=10 + ci)
            act = btf.quant_q8(torch.from_numpy(synth.activations(M, K, seed=20 + ci)).to(dev))
            gate = shard.ShardedMatrix(btf, src, N, K, world, rank, dev)
            up = shard.ShardedMatrix(btf, synth.ternary_ptq(N, K, seed=30 + ci), N, K, world, rank, dev) \
                if mode == btf.SWIGLU else None
            sh = gate.shard
            off, words = arena.buffer((M, N), tagged=True)
            y0 = torch.from_numpy(np.random.default_rng(ci).standard_normal((M, N)).astype(np.float32)).to(dev)
            words.copy_(y0.view(torch.int32).to(torch.int64) & 0xFFFFFFFF)  # tag 0
            torch.cuda.synchronize()
            dist.barrier()
            segs = [(gate.pm, words[:, sh.r0:], N)]
            if up is not None:
                segs.append((up.pm, None, 0))
            btf.launch_gemv_gather(segs, K, M, act, mode,
                                   arena.gather_desc([off + 8 * sh.r0], tagged=True, site=ci))
            btf.gather_wait([(arena.word_ptr(off), M * N, ci)], arena.epoch_ptr)
            btf.gather_barrier(arena.gather_desc([]))
            torch.cuda.synchronize()
            assert btf.device_error() == 0
            np.save(os.path.join(out_dir, f"t{ci}_r{rank}.npy"), shard.GatherArena.values(words).cpu().numpy())
        dist.barrier()
        arena.close()
    finally:
        dist.destroy_process_group()


def test_sharded_gemv_nccl_matches_oracle(orc, tmp_path):
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    for ci, (N, K, M, mode) in enumerate(CASES):
        codes, scales = orc.repack_t2(synth.ternary_ptq(N, K, seed=10 + ci), N, K)
        q, d, s = orc.q8_rows(synth.activations(M, K, seed=20 + ci))
        y0 = np.random.default_rng(ci).standard_normal((M, N)).astype(np.float32)
        if mode == 2:
            uc, us = orc.repack_t2(synth.ternary_ptq(N, K, seed=30 + ci), N, K)
            want = orc.gemv_swiglu((codes, scales), (uc, us), K, q, d, s, threads=8)
        else:
            want = orc.gemv(codes, scales, K, q, d, s, y=y0.copy() if mode == 1 else None, add=mode == 1, threads=8)
        for r in range(world):
            got = np.load(tmp_path / f"c{ci}_r{r}.npy")
            assert rel_rms(got, want) <= 1e-5, (ci, r, rel_rms(got, want))
            got = np.load(tmp_path / f"g{ci}_r{r}.npy")  # NVLink-gathered in the epilogue
            assert rel_rms(got, want) <= 1e-5, ("gather", ci, r, rel_rms(got, want))
            got = np.load(tmp_path / f"t{ci}_r{r}.npy")  # tagged (value, tag) words
            assert rel_rms(got, want) <= 1e-5, ("tagged", ci, r, rel_rms(got, want))
    for ci, (N, K, M, mode) in enumerate(TAGGED_EXTRA, start=len(CASES)):
        codes, scales = orc.repack_t2(synth.ternary_ptq(N, K, seed=10 + ci), N, K)
        q, d, s = orc.q8_rows(synth.activations(M, K, seed=20 + ci))
        want = orc.gemv(codes, scales, K, q, d, s, threads=8)
        for r in range(world):
            got = np.load(tmp_path / f"t{ci}_r{r}.npy")
            assert rel_rms(got, want) <= 1e-5, ("tagged, small batch", ci, r, rel_rms(got, want))
