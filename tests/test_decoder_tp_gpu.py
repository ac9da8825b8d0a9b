"""Tensor-parallel decode (btf_decoder_synthetic_tp) on 2 GPUs: every ternary
matmul of the step is N-sharded over the ranks and all-gathered by the GEMV's
NVLink epilogue, the rest runs replicated. Both ranks must produce bit-identical
logits (every rank's copy of a gathered output receives the same values), and
they must agree with the one-GPU decoder of the same seeded model: the same
greedy tokens and logits within rel-RMS 1e-3 (a shard's CTA split can change
the fp32 summation order of a GEMV row, which is within the GEMV's 1e-5 per
launch; 1e-3 bounds its growth over the layers). Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

from conftest import rel_rms

pytestmark = pytest.mark.gpu

DIMS = dict(n_layer=4, n_embd=512, n_ff=1024, n_vocab=1000, n_head=4, n_head_kv=2, head_dim=128, n_rot=64,
            d_state=64, n_group=2, dt_rank=4, conv_kernel=4, hadamard_block=128, rope_base=1e7, rms_eps=1e-6)
TOKENS = [7, 11, 3, 999, 42, 5]


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
        dec = btf.Decoder(dims=DIMS, seed=11, n_ctx=32, device=rank, world=world, rank=rank)
        plan = btf.plan_memory(dims=DIMS, n_ctx=32, world=world, rank=rank)
        np.save(os.path.join(out_dir, f"mem_r{rank}.npy"), np.array([dec.info()["device_bytes"], plan["device_bytes"]]))
        dec.connect_tp()
        logits, toks = [], []
        for t in TOKENS:
            nxt, lg = dec.step(t, logits=True)
            logits.append(lg)
            toks.append(nxt)
        dec.run(3)  # device-side loop, every rank in step
        torch.cuda.synchronize()
        assert btf.device_error() == 0
        np.save(os.path.join(out_dir, f"tp_r{rank}.npy"), np.stack(logits))
        np.save(os.path.join(out_dir, f"tok_r{rank}.npy"), np.array(toks))
        dist.barrier()  # no rank still stores into another's arena
        dec.close()
        dist.barrier()
        if rank == 0:
            with btf.Decoder(dims=DIMS, seed=11, n_ctx=32, device=0) as one:
                ref = [one.step(t, logits=True) for t in TOKENS]
            np.save(os.path.join(out_dir, "one.npy"), np.stack([lg for _, lg in ref]))
            np.save(os.path.join(out_dir, "one_tok.npy"), np.array([n for n, _ in ref]))
    finally:
        dist.destroy_process_group()


def test_tp_decode_matches_one_gpu(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    tp = [np.load(tmp_path / f"tp_r{r}.npy") for r in range(world)]
    assert all(np.array_equal(tp[0], t) for t in tp[1:]), "ranks disagree"
    one = np.load(tmp_path / "one.npy")
    assert np.array_equal(np.load(tmp_path / "tok_r0.npy"), np.load(tmp_path / "one_tok.npy"))
    for s in range(len(TOKENS)):
        assert np.all(np.isfinite(tp[0][s]))
        assert rel_rms(tp[0][s], one[s]) <= 1e-3, (s, rel_rms(tp[0][s], one[s]))
    for r in range(world):  # each rank allocated exactly its memory plan
        held, planned = np.load(tmp_path / f"mem_r{r}.npy")
        assert held == planned > 0, (r, held, planned)
