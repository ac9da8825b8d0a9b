"""N-sharding of the ternary GEMV across the GPUs of one node (host-side plumbing).

Output rows are independent, so the weight stream splits along N with a single
exchange step: rank g owns a contiguous range of whole row groups of every
matrix and only those panels; the Q8 activation is replicated (each rank
quantises the same x bit-identically, so it is not sent anywhere); after the
GEMV, the fp32 output slices are all-gathered.

Every rank gets the same padded slice width `per` (a multiple of `align`
rows), which is what an equal-count all-gather needs; the last rank(s) may own
fewer real rows than `per` (its tail is padding and is dropped after the
gather). The reference has no multi-GPU path (src/cuda/gpu_decoder.cu is a
single-device decoder); this module is the B200 build's own.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence


@dataclass(frozen=True)
class RowShard:
    """Rows [r0, r0 + n) of an N-row matrix, stored in a slice of width `per`."""

    r0: int
    n: int
    per: int


def shard_rows(N: int, world: int, rank: int, align: int = 8) -> RowShard:
    """Contiguous, group-aligned row range of `rank` among `world` ranks."""
    if N <= 0 or world <= 0 or not 0 <= rank < world or align <= 0:
        raise ValueError(f"shard_rows: bad arguments N={N} world={world} rank={rank} align={align}")
    groups = -(-N // align)
    per = -(-groups // world) * align
    r0 = min(N, rank * per)
    n = max(0, min(N, r0 + per) - r0)
    return RowShard(r0, n, per)


def gathered_rows(N: int, world: int, align: int = 8) -> int:
    """Width of the all-gathered output (world * per >= N)."""
    return shard_rows(N, world, 0, align).per * world


class ShardedMatrix:
    """This rank's shard of a ternary [N][K] matrix, resident as panels.

    `src` is the full PTQ1_0 matrix as a uint8 array [N][K/128*28] (numpy or
    torch, host or device); only this rank's rows are copied to the device."""

    def __init__(self, btf, src, N: int, K: int, world: int, rank: int, device, align: int = 8):
        import numpy as np
        import torch

        self.N, self.K, self.world, self.rank = N, K, world, rank
        self.shard = shard_rows(N, world, rank, align)
        self.pm = None
        if self.shard.n > 0:
            part = src[self.shard.r0:self.shard.r0 + self.shard.n]
            if isinstance(part, np.ndarray):
                part = torch.from_numpy(np.ascontiguousarray(part))
            self.pm = btf.repack_panels(part.to(device).contiguous(), self.shard.n, K)

    def segment(self, y_local, ldy: Optional[int] = None):
        """(PanelMatrix, y, ldy) for btf_b200.launch_gemv; y_local is [M][per]."""
        return (self.pm, y_local, ldy if ldy is not None else y_local.shape[-1])


def all_gather_rows(y_local, y_full, group=None) -> None:
    """All-gathers [M][per] slices into y_full [M][world*per] (rank-major columns).

    M == 1 uses all_gather_into_tensor directly on the flat buffers (the slices
    are contiguous); M > 1 gathers into a [world][M][per] staging tensor first."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M, per = y_local.shape
    if M == 1 and y_full.is_contiguous() and dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(y_full.view(-1), y_local.contiguous().view(-1), group=group)
        return
    parts = [torch.empty_like(y_local) for _ in range(world)]
    dist.all_gather(parts, y_local.contiguous(), group=group)
    for g, p in enumerate(parts):
        y_full[:, g * per:(g + 1) * per] = p


def unpad(y_full, N: int):
    """The first N gathered columns (drops the padding rows of the last shards)."""
    return y_full[..., :N]


def local_widths(Ns: Sequence[int], world: int, align: int = 8):
    """Per-rank slice widths of several matrices."""
    return [shard_rows(N, world, 0, align).per for N in Ns]


class _DeviceArray:
    """__cuda_array_interface__ view of raw device memory (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class GatherArena:
    """Full-width output buffers of N-sharded GEMVs, shared by all ranks.

    Each rank allocates one device buffer (btf_alloc): a 256-byte control block
    (its arrival counter at +0, its consumed-arrivals counter at +4, its CTA
    completion counter at +8, its tag epoch at +12) followed by the output
    buffers (float32, or 64-bit (value, tag) words for tagged launches), laid out the same
    on every rank. The buffers' IPC handles are exchanged over the default
    process group, so each process can address every rank's buffer; a sharded
    GEMV then stores each output value into all of them (btf_gemv_gather).
    Collective: every rank constructs it with the same `nbytes`."""

    CTL = 256

    def __init__(self, btf, nbytes: int, world: int, rank: int, device):
        import torch
        import torch.distributed as dist

        self.btf, self.world, self.rank, self.device = btf, world, rank, device
        self.nbytes = (nbytes + 255) // 256 * 256
        self.base = btf.alloc(self.CTL + self.nbytes)
        torch.as_tensor(_DeviceArray(self.base, ((self.CTL + self.nbytes) // 4,), "<u4"), device=device).zero_()
        torch.cuda.synchronize(device)
        handles = [None] * world
        dist.all_gather_object(handles, btf.ipc_handle(self.base))
        self.bases = [self.base if r == rank else btf.ipc_open(handles[r]) for r in range(world)]
        dist.barrier()
        self._next = 0

    def buffer(self, shape, tagged: bool = False) -> tuple:
        """Reserves an output buffer of `shape`: float32, or (tagged) 64-bit (value, tag) words
        as int64. Returns (offset, torch view of this rank's copy)."""
        import torch

        n = 1
        for d in shape:
            n *= d
        esz = 8 if tagged else 4
        off = self._next
        self._next = (off + esz * n + 255) // 256 * 256
        if self._next > self.nbytes:
            raise ValueError("GatherArena: out of space")
        return off, torch.as_tensor(_DeviceArray(self.base + self.CTL + off, shape, "<i8" if tagged else "<f4"),
                                    device=self.device)

    @property
    def epoch_ptr(self) -> int:
        """This rank's tag epoch counter (control block +12)."""
        return self.base + 12

    def word_ptr(self, offset: int) -> int:
        return self.base + self.CTL + offset

    @staticmethod
    def values(words):
        """float32 values of a tagged int64 buffer (low halves)."""
        return words.view(dtype=__import__("torch").float32)[..., ::2]

    def gather_desc(self, seg_offsets_bytes, tagged: bool = False, site: int = 0):
        """btf_gather for a launch whose segment s has its y (this rank's first
        output row, i.e. the buffer offset plus 4 * row0 of this rank's shard) at
        byte offset seg_offsets_bytes[s] within every rank's output area."""
        g = self.btf.GatherC()
        g.world, g.rank = self.world, self.rank
        for s, off in enumerate(seg_offsets_bytes):
            for r in range(self.world):
                g.peer_y[s][r] = self.bases[r] + self.CTL + off
        for r in range(self.world):
            g.flags[r] = self.bases[r]
        g.expect = self.base + 4
        g.done = self.base + 8
        g.tagged, g.site, g.epoch = int(tagged), site, self.epoch_ptr
        return g

    def close(self):
        for r, b in enumerate(self.bases):
            if r != self.rank:
                self.btf.ipc_close(b)
        self.btf.free(self.base)
        self.bases = []
