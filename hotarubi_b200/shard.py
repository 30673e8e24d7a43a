"""Column-sharded GEMMs over the GPUs of one node, one process per GPU.

BASELINE configs[4] shards large GEMMs along N: rank r of G computes output
columns [n0, n1) (whole 128-column tiles, ``columns``) with its slice of the
weights, and every rank needs all of C afterwards.  Two ways to gather:

* ``PeerOutput`` + ``Plan.set_peers`` (the product path): every rank's C
  buffer is mapped into every other rank with CUDA IPC, and the GEMM
  kernel's epilogue stores each output into all of them over NVLink, so the
  all-gather overlaps the next tiles' MMAs; ranks only synchronise once at
  the end (``complete``).
* ``gather_columns`` (the library baseline): each rank's slice is gathered
  with ``torch.distributed.all_gather`` (NCCL on GPUs, gloo on CPU) and
  interleaved back into [M, N].

Host logic only; the rank set is torch.distributed's default group.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import capi


def columns(n: int, rank: int | None = None, ranks: int | None = None) -> tuple[int, int]:
    """Output columns [n0, n1) of this (or the given) rank."""
    rank = dist.get_rank() if rank is None else rank
    ranks = dist.get_world_size() if ranks is None else ranks
    return capi.shard_columns(n, rank, ranks)


def exchange(obj) -> list:
    """Every rank's `obj`, in rank order (any backend)."""
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


class _CudaBlock:
    """A raw device range as a CUDA array (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape: tuple, dtype: str, device: int):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": dtype,
                                         "data": (ptr, False), "version": 3}
        self.device = device


class PeerOutput:
    """A float32 buffer of `shape` on every rank, mapped into every other
    rank: `tensor` is the local buffer, `peer_bases` the peers' mappings in
    rank order (this rank left out), ready for ``Plan.set_peers``."""

    def __init__(self, lib: capi.Library, shape: tuple[int, ...]):
        self.lib = lib
        n = 1
        for d in shape:
            n *= d
        self.ptr, handle = lib.shared_alloc(4 * n)
        handles = exchange(handle)
        me = dist.get_rank()
        self.peer_bases = [lib.peer_open(h) for r, h in enumerate(handles) if r != me]
        self.tensor = torch.as_tensor(_CudaBlock(self.ptr, tuple(shape), "<f4",
                                                 torch.cuda.current_device()), device="cuda")

    def close(self) -> None:
        for p in self.peer_bases:
            self.lib.peer_close(p)
        self.peer_bases = []
        if self.ptr:
            self.tensor = None
            self.lib.shared_free(self.ptr)
            self.ptr = 0


def complete(stream=None) -> None:
    """Every rank's queued GEMMs (and their peer stores) are finished when
    this returns on every rank: the local work, then a barrier."""
    (stream or torch.cuda.current_stream()).synchronize()
    dist.barrier()


def gather_columns(c_slice: torch.Tensor, n: int) -> torch.Tensor:
    """The library all-gather: [M, n1 - n0] slices of all ranks -> [M, n]."""
    ranks = dist.get_world_size()
    m = c_slice.shape[0]
    width = max(columns(n, r, ranks)[1] - columns(n, r, ranks)[0] for r in range(ranks))
    padded = torch.zeros((m, width), dtype=c_slice.dtype, device=c_slice.device)
    padded[:, :c_slice.shape[1]] = c_slice
    parts = [torch.empty_like(padded) for _ in range(ranks)]
    dist.all_gather(parts, padded)
    out = torch.empty((m, n), dtype=c_slice.dtype, device=c_slice.device)
    for r in range(ranks):
        n0, n1 = columns(n, r, ranks)
        out[:, n0:n1] = parts[r][:, :n1 - n0]
    return out
