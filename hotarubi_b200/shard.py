"""Sharded GEMMs and convolutions over the GPUs of one node, one process per GPU.

Two partitions, each an independent split with one real exchange step (every
rank needs the whole output afterwards):

* columns (BASELINE configs[4]'s large GEMMs): rank r of G computes output
  columns [n0, n1) (whole 128-column tiles, ``columns``) with its slice of
  the weights;
* rows (the C5 convolution): rank r convolves images [i0, i1) of the batch
  (``rows``), i.e. output rows [i0 Ho Wo, i1 Ho Wo), with all the weights.

The product path fuses the exchange into the kernel: every rank's output
buffer is mapped into every other rank with CUDA IPC (``PeerOutput``), and
the epilogue stores each output (FP32 and the MXINT8 copy) into all of them
over NVLink (``Plan.set_peers`` / ``ConvPlan.set_peers``), so the gather
overlaps the next tiles' MMAs; a step ends with ``Group.fence``.

The data plane is the library's own communicator (hrb_comm: NCCL, through
the C ABI, as a C++ host would use it): IPC handle exchange, barriers,
fences and the in-place all-gather (``Group.allgather``, the library
baseline for rows).  torch.distributed only hands rank 0's 128-byte
bootstrap id to the other ranks (any backend, ``Group``), and provides the
column baseline ``gather_columns``.
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


def rows(units: int, rank: int | None = None, ranks: int | None = None) -> tuple[int, int]:
    """Units (images of a convolution batch) [u0, u1) of this (or the given)
    rank: hrb_shard_rows."""
    rank = dist.get_rank() if rank is None else rank
    ranks = dist.get_world_size() if ranks is None else ranks
    return capi.shard_rows(units, rank, ranks)


def row_offsets(units: int, unit_bytes: int, ranks: int, base: int = 0) -> list[int]:
    """Byte offsets of every rank's rows in a buffer of `units` units of
    `unit_bytes` bytes: ranks + 1 entries, for ``Group.allgather``."""
    out = [base + rows(units, r, ranks)[0] * unit_bytes for r in range(ranks)]
    return out + [base + units * unit_bytes]


def exchange(obj) -> list:
    """Every rank's `obj`, in rank order (any torch.distributed backend)."""
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


class Group:
    """The ranks of torch.distributed's default group as an hrb_comm: rank 0
    makes the bootstrap id, torch.distributed passes it on, and from then on
    everything goes through the library."""

    def __init__(self, lib: capi.Library):
        self.rank, self.ranks = dist.get_rank(), dist.get_world_size()
        box = [capi.comm_id_new() if self.rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        self.comm = capi.Comm(lib, box[0], self.rank, self.ranks)

    def exchange(self, record: bytes) -> list[bytes]:
        return self.comm.exchange(record)

    def barrier(self) -> None:
        self.comm.barrier()

    def fence(self, stream: int = 0) -> None:
        self.comm.fence(stream)

    def allgather(self, buf, offsets: list[int], stream: int = 0) -> None:
        self.comm.allgather(buf, offsets, stream)

    def close(self) -> None:
        self.comm.close()


class _CudaBlock:
    """A raw device range as a CUDA array (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape: tuple, dtype: str, device: int):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": dtype,
                                         "data": (ptr, False), "version": 3}
        self.device = device


class PeerOutput:
    """One device buffer per rank, mapped into every other rank: `tensor` is
    a float32 view of `shape` at its start, `q` and `s` (with `mx_shape`
    [rows, kpN]) an int8 MXINT8 copy and its uint8 scales [rows, kpN / 32]
    after it, `peer_bases` the peers' mappings in rank order (this rank left
    out), ready for ``Plan.set_peers`` / ``ConvPlan.set_peers``."""

    def __init__(self, lib: capi.Library, group: Group, shape: tuple[int, ...],
                 mx_shape: tuple[int, int] | None = None):
        self.lib = lib
        n = 1
        for d in shape:
            n *= d
        self.fp32_bytes = (4 * n + 255) // 256 * 256
        q_bytes = s_bytes = 0
        if mx_shape is not None:
            q_bytes = (mx_shape[0] * mx_shape[1] + 255) // 256 * 256
            s_bytes = (mx_shape[0] * (mx_shape[1] // 32) + 255) // 256 * 256
        self.ptr, handle = lib.shared_alloc(self.fp32_bytes + q_bytes + s_bytes)
        handles = group.exchange(handle)
        me = group.rank
        self.peer_bases = [lib.peer_open(h) for r, h in enumerate(handles) if r != me]
        dev = torch.cuda.current_device()
        self.tensor = torch.as_tensor(_CudaBlock(self.ptr, tuple(shape), "<f4", dev),
                                      device="cuda")
        self.q = self.s = None
        if mx_shape is not None:
            r, kp = mx_shape
            self.q = torch.as_tensor(_CudaBlock(self.ptr + self.fp32_bytes, (r, kp), "|i1", dev),
                                     device="cuda")
            self.s = torch.as_tensor(_CudaBlock(self.ptr + self.fp32_bytes + q_bytes,
                                                (r, kp // 32), "|u1", dev), device="cuda")

    def close(self) -> None:
        for p in self.peer_bases:
            self.lib.peer_close(p)
        self.peer_bases = []
        if self.ptr:
            self.tensor = self.q = self.s = None
            self.lib.shared_free(self.ptr)
            self.ptr = 0


def gather_columns(c_slice: torch.Tensor, n: int) -> torch.Tensor:
    """The library all-gather of column slices: [M, n1 - n0] of all ranks ->
    [M, n] (torch.distributed all_gather, then an interleave)."""
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
