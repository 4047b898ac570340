"""Device buffers shared by the ranks of one sequence group through peer mappings.

The head-sharded layer (`sharded.HeadShardedFastMKA`) exchanges the attention
output and the o_proj output by storing straight into the other ranks' memory
over NVLink instead of calling an NCCL all-gather. Each rank (one process per
GPU of a box) allocates one region with `fmka_peer_alloc` (a zero-filled
cudaMalloc), exports its CUDA IPC handle, and maps every other rank's region
with `fmka_peer_import`; the handles cross the torch.distributed group once.
No NVLink multicast object is created: every transfer is a plain load or store
through a peer mapping.

A region holds, at fixed offsets (same layout on every rank):
    flags    uint32 [8]                 barrier slots, one per rank of the group
    gather   bf16 [gs, rows, width]     block j: the attention rows of this
                                        rank's row block computed by rank j
    out      bf16 [T, D]                the layer output of the whole sequence

The reference has no distributed code in the layer (scripts/train_hf_patch.py:97-129
holds its DDP / tensor-parallel use).
"""
from __future__ import annotations

import contextlib
import ctypes
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import torch

from . import _lib

HANDLE_BYTES = 64
_ALIGN = 1024
FLAGS_BYTES = 256


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def region_layout(gs: int, rows: int, width: int, T: int, D: int) -> Tuple[int, int, int]:
    """Byte offsets of the gather and out areas and the region size."""
    gather_off = _align(FLAGS_BYTES)
    out_off = _align(gather_off + gs * rows * width * 2)
    return gather_off, out_off, _align(out_off + T * D * 2)


@dataclass(frozen=True)
class ExchangePlan:
    """Where rank `me` of a group of `gs` puts its data for one sequence of T
    tokens (D model channels, `width` = its heads x 128 attention channels).

    Attention rows [j * rows, (j + 1) * rows) go to region j at byte offset
    `attn_dst_off` ([rows, width] bf16, block `me` of j's gather area); after
    the first barrier rank `me` runs o_proj on the gather area of its own
    region ([gs, rows, width] at `gather_off`) and writes output row m to row
    `gemm_row0` + m of the out area ([T, D] at `out_off`) of every region.
    """
    gs: int
    me: int
    rows: int
    width: int
    gather_off: int
    out_off: int
    nbytes: int
    attn_dst_off: int
    gemm_row0: int


def exchange_plan(gs: int, me: int, T: int, D: int, width: int) -> ExchangePlan:
    if T % gs:
        raise ValueError(f"{T} tokens do not split into {gs} row blocks")
    rows = T // gs
    gather_off, out_off, nbytes = region_layout(gs, rows, width, T, D)
    return ExchangePlan(gs, me, rows, width, gather_off, out_off, nbytes,
                        gather_off + me * rows * width * 2, me * rows)


class _CudaArray:
    """Exposes a device address as a __cuda_array_interface__ object (int16
    elements; bf16 has no type string there) so torch can view it."""

    def __init__(self, ptr: int, shape: Sequence[int]):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": "<i2",
                                         "data": (int(ptr), False), "version": 3, "strides": None,
                                         "stream": None}


def bf16_view(ptr: int, shape: Sequence[int], device: torch.device) -> torch.Tensor:
    """A bf16 tensor over `shape` contiguous elements at device address `ptr`
    (memory owned elsewhere: it stays valid while the owner keeps it)."""
    return torch.as_tensor(_CudaArray(ptr, shape), device=device).view(torch.bfloat16)


def _on(device: torch.device):
    """The CUDA device context for `device` (nothing to enter for a host device)."""
    return torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext()


class PeerRegion:
    """One region per rank of a group, mapped into every rank of the group.

    Collective: construct, `barrier` and `close` on every rank of `group` in
    the same order. `ptrs[j]` is rank j's region as mapped in this process.
    """

    def __init__(self, group, index: int, size: int, nbytes: int, device: torch.device):
        import torch.distributed as dist

        if not 1 <= size <= 8 or not 0 <= index < size:
            raise ValueError("a peer group has 1 to 8 ranks")
        self.index, self.size, self.nbytes, self.device = index, size, nbytes, device
        self.group = group
        self.epoch = 0
        p = ctypes.c_void_p()
        with _on(device):
            _lib.call("fmka_peer_alloc", nbytes, ctypes.byref(p))
        self.local = int(p.value)
        h = (ctypes.c_char * HANDLE_BYTES)()
        _lib.call("fmka_peer_export", self.local, h)
        handles: List[bytes] = [b""] * size
        dist.all_gather_object(handles, bytes(h), group=group)
        self.ptrs: List[int] = []
        self._imported: List[int] = []
        for j, hb in enumerate(handles):
            if j == index:
                self.ptrs.append(self.local)
                continue
            q = ctypes.c_void_p()
            buf = (ctypes.c_char * HANDLE_BYTES).from_buffer_copy(hb)
            with _on(device):
                _lib.call("fmka_peer_import", buf, ctypes.byref(q))
            self.ptrs.append(int(q.value))
            self._imported.append(int(q.value))

    def barrier(self, stream: int) -> None:
        """In stream order: waits until every rank of the group has reached this
        barrier (their earlier work, peer stores included, is visible here)."""
        self.epoch += 1
        arr = (ctypes.c_void_p * self.size)(*[p for p in self.ptrs])  # flags sit at offset 0
        _lib.call("fmka_peer_barrier", arr, self.index, self.size, self.epoch, stream)

    def close(self) -> None:
        """Unmaps the peers' regions and frees this rank's (collective)."""
        import torch.distributed as dist

        if self.local is None:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # nobody touches another rank's region any more
        for p in self._imported:
            _lib.call("fmka_peer_close", p)
        dist.barrier(group=self.group)  # every mapping of this rank's region is closed
        _lib.call("fmka_peer_free", self.local)
        self.local = None
        self.ptrs = []
        self._imported = []
