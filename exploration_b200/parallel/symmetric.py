"""Symmetric heap: one peer-mapped device region per rank of a CP group.

Every rank allocates a region of the same size, exports it with a CUDA IPC
handle and maps all peers' regions (NVLink through NVSwitch on a B200 node),
so a kernel can load from or store to any rank's copy of a slot directly.
Slots come from a bump allocator that every rank drives with the same
sequence of calls, which makes offsets identical across ranks: rank ``r``'s
copy of slot ``s`` is ``ptrs[r] + s``. ``reset()`` recycles the arena at
the start of each training micro-step (after a barrier, so no rank still
reads a slot that a peer is about to overwrite).

The barrier is a device kernel over signal words in each region (bounded
wait; a timeout sets the device error slot instead of hanging). NVLS
objects and ``multimem`` are not used: all traffic is plain peer loads and
stores.

The reference has no counterpart (its exchanges are NCCL collectives only:
st/runtime/parallel.py:16-38).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import _native

ALIGN = 256
DEFAULT_BYTES = 512 << 20


def barrier_timeout_s() -> float:
    return float(os.environ.get("EB200_PEER_TIMEOUT_S", "10"))


class SymmetricHeap:
    """Peer-mapped arena shared by the ranks of ``group`` (one process per GPU)."""

    def __init__(self, group, device: torch.device, nbytes: int = 0):
        self.ext = _native.load(required=True)
        self.group = group
        self.device = torch.device(device)
        self.index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.nbytes = int(nbytes or os.environ.get("EB200_HEAP_BYTES", DEFAULT_BYTES))
        self.base = self.ext.heap_alloc(self.nbytes, self.index)
        self.ptrs = [0] * self.world
        self.ptrs[self.rank] = self.base
        self._opened = []
        if self.world > 1:
            handle = self.ext.heap_ipc_handle(self.base, self.index)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
            for r, raw in enumerate(handles):
                if r != self.rank:
                    ptr = self.ext.heap_open(torch.frombuffer(bytearray(raw), dtype=torch.uint8), self.index)
                    self.ptrs[r] = ptr
                    self._opened.append(ptr)
        self.start = self.ext.heap_signal_bytes()
        self.offset = self.start
        self.high_water = self.start

    # -- arena -------------------------------------------------------------

    def alloc(self, nbytes: int) -> int:
        offset = -(-self.offset // ALIGN) * ALIGN
        if offset + nbytes > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted: need {offset + nbytes} of {self.nbytes} bytes "
                              "(raise EB200_HEAP_BYTES)")
        self.offset = offset + nbytes
        self.high_water = max(self.high_water, self.offset)
        return offset

    def reset(self) -> None:
        self.barrier()
        self.offset = self.start

    def tensor(self, offset: int, shape, dtype=torch.bfloat16) -> torch.Tensor:
        """Local view of a slot."""
        return self.ext.heap_tensor(self.base, offset, list(shape), dtype, self.index)

    def peer_ptrs(self, offset: int) -> list[int]:
        return [p + offset for p in self.ptrs]

    # -- synchronisation ---------------------------------------------------

    def barrier(self) -> None:
        if self.world > 1:
            self.ext.heap_barrier(self.ptrs, self.rank, barrier_timeout_s())

    def close(self) -> None:
        """Collective: every rank closes together (no peer may still read this region)."""
        if self.base:
            self.barrier()
            torch.cuda.synchronize(self.index)
            for ptr in self._opened:
                self.ext.heap_close(ptr, self.index)
            self._opened = []
            self.ext.heap_free(self.base, self.index)
            self.base = 0
