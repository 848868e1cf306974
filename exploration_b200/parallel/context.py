"""Data x context parallelism for 1..8 ranks of one node.

* **DP**: replicas of the model; gradients are averaged over all ranks.
* **CP** (Ulysses): the ranks of one CP group hold consecutive, block-aligned
  sequence shards of the same sample. The L layers stay sequence-sharded and
  exchange a one-block *halo* (the previous rank's last layer-input block)
  before every L application, including every pass of a shared layer. The G
  rounds switch layout with a sequence<->head all-to-all, so each rank owns
  ``H / cp`` heads over the whole sequence inside attention.

CP groups are contiguous rank ranges (reference: st/runtime/parallel.py:60-133).
The halo is a point-to-point exchange (rank r -> r+1) rather than an
all-gather, and its backward returns the gradient to the rank that owns the
block. The exchanges here are the NCCL/gloo path; on CUDA the fused
peer-memory kernels of :mod:`.ulysses` replace the all-to-all when a
symmetric heap is attached (``cp_group`` unchanged).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch.autograd import Function

MAX_WORLD = 8


def process_group_timeout() -> datetime.timedelta:
    """Collective timeout; short, so a rank that never arrives ends the job with an error."""
    return datetime.timedelta(seconds=float(os.environ.get("EB200_PG_TIMEOUT_S", "300")))


def init_distributed(device_type: str) -> None:
    if not dist.is_initialized():
        backend = "nccl" if device_type == "cuda" else "gloo"
        kwargs = {"backend": backend, "timeout": process_group_timeout()}
        if device_type == "cuda":
            kwargs["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(**kwargs)


def _to_heads_layout(x, cp):
    """``[B, L, H, D]`` -> send buffer ``[cp, B, L, H/cp, D]`` (chunk s goes to rank s)."""
    batch, length, heads, dim = x.shape
    return x.view(batch, length, cp, heads // cp, dim).permute(2, 0, 1, 3, 4).contiguous()


def _from_heads_layout(buf):
    """Receive buffer ``[cp, B, L, Hc, D]`` (chunk s = rank s's shard) -> ``[B, cp*L, Hc, D]``."""
    cp, batch, length, hc, dim = buf.shape
    return buf.permute(1, 0, 2, 3, 4).reshape(batch, cp * length, hc, dim)


def _to_sequence_layout(x, cp):
    """``[B, cp*L, Hc, D]`` -> send buffer ``[cp, B, L, Hc, D]`` (chunk s = shard s)."""
    batch, total, hc, dim = x.shape
    return x.view(batch, cp, total // cp, hc, dim).permute(1, 0, 2, 3, 4).contiguous()


def _from_sequence_layout(buf):
    """Receive buffer ``[cp, B, L, Hc, D]`` (chunk s = head group s) -> ``[B, L, cp*Hc, D]``."""
    cp, batch, length, hc, dim = buf.shape
    return buf.permute(1, 2, 0, 3, 4).reshape(batch, length, cp * hc, dim)


def exchange(x, group, to_heads: bool):
    cp = dist.get_world_size(group)
    send = _to_heads_layout(x, cp) if to_heads else _to_sequence_layout(x, cp)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return _from_heads_layout(recv) if to_heads else _from_sequence_layout(recv)


class _Ulysses(Function):
    @staticmethod
    def forward(ctx, x, group, to_heads):
        ctx.group, ctx.to_heads = group, to_heads
        return exchange(x, group, to_heads)

    @staticmethod
    def backward(ctx, grad):
        return exchange(grad.contiguous(), ctx.group, not ctx.to_heads), None, None


def _p2p(send_to, send, recv_from, recv, group):
    ops = []
    if send_to is not None:
        ops.append(dist.P2POp(dist.isend, send, dist.get_global_rank(group, send_to), group))
    if recv_from is not None:
        ops.append(dist.P2POp(dist.irecv, recv, dist.get_global_rank(group, recv_from), group))
    for req in dist.batch_isend_irecv(ops):
        req.wait()


class _Halo(Function):
    """Previous rank's last block; rank 0 receives zeros (masked by the layer)."""

    @staticmethod
    def forward(ctx, tail, group):
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        ctx.group, ctx.rank, ctx.size = group, rank, size
        tail = tail.contiguous()
        received = torch.zeros_like(tail)
        _p2p(rank + 1 if rank + 1 < size else None, tail,
             rank - 1 if rank > 0 else None, received, group)
        return received

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        back = torch.zeros_like(grad)
        _p2p(ctx.rank - 1 if ctx.rank > 0 else None, grad,
             ctx.rank + 1 if ctx.rank + 1 < ctx.size else None, back, ctx.group)
        return back, None


@dataclass
class ParallelContext:
    world_size: int = 1
    rank: int = 0
    cp_size: int = 1
    cp_rank: int = 0
    dp_size: int = 1
    dp_rank: int = 0
    cp_group: object = None
    dp_group: object = None
    ulysses: object = None      # optional fused peer-memory exchange (CUDA)

    @classmethod
    def initialize(cls, cp_size: int = 1, device: str = "cuda") -> "ParallelContext":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if not 1 <= world <= MAX_WORLD or cp_size < 1 or world % cp_size:
            raise ValueError(f"need 1..{MAX_WORLD} processes and context_parallel dividing WORLD_SIZE")
        if device == "cuda":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        if world == 1:
            return cls()
        init_distributed(device)
        if dist.get_world_size() != world:
            raise ValueError("initialized process group differs from WORLD_SIZE")
        rank = dist.get_rank()
        cp_group = dp_group = None
        for first in range(0, world, cp_size):
            members = list(range(first, first + cp_size))
            group = dist.new_group(members, timeout=process_group_timeout())
            if rank in members:
                cp_group = group
        for offset in range(cp_size):
            members = list(range(offset, world, cp_size))
            group = dist.new_group(members, timeout=process_group_timeout())
            if rank in members:
                dp_group = group
        return cls(world, rank, cp_size, rank % cp_size, world // cp_size, rank // cp_size,
                   cp_group, dp_group)

    def fused_heap_bytes(self, model, batch: int, length: int) -> int:
        """Symmetric-heap bytes one micro-step of ``model`` needs for the fused exchange.

        Per step the heap holds head-layout slots of ``batch x length x C``
        bf16 values (C = heads per rank x head dim): K and V (two) plus their
        gradients (two), and per read round the query, the attention output and
        their gradients (four); 16 MB covers alignment and signal words.
        """
        heads, hd = int(model.heads), int(model.hd)
        C = heads // max(1, self.cp_size) * hd
        rounds = max(1, len(getattr(model, "reads", [])) or 1)
        slot = batch * length * C * 2
        return (4 + 4 * rounds) * slot + (16 << 20)

    def attach_fused(self, device, nbytes: int = 0) -> bool:
        """Attach the NVLink-fused Ulysses exchange (CUDA, CP > 1; collective).

        ``nbytes``: heap size per rank (``fused_heap_bytes``; default 512 MB or
        ``EB200_HEAP_BYTES``). Disabled with ``EB200_FUSED_ULYSSES=0`` (the NCCL
        path is then used).
        """
        if self.cp_size == 1 or self.ulysses is not None:
            return self.ulysses is not None
        if torch.device(device).type != "cuda" or os.environ.get("EB200_FUSED_ULYSSES", "1") == "0":
            return False
        from .ulysses import UlyssesFused
        self.ulysses = UlyssesFused(self.cp_group, self.cp_rank, self.cp_size, device, nbytes)
        return True

    def begin_step(self) -> None:
        """Start of a micro-step: recycle the fused exchange's buffers."""
        if self.ulysses is not None:
            self.ulysses.begin_step()

    def fused(self, x, heads, head_dim):
        """The fused exchange when it applies to ``x`` (same answer on every rank)."""
        if self.ulysses is not None and self.ulysses.usable(x, heads, head_dim):
            return self.ulysses
        return None

    def close(self) -> None:
        if self.ulysses is not None:
            self.ulysses.close()
            self.ulysses = None

    def shard(self, tensor, block_size, value=0):
        """``[B, N, ...]`` -> this rank's equal, block-aligned slice (tail padded with ``value``)."""
        n = tensor.shape[1]
        quantum = block_size * self.cp_size
        length = -(-n // quantum) * block_size
        start = self.cp_rank * length
        local = tensor[:, start:min(start + length, n)]
        if local.shape[1] < length:
            fill = tensor.new_full((tensor.shape[0], length - local.shape[1], *tensor.shape[2:]), value)
            local = torch.cat((local, fill), 1)
        return local.contiguous(), start

    def halo(self, x, block_size):
        if self.cp_size == 1:
            return None
        return _Halo.apply(x[:, -block_size:], self.cp_group)

    def to_heads(self, x):
        if self.cp_size == 1:
            return x
        if x.shape[2] % self.cp_size:
            raise ValueError("heads must be divisible by context_parallel")
        if self.ulysses is not None and x.is_cuda:
            return self.ulysses.to_heads(x)
        return _Ulysses.apply(x, self.cp_group, True)

    def to_sequence(self, x):
        if self.cp_size == 1:
            return x
        if self.ulysses is not None and x.is_cuda:
            return self.ulysses.to_sequence(x)
        return _Ulysses.apply(x, self.cp_group, False)

    def gather_positions(self, positions):
        if self.cp_size == 1:
            return positions
        parts = [torch.empty_like(positions) for _ in range(self.cp_size)]
        dist.all_gather(parts, positions.contiguous(), group=self.cp_group)
        return torch.cat(parts, 1)

    def max_query_count(self, count, device):
        if self.cp_size == 1:
            return max(1, count)
        value = torch.tensor(count, device=device, dtype=torch.long)
        dist.all_reduce(value, op=dist.ReduceOp.MAX, group=self.cp_group)
        return max(1, int(value))


def sum_all(value):
    """Detached sum over every rank (identity without a process group)."""
    result = value.detach().clone()
    if dist.is_initialized():
        dist.all_reduce(result)
    return result
