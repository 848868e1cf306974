"""Ulysses context parallelism fused with its projections over NVLink.

The reference exchanges sequence shards and head shards with NCCL
``all_to_all_single`` on permuted copies, before and after the projection
GEMMs (st/runtime/parallel.py:16-38,111-119; st/models/stack.py:196-213).
Here the exchange lives inside the GEMMs:

* ``project_to_heads``: ``h W^T`` in the sequence layout is never written;
  the GEMM epilogue stores every output tile straight into the owning rank's
  head-layout slot of the symmetric heap (peer stores), then one peer
  barrier publishes the slots. Used for the query projection (one part)
  and the raw K/V projection (two parts).
* ``heads_to_linear_residual``: the output projection (bias and fp32
  residual in its epilogue) over the sequence layout of the owners'
  head-layout slots. By default each remote row is pulled over NVLink once
  (``gather_rows``, 16-byte peer loads) and the tcgen05 GEMM reads the
  landed copy; ``EB200_ULYSSES_GATHER=fused`` reads the A tiles with TMA
  straight from peer memory inside the GEMM instead (see ``gather_mode``).

Backward is the mirror image: the gradient of a scatter is a gather and a
GEMM (``dx = dY W``) and the gradient of a gather is a scatter-GEMM
(``dctx = dOut W`` stored to the head owners). Weight gradients use the
landed sequence-layout activation as a plain local operand.

Every rank issues the same sequence of heap allocations and barriers (the
model runs the same layers on every rank), which keeps slot offsets
identical and the barrier epochs aligned.
"""
from __future__ import annotations

import os

import torch

from ..ops import gemm as G
from ..ops.fused import _cached_copy
from .symmetric import SymmetricHeap

TILE_M = 128


def _bf16(param):
    return _cached_copy(param, torch.bfloat16)


def gather_mode() -> str:
    """How the head -> sequence direction reads the owners' buffers.

    ``landed`` (default): ``gather_rows`` pulls every remote row over NVLink
    once into a local sequence-layout buffer (16-byte peer loads) and the
    tcgen05 GEMM reads it from there; the landed copy is kept for the weight
    gradient. ``fused`` (``EB200_ULYSSES_GATHER=fused``): the GEMM's TMA
    producer reads A tiles straight from the owners' buffers, which overlaps
    transfer and math inside one kernel but fetches each remote row once per
    output-column tile (N / 256 times).
    """
    return "fused" if os.environ.get("EB200_ULYSSES_GATHER", "landed") == "fused" else "landed"


class _ProjectToHeads(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, U, parts, heads_per_rank, head_dim):
        heap = U.heap
        batch, n_local, k = x.shape
        C = heads_per_rank * head_dim
        x2 = x.reshape(-1, k)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        w = _bf16(weight)
        slot = heap.alloc(parts * batch * n_local * U.world * C * 2)
        U.ext.gemm_scatter(x2, w, False, heap.peer_ptrs(slot), U.rank, parts, batch, n_local, C)
        heap.barrier()
        out = heap.tensor(slot, (parts, batch, n_local * U.world, heads_per_rank, head_dim))
        ctx.save_for_backward(x2, w)
        ctx.param = weight
        ctx.meta = (U, parts, batch, n_local, C, x.shape)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        x2, w = ctx.saved_tensors
        U, parts, batch, n_local, C, shape = ctx.meta
        heap = U.heap
        gslot = heap.alloc(grad.numel() * 2)
        heap.tensor(gslot, grad.shape).copy_(grad)
        heap.barrier()
        ptrs = heap.peer_ptrs(gslot)
        dx = torch.empty(batch * n_local, x2.shape[1], device=x2.device, dtype=torch.bfloat16)
        dy_seq = torch.empty(batch * n_local, parts * U.world * C, device=x2.device, dtype=torch.bfloat16)
        U.ext.gather_rows(ptrs, U.rank, parts, batch, n_local, C, dy_seq)
        # dx = dY_seq W  (W stored [parts*dim, K] = [K_red, N]: MN-major B)
        if gather_mode() == "fused":
            U.ext.gemm_gather(ptrs, U.rank, parts, batch, n_local, C, w, True, dx, G.STORE_BF16, None, None)
        else:
            G.plain(dy_seq, False, w, True, dx)
        dw = G.accumulate_weight_grad(ctx.param, dy_seq, x2)
        return dx.view(shape), dw, None, None, None, None


class _HeadsToLinearResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, heads, weight, bias, residual, U, link=None):
        heap = U.heap
        batch, n_total, hpr, hd = heads.shape
        n_local, C = n_total // U.world, hpr * hd
        slot = heap.alloc(heads.numel() * 2)
        heap.tensor(slot, heads.shape).copy_(heads)
        heap.barrier()
        w = _bf16(weight)
        res = residual.reshape(-1, residual.shape[-1])
        if not res.is_contiguous():
            res = res.contiguous()
        out = torch.empty(res.shape, device=res.device, dtype=torch.float32)
        ctx_seq = None
        if gather_mode() == "fused":
            U.ext.gemm_gather(heap.peer_ptrs(slot), U.rank, 1, batch, n_local, C, w, False, out,
                              G.BIAS_RESIDUAL, bias, res)
        else:
            # Each remote row crosses NVLink once; the landed copy also serves dW.
            ctx_seq = torch.empty(batch * n_local, U.world * C, device=res.device, dtype=torch.bfloat16)
            U.ext.gather_rows(heap.peer_ptrs(slot), U.rank, 1, batch, n_local, C, ctx_seq)
            G.gemm(ctx_seq, False, w, False, out, G.BIAS_RESIDUAL, bias=bias, residual=res)
        ctx.ctx_seq = ctx_seq
        ctx.save_for_backward(w)
        ctx.param = weight
        ctx.link = link if link is not None and link.armed else None
        ctx.meta = (U, slot, batch, n_local, hpr, hd, bias is not None)
        return out.view(residual.shape)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dout):
        (w,) = ctx.saved_tensors
        U, slot, batch, n_local, hpr, hd, has_bias = ctx.meta
        heap = U.heap
        C = hpr * hd
        d32 = dout.reshape(-1, dout.shape[-1])
        g = d32.to(torch.bfloat16)
        # dctx_seq = g W  (W stored [dout, dim] = [K_red, N]: MN-major B), stored to the head owners.
        gslot = heap.alloc(batch * n_local * U.world * C * 2)
        U.ext.gemm_scatter(g, w, True, heap.peer_ptrs(gslot), U.rank, 1, batch, n_local, C)
        heap.barrier()
        dheads = heap.tensor(gslot, (batch, n_local * U.world, hpr, hd))
        ctx_seq, ctx.ctx_seq = ctx.ctx_seq, None
        if ctx_seq is None:
            ctx_seq = torch.empty(batch * n_local, U.world * C, device=g.device, dtype=torch.bfloat16)
            U.ext.gather_rows(heap.peer_ptrs(slot), U.rank, 1, batch, n_local, C, ctx_seq)
        dw = G.accumulate_weight_grad(ctx.param, g, ctx_seq)
        db = d32.sum(0) if has_bias else None
        return dheads, dw, db, G.hand_residual(ctx.link, dout), None, None


class UlyssesFused:
    """Fused sequence<->head exchange for one CP group on CUDA."""

    def __init__(self, group, rank: int, world: int, device, nbytes: int = 0):
        self.heap = SymmetricHeap(group, device, nbytes)
        self.ext = self.heap.ext
        self.group, self.rank, self.world = group, rank, world

    def begin_step(self) -> None:
        """Recycle the heap arena (all ranks, between micro-steps)."""
        self.heap.reset()

    def usable(self, x: torch.Tensor, heads: int, head_dim: int) -> bool:
        """Same answer on every rank (depends only on shapes, dtype and config)."""
        if not (x.is_cuda and x.dtype == torch.bfloat16):
            return False
        if heads % self.world:
            return False
        C = heads // self.world * head_dim
        return C % 64 == 0 and x.shape[1] % TILE_M == 0 and (x.shape[-1] * 2) % 16 == 0

    def project_to_heads(self, x, weight, parts: int, heads: int, head_dim: int):
        """``x [B, n_local, K]`` -> ``[parts, B, world * n_local, heads / world, head_dim]``."""
        return _ProjectToHeads.apply(x, weight, self, parts, heads // self.world, head_dim)

    def heads_to_linear_residual(self, heads, layer, residual, link=None):
        """``residual + to_sequence(heads) W^T + b`` (fp32) for this rank's shard."""
        bias = layer.bias if layer.bias is None or layer.bias.dtype == torch.float32 else layer.bias.float()
        return _HeadsToLinearResidual.apply(heads, layer.weight, bias, residual, self, link)

    # Generic exchanges (no projection to fuse with) stay on the collective path.
    def to_heads(self, x):
        from .context import _Ulysses
        return _Ulysses.apply(x, self.group, True)

    def to_sequence(self, x):
        from .context import _Ulysses
        return _Ulysses.apply(x, self.group, False)

    def close(self) -> None:
        self.heap.close()
