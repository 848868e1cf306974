"""Exact block-gated dense attention: the training-time read operator.

``dense_attention(q, k, v, positions, block_size)`` with ``q [B,Q,H,D]``,
``k, v [B,N,H,D]`` and integer ``positions [B,Q]`` (``-1`` marks a padding
row, whose output is zero). See :mod:`.gated_reference` for the definition.

Two code paths, chosen by device, never by trial and error:

* CUDA tensors run the hand-written sm_100a kernels of the extension
  (``csrc/attention``): a tcgen05/TMEM/TMA kernel for bf16 with head_dim
  64 or 128, and an fp32-accumulating SIMT kernel for fp32 inputs and other
  head dims, which keeps IEEE fp32 accuracy (no TF32). dQ and dK/dV have
  separate owner kernels, so results are deterministic and atomic-free.
* CPU tensors (and ``backend="torch"``) run the bounded-memory torch
  reference, which is also the oracle.

Reference parity: st/ops/attention.py:148-176 (dispatch) and
st/ops/kernels/dense.py:32-239 (kernels K1-K4).
"""
from __future__ import annotations

import torch

from ..config import canonical_backend
from . import _native
from .gated_reference import gated_backward, gated_forward
from .launch import record

MAX_HEAD_DIM = 256
MAX_BLOCK = 128


def native_supported(q: torch.Tensor, block_size: int) -> bool:
    return (q.is_cuda and q.dtype in (torch.float32, torch.bfloat16)
            and 2 <= block_size <= MAX_BLOCK and block_size & (block_size - 1) == 0
            and q.shape[-1] <= MAX_HEAD_DIM and q.shape[-1] % 2 == 0)


class _ReferenceGated(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, positions, block_size, q_chunk, kv_chunk):
        out, rc, pr, zr, lse = gated_forward(q, k, v, positions, block_size, q_chunk, kv_chunk)
        ctx.save_for_backward(q, k, v, positions, out, rc, pr, zr, lse)
        ctx.config = (block_size, q_chunk, kv_chunk)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        q, k, v, positions, out, rc, pr, zr, lse = ctx.saved_tensors
        b, qc, kc = ctx.config
        dq, dk, dv = gated_backward(grad, q, k, v, positions, out, rc, pr, zr, lse, b, qc, kc)
        return dq, dk, dv, None, None, None, None


class _NativeGated(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, positions, block_size):
        ext = _native.native(q)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        pos = positions.to(torch.int32).contiguous()
        out, rc, pr, zr, lse = ext.gated_attention_fwd(q, k, v, pos, block_size)
        record("gated_attention_fwd", dtype=str(q.dtype), head_dim=q.shape[-1], block=block_size,
               path=ext.gated_attention_path(q, block_size))
        ctx.save_for_backward(q, k, v, pos, out, rc, pr, zr, lse)
        ctx.block_size = block_size
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        q, k, v, pos, out, rc, pr, zr, lse = ctx.saved_tensors
        ext = _native.native(q)
        dq, dk, dv = ext.gated_attention_bwd(grad.contiguous(), q, k, v, pos, out, rc, pr, zr, lse,
                                            ctx.block_size)
        return dq, dk, dv, None, None


def _check(q, k, v, positions, block_size, q_chunk, kv_chunk):
    if q.ndim != 4 or k.ndim != 4 or k.shape != v.shape or positions.shape != q.shape[:2]:
        raise ValueError("expected q[B,Q,H,D], k/v[B,N,H,D] and positions[B,Q]")
    if k.shape[0] != q.shape[0] or k.shape[2:] != q.shape[2:]:
        raise ValueError("query and key batch/head dimensions differ")
    if min(q.shape) < 1 or k.shape[1] < 1 or min(block_size, q_chunk, kv_chunk) < 1:
        raise ValueError("attention dimensions and tile sizes must be positive")


def dense_attention(q, k, v, positions, block_size, backend="auto", q_chunk=128, kv_chunk=4096):
    """Exact gated attention with first derivatives (no ``Q x N`` tensor is kept)."""
    _check(q, k, v, positions, block_size, q_chunk, kv_chunk)
    path = canonical_backend(backend)
    if path != "torch" and q.is_cuda:
        if native_supported(q, block_size) and q.dtype == k.dtype == v.dtype:
            return _NativeGated.apply(q, k, v, positions, block_size)
        if path == "cuda":
            raise ValueError("native gated attention needs matching fp32/bf16 q/k/v, head_dim "
                             f"<= {MAX_HEAD_DIM} (even) and a power-of-two block size <= {MAX_BLOCK}")
    elif path == "cuda":
        raise ValueError("the native backend runs on CUDA tensors")
    # Autograd Function bodies run outside autocast, so the reference
    # accumulates in fp32 (or fp64 for the oracle tests).
    with torch.autocast(q.device.type, enabled=False):
        return _ReferenceGated.apply(q, k, v, positions, block_size, q_chunk, kv_chunk)
