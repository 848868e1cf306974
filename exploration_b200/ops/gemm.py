"""Linear layers on the persistent tcgen05 GEMM (``csrc/gemm/gemm_tc.cu``).

All three GEMMs of a layer run on the same kernel without transposing any
tensor: ``y = x W^T`` (both operands K-major), ``dx = dy W`` (W read
MN-major) and ``dW = dy^T x`` (both read MN-major, fp32 output for the fp32
master gradient). The fused layers keep elementwise work inside the GEMM
epilogues:

* ``linear_residual``: ``out = residual + x W^T (+ b)`` in fp32 (the residual
  stream update), one kernel instead of GEMM + add;
* ``ffn_residual``: ``out = y + W2 gelu(W1 h + b1) + b2``; the first GEMM
  applies bias + exact GELU and keeps the pre-activation for backward, the
  second adds bias and residual; backward fuses the GELU derivative (and the
  per-tile bias-gradient partial sums) into the ``dU = dOut W2`` epilogue.

Weights stay fp32 parameters (autograd accumulates their fp32 gradients);
the GEMMs read a bf16 copy refreshed once per optimizer step.
"""
from __future__ import annotations

import torch

from . import _native
from .launch import record

STORE_BF16, STORE_F32, ACCUM_F32, BIAS_GELU, BIAS_RESIDUAL, GELU_BACK = range(6)
TILE_M = 128


def _aligned(t: torch.Tensor) -> bool:
    return (t.dim() == 2 and t.stride(1) == 1 and (t.stride(0) * t.element_size()) % 16 == 0
            and t.data_ptr() % 16 == 0)


def supported(*tensors) -> bool:
    """bf16, 2-D, unit inner stride, 16-byte aligned rows (TMA requirements)."""
    return all(t.is_cuda and _aligned(t) for t in tensors)


def gemm(a, a_mn, b, b_mn, out, epilogue, alpha=1.0, bias=None, residual=None, aux=None, partial=None):
    ext = _native.native(a)
    ext.gemm(a, a_mn, b, b_mn, out, epilogue, alpha, bias, residual, aux, partial)
    record("gemm_tc", epilogue=epilogue, a_mn=a_mn, b_mn=b_mn)
    return out


def _bf16_weight(param):
    from .fused import _cached_copy
    return _cached_copy(param, torch.bfloat16)


def _flat(x):
    return x.reshape(-1, x.shape[-1]).contiguous()


class Linear(torch.autograd.Function):
    """``y = x W^T`` with bf16 (or fp32 for ``out_f32``) output; no bias."""

    @staticmethod
    def forward(ctx, x, weight, out_f32):
        x2 = _flat(x)
        w = _bf16_weight(weight)
        out = torch.empty(x2.shape[0], w.shape[0], device=x.device,
                          dtype=torch.float32 if out_f32 else torch.bfloat16)
        gemm(x2, False, w, False, out, STORE_F32 if out_f32 else STORE_BF16)
        ctx.save_for_backward(x2, w)
        ctx.shape = x.shape
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        g = _flat(dy).to(torch.bfloat16)
        dx = torch.empty_like(x2)
        gemm(g, False, w, True, dx, STORE_BF16)
        dw = torch.empty(w.shape, device=w.device, dtype=torch.float32)
        gemm(g, True, x2, True, dw, STORE_F32)
        return dx.view(ctx.shape), dw, None


class LinearResidual(torch.autograd.Function):
    """``out = residual + x W^T (+ bias)`` in fp32."""

    @staticmethod
    def forward(ctx, x, weight, bias, residual):
        x2 = _flat(x)
        w = _bf16_weight(weight)
        res = residual.reshape(-1, residual.shape[-1]).contiguous()
        out = torch.empty(res.shape, device=x.device, dtype=torch.float32)
        gemm(x2, False, w, False, out, BIAS_RESIDUAL, bias=bias, residual=res)
        ctx.save_for_backward(x2, w)
        ctx.has_bias = bias is not None
        ctx.shape = x.shape
        return out.view(residual.shape)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dout):
        x2, w = ctx.saved_tensors
        d32 = _flat(dout)
        g = d32.to(torch.bfloat16)
        dx = torch.empty_like(x2)
        gemm(g, False, w, True, dx, STORE_BF16)
        dw = torch.empty(w.shape, device=w.device, dtype=torch.float32)
        gemm(g, True, x2, True, dw, STORE_F32)
        db = d32.sum(0) if ctx.has_bias else None
        return dx.view(ctx.shape), dw, db, dout


class FFNResidual(torch.autograd.Function):
    """``out = y + W2 gelu(W1 h + b1) + b2`` (fp32 out, bf16 GEMMs)."""

    @staticmethod
    def forward(ctx, h, y, w1, b1, w2, b2):
        h2 = _flat(h)
        y2 = y.reshape(-1, y.shape[-1]).contiguous()
        w1b, w2b = _bf16_weight(w1), _bf16_weight(w2)
        rows, hidden = h2.shape[0], w1b.shape[0]
        pre = torch.empty(rows, hidden, device=h.device, dtype=torch.bfloat16)
        u = torch.empty_like(pre)
        gemm(h2, False, w1b, False, u, BIAS_GELU, bias=b1, aux=pre)
        out = torch.empty(y2.shape, device=h.device, dtype=torch.float32)
        gemm(u, False, w2b, False, out, BIAS_RESIDUAL, bias=b2, residual=y2)
        ctx.save_for_backward(h2, pre, u, w1b, w2b)
        ctx.shape = h.shape
        return out.view(y.shape)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dout):
        h2, pre, u, w1b, w2b = ctx.saved_tensors
        d32 = _flat(dout)
        g = d32.to(torch.bfloat16)
        db2 = d32.sum(0)
        dw2 = torch.empty(w2b.shape, device=g.device, dtype=torch.float32)
        gemm(g, True, u, True, dw2, STORE_F32)
        dh_pre = torch.empty_like(pre)
        partial = torch.empty(-(-g.shape[0] // TILE_M), pre.shape[1], device=g.device, dtype=torch.float32)
        gemm(g, False, w2b, True, dh_pre, GELU_BACK, aux=pre, partial=partial)
        db1 = partial.sum(0)
        dw1 = torch.empty(w1b.shape, device=g.device, dtype=torch.float32)
        gemm(dh_pre, True, h2, True, dw1, STORE_F32)
        dh = torch.empty_like(h2)
        gemm(dh_pre, False, w1b, True, dh, STORE_BF16)
        return dh.view(ctx.shape), dout, dw1, db1, dw2, db2


def usable(x, *layers) -> bool:
    """The fused GEMM path needs bf16 activations and TMA-aligned weight rows."""
    if not (x.is_cuda and x.dtype == torch.bfloat16):
        return False
    for layer in layers:
        k = layer.weight.shape[1]
        n = layer.weight.shape[0]
        if (k * 2) % 16 or (n * 2) % 16 or (x.shape[-1] * 2) % 16:
            return False
    return True
