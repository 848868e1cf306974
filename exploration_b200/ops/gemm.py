"""Linear layers on the persistent tcgen05 GEMM (``csrc/gemm/gemm_tc.cu``).

The kernel reads either operand K-major or MN-major, so every GEMM of a
layer runs on it without a transpose copy: the forward ``y = x W^T``, the
input gradient ``dx = dy W`` (W read MN-major) and the weight gradient
``dW = dy^T x`` (both operands MN-major), which is added straight into the
fp32 gradient. Weight gradients have few output tiles and a long reduction
(the tokens), so the kernel splits K across CTAs there and one reduce kernel
sums the fp32 partials in a fixed order (deterministic). The fused layers
keep elementwise work inside the GEMM epilogues:

* ``linear_residual``: ``out = residual + x W^T (+ b)`` in fp32 (the residual
  stream update), one kernel instead of GEMM + add;
* ``ffn_residual``: ``out = y + W2 gelu(W1 h + b1) + b2``; the first GEMM
  applies bias + exact GELU and keeps ``gelu'`` of the pre-activation (bf16)
  for backward, the second adds bias and residual; backward multiplies by
  the kept derivative (and forms the per-tile bias-gradient partial sums) in
  the ``dU = dOut W2`` epilogue, so no erf is evaluated twice.

Weights stay fp32 parameters (autograd accumulates their fp32 gradients);
the GEMMs read a bf16 copy refreshed once per optimizer step.
"""
from __future__ import annotations

import weakref

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


# Tile shapes of the kernel (``shape=`` forces one; 0 lets the cost model choose).
AUTO, NARROW, WIDE, PAIR = range(4)      # -, 128 x 128, 128 x 256, 256 x 256 on a CTA pair


def gemm(a, a_mn, b, b_mn, out, epilogue, alpha=1.0, bias=None, residual=None, aux=None, partial=None,
         shape=AUTO):
    ext = _native.native(a)
    ext.gemm(a, a_mn, b, b_mn, out, epilogue, alpha, bias, residual, aux, partial, shape)
    record("gemm_tc", epilogue=epilogue, a_mn=a_mn, b_mn=b_mn)
    return out


def plain(a, a_mn, b, b_mn, out, accumulate=False, splits=0, shape=AUTO):
    """``out (+)= op(A) op(B)^T`` with no epilogue (split-K when the output has few tiles)."""
    ext = _native.native(a)
    used = ext.gemm_plain(a, a_mn, b, b_mn, out, accumulate, splits, shape)
    record("gemm_tc", epilogue="accumulate" if accumulate else "store", a_mn=a_mn, b_mn=b_mn, splits=used)
    return out


def forward(x2, w, out_f32=False):
    """``x W^T`` (x [T, K], W [N, K]), bf16 or fp32 output."""
    out = torch.empty(x2.shape[0], w.shape[0], device=x2.device,
                      dtype=torch.float32 if out_f32 else torch.bfloat16)
    return plain(x2, False, w, False, out)


def input_grad(g, w):
    """``dx = g W`` (g [T, N], W [N, K]; W read MN-major), bf16."""
    out = torch.empty(g.shape[0], w.shape[1], device=g.device, dtype=torch.bfloat16)
    return plain(g, False, w, True, out)


def weight_grad(g, x, out=None):
    """``dW = g^T x`` in fp32 (g [T, N], x [T, K]: both read MN-major); added into ``out`` when given."""
    if out is None:
        out = torch.empty(g.shape[1], x.shape[1], device=g.device, dtype=torch.float32)
        return plain(g, True, x, True, out)
    return plain(g, True, x, True, out, accumulate=True)


# id(param) -> (weak reference to param, callback). A registered parameter
# receives its weight gradient straight into ``param.grad`` (the GEMM adds
# into it, beta = 1) instead of through autograd's accumulation (a separate
# read-add-write pass over the gradient); the callback then reports the
# gradient complete, in place of a post-accumulate-grad hook.
_grad_sinks: dict = {}


def register_grad_sink(param, callback) -> None:
    key = id(param)
    _grad_sinks[key] = (weakref.ref(param, lambda _ref, k=key: _grad_sinks.pop(k, None)), callback)


def remove_grad_sink(param) -> None:
    _grad_sinks.pop(id(param), None)


def accumulate_weight_grad(param, g, x):
    """``dW = g^T x`` for ``param``: added into ``param.grad`` when it is a sink (returns
    ``None``), else returned for autograd to accumulate."""
    sink = _grad_sinks.get(id(param)) if param is not None else None
    if (sink is not None and sink[0]() is param and g.is_cuda and param.grad is not None
            and param.grad.dtype == torch.float32 and param.grad.is_contiguous()):
        weight_grad(g, x, out=param.grad.view(param.shape))
        sink[1](param)
        return None
    return weight_grad(g, x)


def _sink_target(param):
    """(param.grad, done callback) when ``param`` is a sink with an fp32 contiguous gradient."""
    sink = _grad_sinks.get(id(param)) if param is not None else None
    if sink is None or sink[0]() is not param:
        return None, None
    grad = param.grad
    if grad is None or grad.dtype != torch.float32 or not grad.is_contiguous():
        return None, None
    return grad, sink[1]


def cast_colsum(d32, bias):
    """``(d32 as bf16, column sums of d32)``: the bias gradient is added straight into
    ``bias.grad`` (returned as ``None``) when the bias is a sink."""
    ext = _native.native(d32)
    acc, done = _sink_target(bias)
    g, sums = ext.cast_colsum(d32, acc)
    if acc is not None:
        done(bias)
        return g, None
    return g, sums


def column_sum(partial, bias):
    """Column sums of fp32 partials, added into ``bias.grad`` when the bias is a sink."""
    ext = _native.native(partial)
    acc, done = _sink_target(bias)
    sums = ext.column_sum(partial, acc)
    if acc is not None:
        done(bias)
        return None
    return sums


def hand_residual(link, dout):
    """The residual input's gradient: left on the link for the paired LayerNorm, or returned."""
    if link is None:
        return dout
    link.grad = dout
    return None


def _bf16_weight(param):
    from .fused import _cached_copy
    return _cached_copy(param, torch.bfloat16)


def _flat(x):
    return x.reshape(-1, x.shape[-1]).contiguous()


class Linear(torch.autograd.Function):
    """``y = x W^T`` (bf16, or fp32 for ``out_f32``), no bias; fp32 weight gradient."""

    @staticmethod
    def forward(ctx, x, weight, out_f32):
        # No epilogue to fuse (fp32 output straight from the accumulator when
        # asked, e.g. for the logits).
        x2 = _flat(x)
        w = _bf16_weight(weight)
        out = forward(x2, w, out_f32)
        ctx.save_for_backward(x2, w)
        ctx.shape = x.shape
        ctx.param = weight
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        g = _flat(dy).to(torch.bfloat16)
        dx = input_grad(g, w)
        return dx.view(ctx.shape), accumulate_weight_grad(ctx.param, g, x2), None


class LinearResidual(torch.autograd.Function):
    """``out = residual + x W^T (+ bias)`` in fp32."""

    @staticmethod
    def forward(ctx, x, weight, bias, residual, link=None):
        x2 = _flat(x)
        w = _bf16_weight(weight)
        res = residual.reshape(-1, residual.shape[-1]).contiguous()
        out = torch.empty(res.shape, device=x.device, dtype=torch.float32)
        gemm(x2, False, w, False, out, BIAS_RESIDUAL, bias=bias, residual=res)
        ctx.save_for_backward(x2, w)
        ctx.param = weight
        ctx.bias = bias
        ctx.has_bias = bias is not None
        ctx.shape = x.shape
        ctx.link = link if link is not None and link.armed else None
        return out.view(residual.shape)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dout):
        x2, w = ctx.saved_tensors
        d32 = _flat(dout)
        if ctx.has_bias:
            g, db = cast_colsum(d32, ctx.bias)
        else:
            g, db = d32.to(torch.bfloat16), None
        dx = input_grad(g, w)
        dw = accumulate_weight_grad(ctx.param, g, x2)
        return dx.view(ctx.shape), dw, db, hand_residual(ctx.link, dout), None


class FFNResidual(torch.autograd.Function):
    """``out = y + W2 gelu(W1 h + b1) + b2`` (fp32 out, bf16 GEMMs)."""

    @staticmethod
    def forward(ctx, h, y, w1, b1, w2, b2, link=None):
        h2 = _flat(h)
        y2 = y.reshape(-1, y.shape[-1]).contiguous()
        w1b, w2b = _bf16_weight(w1), _bf16_weight(w2)
        rows, hidden = h2.shape[0], w1b.shape[0]
        dgelu = torch.empty(rows, hidden, device=h.device, dtype=torch.bfloat16)
        u = torch.empty_like(dgelu)
        gemm(h2, False, w1b, False, u, BIAS_GELU, bias=b1, aux=dgelu)
        out = torch.empty(y2.shape, device=h.device, dtype=torch.float32)
        gemm(u, False, w2b, False, out, BIAS_RESIDUAL, bias=b2, residual=y2)
        ctx.save_for_backward(h2, dgelu, u, w1b, w2b)
        ctx.params = (w1, w2)
        ctx.biases = (b1, b2)
        ctx.shape = h.shape
        ctx.link = link if link is not None and link.armed else None
        return out.view(y.shape)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dout):
        h2, dgelu, u, w1b, w2b = ctx.saved_tensors
        d32 = _flat(dout)
        g, db2 = cast_colsum(d32, ctx.biases[1])
        dw2 = accumulate_weight_grad(ctx.params[1], g, u)
        dh_pre = torch.empty_like(dgelu)
        partial = torch.empty(-(-g.shape[0] // TILE_M), dgelu.shape[1], device=g.device, dtype=torch.float32)
        gemm(g, False, w2b, True, dh_pre, GELU_BACK, aux=dgelu, partial=partial)
        db1 = column_sum(partial, ctx.biases[0])
        dw1 = accumulate_weight_grad(ctx.params[0], dh_pre, h2)
        dh = input_grad(dh_pre, w1b)
        return dh.view(ctx.shape), hand_residual(ctx.link, dout), dw1, db1, dw2, db2, None


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
