"""Fused building-block ops used by the models.

Each op has one definition and two executions: the torch composition below
(CPU, fp64 oracle tests, ``backend="torch"``) and an sm_100a kernel of the
extension for CUDA tensors (``csrc/fused``, ``csrc/attention/local_halo.cu``).

Mixed precision follows the reference's autocast contract
(st/runtime/engine.py:166): parameters stay fp32, matmuls and attention run
in the autocast dtype, norms and softmax statistics accumulate in fp32 and
the residual stream keeps the dtype of the embedding (fp32). The native ops
read the autocast state themselves, so the models never call
``torch.autocast`` casts on the hot path: weights are cast once per
optimizer step (:func:`cast_param`) instead of once per use.
"""
from __future__ import annotations

import math
import weakref

import torch
from torch.nn import functional as F

from . import _native, gemm
from .launch import record

# ----------------------------------------------------------------------------
# precision helpers
# ----------------------------------------------------------------------------


def compute_dtype(x: torch.Tensor, param_dtype: torch.dtype) -> torch.dtype:
    """Dtype matmuls run in for ``x``: the autocast dtype if active, else the params'."""
    if torch.is_autocast_enabled(x.device.type):
        return torch.get_autocast_dtype(x.device.type)
    return param_dtype


def use_native(x: torch.Tensor, backend: str, cdt: torch.dtype) -> bool:
    return x.is_cuda and backend != "torch" and cdt in (torch.bfloat16, torch.float32)


# id(param) -> (weak reference to param, {dtype: (param version, copy)}). Tensors
# define elementwise ``==``, so they cannot be keys of a WeakKeyDictionary.
_cast_cache: dict = {}
_shadows: dict = {}


def register_shadow(param: torch.Tensor, shadow: torch.Tensor) -> None:
    """Use ``shadow`` (kept current by the optimizer) as ``param``'s low-precision copy."""
    key = id(param)
    _shadows[key] = (weakref.ref(param, lambda _ref, k=key: _shadows.pop(k, None)), shadow)


def clear_shadows() -> None:
    _shadows.clear()


def _cached_copy(param: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    key = id(param)
    shadow = _shadows.get(key)
    if shadow is not None and shadow[0]() is param and shadow[1].dtype == dtype:
        return shadow[1]
    entry = _cast_cache.get(key)
    if entry is None or entry[0]() is not param:
        entry = (weakref.ref(param, lambda _ref, k=key: _cast_cache.pop(k, None)), {})
        _cast_cache[key] = entry
    hit = entry[1].get(dtype)
    if hit is not None and hit[0] == param._version:
        return hit[1]
    value = param.detach().to(dtype)
    entry[1][dtype] = (param._version, value)
    return value


def cast_param(param: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Differentiable low-precision view of a parameter, cached per parameter version.

    The optimizer bumps ``param._version`` when it updates a weight, so a
    weight is converted once per step rather than at every use.
    """
    if param.dtype == dtype:
        return param
    if not torch.is_grad_enabled() or not param.requires_grad:
        return _cached_copy(param, dtype)
    return _CachedCast.apply(param, dtype)


class _CachedCast(torch.autograd.Function):
    @staticmethod
    def forward(ctx, param, dtype):
        ctx.src_dtype = param.dtype
        value = _cached_copy(param, dtype)
        return value.view_as(value)

    @staticmethod
    def backward(ctx, grad):
        return grad.to(ctx.src_dtype), None


def clear_cast_cache() -> None:
    _cast_cache.clear()


# ----------------------------------------------------------------------------
# LayerNorm
# ----------------------------------------------------------------------------


class ResidualLink:
    """Pairs the LayerNorm and the residual op that read one residual-stream tensor.

    ``x`` feeds both ``LayerNorm(x)`` (whose output leads, through the block,
    to the residual op's other input) and the residual op itself
    (``x + f(...)``), so autograd would add the two gradients of ``x`` in a
    separate pass. With a link the residual op's backward leaves its
    gradient here instead of returning it, and the LayerNorm backward, which
    always runs later, adds it to ``dx`` inside the kernel. The LayerNorm
    arms the link in its forward; a residual op that finds the link unarmed
    (no native LayerNorm on the other branch) returns its gradient normally.
    """

    __slots__ = ("armed", "grad")

    def __init__(self):
        self.armed = False
        self.grad = None

    def take(self):
        grad, self.grad = self.grad, None
        return grad


def _sink_grad(param):
    """``param.grad`` if gradients of ``param`` are accumulated in place (a registered sink)."""
    return gemm._sink_target(param)


class _LayerNormNative(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps, out_dtype, link):
        ext = _native.native(x)
        flat = x.reshape(-1, x.shape[-1]).contiguous()
        y, mean, rstd = ext.layer_norm_fwd(flat, weight, bias, eps, out_dtype)
        record("layer_norm_fwd", width=x.shape[-1], in_dtype=str(x.dtype), out_dtype=str(out_dtype))
        ctx.save_for_backward(flat, weight, mean, rstd)
        ctx.params = (weight, bias)
        ctx.shape = x.shape
        ctx.link = link
        if link is not None:
            link.armed = True
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        flat, weight, mean, rstd = ctx.saved_tensors
        ext = _native.native(flat)
        dres = ctx.link.take() if ctx.link is not None else None
        if dres is not None:
            dres = dres.reshape(flat.shape)
            if dres.dtype != torch.float32 or not dres.is_contiguous():
                dres = dres.float().contiguous()
        w_acc, w_done = _sink_grad(ctx.params[0])
        b_acc, b_done = _sink_grad(ctx.params[1])
        if w_acc is None or b_acc is None:
            w_acc = b_acc = None
        dx, dw, db = ext.layer_norm_bwd(grad.reshape(flat.shape).contiguous(), flat, weight, mean, rstd,
                                        dres, w_acc, b_acc)
        if w_acc is not None:
            # Added into the parameters' gradients in place: report them complete.
            w_done(ctx.params[0])
            b_done(ctx.params[1])
            return dx.view(ctx.shape), None, None, None, None, None
        return dx.view(ctx.shape), dw, db, None, None, None


def _fp32(t):
    return t if t is None or t.dtype == torch.float32 else t.float()


def layer_norm(x, norm: torch.nn.LayerNorm, backend: str = "auto", link: ResidualLink | None = None):
    """``norm(x)``; on CUDA the output is already in the matmul dtype.

    ``link``: the residual op that also reads ``x`` (see :class:`ResidualLink`)."""
    cdt = compute_dtype(x, norm.weight.dtype)
    if use_native(x, backend, cdt) and x.dtype in (torch.float32, torch.bfloat16):
        # The kernels read fp32 affine parameters (a bf16-cast model passes copies).
        return _LayerNormNative.apply(x, _fp32(norm.weight), _fp32(norm.bias), norm.eps, cdt, link)
    return F.layer_norm(x, norm.normalized_shape, norm.weight, norm.bias, norm.eps)


# ----------------------------------------------------------------------------
# Linear / FFN
# ----------------------------------------------------------------------------


def linear(x, layer: torch.nn.Linear, backend: str = "auto", out_f32: bool = False):
    """``layer(x)`` (no-bias layers on the tcgen05 GEMM when native)."""
    cdt = compute_dtype(x, layer.weight.dtype)
    if use_native(x, backend, cdt):
        if cdt == torch.bfloat16 and layer.bias is None and gemm.usable(x.to(cdt), layer):
            return gemm.Linear.apply(x.to(cdt), layer.weight, out_f32)
        w = cast_param(layer.weight, cdt)
        b = None if layer.bias is None else cast_param(layer.bias, cdt)
        out = F.linear(x.to(cdt), w, b)
        return out.float() if out_f32 else out
    out = layer(x)
    return out.float() if out_f32 else out


def linear_residual(x, layer: torch.nn.Linear, residual, backend: str = "auto", link: ResidualLink | None = None):
    """``residual + layer(x)``; on the native path one GEMM whose epilogue adds the fp32 residual."""
    cdt = compute_dtype(x, layer.weight.dtype)
    if use_native(x, backend, cdt) and cdt == torch.bfloat16 and residual.dtype == torch.float32 \
            and gemm.usable(x.to(cdt), layer):
        return gemm.LinearResidual.apply(x.to(cdt), layer.weight, _fp32(layer.bias), residual, link)
    return residual + linear(x, layer, backend)


def ffn_residual(h, y, ffn: torch.nn.Sequential, backend: str = "auto", link: ResidualLink | None = None):
    """``y + ffn(h)``: two GEMMs with bias+GELU and bias+residual epilogues when native."""
    up, down = ffn[0], ffn[2]
    cdt = compute_dtype(h, up.weight.dtype)
    if use_native(h, backend, cdt) and cdt == torch.bfloat16 and y.dtype == torch.float32 \
            and gemm.usable(h.to(cdt), up, down):
        return gemm.FFNResidual.apply(h.to(cdt), y, up.weight, _fp32(up.bias), down.weight, _fp32(down.bias),
                                      link)
    return y + feed_forward(h, ffn, backend)


class _BiasGeluNative(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, bias):
        ext = _native.native(h)
        flat = h.reshape(-1, h.shape[-1]).contiguous()
        out = ext.bias_gelu_fwd(flat, bias)
        ctx.save_for_backward(flat, bias)
        ctx.shape = h.shape
        return out.view(h.shape)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        flat, bias = ctx.saved_tensors
        ext = _native.native(flat)
        dh, dbias = ext.bias_gelu_bwd(grad.reshape(flat.shape).contiguous(), flat, bias)
        return dh.view(ctx.shape), dbias


def feed_forward(x, ffn: torch.nn.Sequential, backend: str = "auto"):
    """``Linear -> GELU -> Linear``; on CUDA the bias and GELU run in one kernel."""
    up, act, down = ffn[0], ffn[1], ffn[2]
    cdt = compute_dtype(x, up.weight.dtype)
    if use_native(x, backend, cdt):
        w1 = cast_param(up.weight, cdt)
        h = torch.matmul(x.to(cdt), w1.t())
        u = _BiasGeluNative.apply(h, _fp32(up.bias))
        return F.linear(u, cast_param(down.weight, cdt), cast_param(down.bias, cdt))
    return down(act(up(x)))


# ----------------------------------------------------------------------------
# Local halo window attention with rotary embedding
# ----------------------------------------------------------------------------


def rope_tables(head_dim: int, offsets: torch.Tensor, base: float = 10_000.0):
    """fp32 ``cos``/``sin`` of split-half RoPE at integer ``offsets``."""
    index = torch.arange(0, head_dim, 2, device=offsets.device, dtype=torch.float32)
    inv = base ** (-index / head_dim)
    angles = offsets.to(torch.float32)[:, None] * inv
    return angles.cos(), angles.sin()


def apply_rope(x, cos, sin):
    """Rotate ``x [..., T, H, D]`` by per-row tables ``[T, D/2]`` (split-half pairs)."""
    cos = cos[:, None, :].to(x.dtype)
    sin = sin[:, None, :].to(x.dtype)
    first, second = x.chunk(2, dim=-1)
    return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


def local_attention_reference(qkv, qkv_prev, start, valid_start, n, block, heads):
    """Torch composition of windowed attention over ``[previous block, block]``.

    ``qkv [B, n, 3, H, D]`` covers one chunk starting at absolute position
    ``start`` (block aligned), ``qkv_prev [B, b, 3, H, D]`` is the halo block
    (``None``: masked). Query row ``r`` of block ``g`` sees window column
    ``c`` (0..2b-1: the previous block, then its own) when ``c <= b + r`` and
    the key's absolute position ``start + (g-1)*b + c`` lies in
    ``[valid_start, start + n)``. RoPE is applied relative to the query block
    origin (q at ``r``, keys at ``c - b``), which keeps every rotation exact at
    any absolute position. Returns ``[B, n, H*D]``.
    """
    batch = qkv.shape[0]
    b = block
    groups = -(-n // b)
    dim = qkv.shape[-1]
    pad = groups * b - n
    if pad:
        qkv = torch.nn.functional.pad(qkv, (0, 0, 0, 0, 0, 0, 0, pad))
    if qkv_prev is None:
        qkv_prev = torch.zeros_like(qkv[:, :b])
    full = torch.cat((qkv_prev, qkv), 1).unflatten(1, (groups + 1, b))     # [B,G+1,b,3,H,D]
    q, k, v = full[:, 1:, :, 0], full[..., 1, :, :], full[..., 2, :, :]
    kw = torch.cat((k[:, :-1], k[:, 1:]), 2)                              # [B,G,2b,H,D]
    vw = torch.cat((v[:, :-1], v[:, 1:]), 2)
    cos_q, sin_q = rope_tables(dim, torch.arange(b, device=qkv.device))
    cos_k, sin_k = rope_tables(dim, torch.arange(-b, b, device=qkv.device))
    q = apply_rope(q, cos_q, sin_q)
    kw = apply_rope(kw, cos_k, sin_k)
    rows = torch.arange(b, device=qkv.device)
    cols = torch.arange(2 * b, device=qkv.device)
    causal = cols[None, :] <= b + rows[:, None]
    key_pos = start + (torch.arange(groups, device=qkv.device)[:, None, None] - 1) * b + cols
    mask = causal[None] & (key_pos >= valid_start) & (key_pos < start + n)   # [G,b,2b]
    qh = q.permute(0, 1, 3, 2, 4).flatten(0, 1)                              # [B*G,H,b,D]
    kh = kw.permute(0, 1, 3, 2, 4).flatten(0, 1)
    vh = vw.permute(0, 1, 3, 2, 4).flatten(0, 1)
    m = mask[None].expand(batch, -1, -1, -1).flatten(0, 1)[:, None]
    ctx = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=m)
    ctx = ctx.unflatten(0, (batch, groups)).permute(0, 1, 3, 2, 4)
    return ctx.reshape(batch, groups * b, heads * dim)[:, :n]


class _LocalAttentionNative(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qkv_prev, start, valid_start, n, block):
        ext = _native.native(qkv)
        qkv = qkv.contiguous()
        prev = None if qkv_prev is None else qkv_prev.contiguous()
        if ext.local_tc_supported(qkv, block):
            out, lse = ext.local_tc_fwd(qkv, prev, start, valid_start, n)
            record("local_attention_fwd", block=block, head_dim=qkv.shape[-1], dtype=str(qkv.dtype), path="tcgen05")
        else:
            out, lse = ext.local_attention_fwd(qkv, prev, start, valid_start, n, block)
            record("local_attention_fwd", block=block, head_dim=qkv.shape[-1], dtype=str(qkv.dtype))
        ctx.save_for_backward(qkv, prev if prev is not None else qkv.new_empty(0), out, lse)
        ctx.has_prev = prev is not None
        ctx.meta = (start, valid_start, n, block)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        qkv, prev, out, lse = ctx.saved_tensors
        ext = _native.native(qkv)
        start, valid_start, n, block = ctx.meta
        if ext.local_tc_supported(qkv, block) and grad.dtype == torch.bfloat16:
            dqkv, dprev = ext.local_tc_bwd(grad.contiguous(), qkv, prev if ctx.has_prev else None,
                                           out, lse, start, valid_start, n)
        else:
            dqkv, dprev = ext.local_attention_bwd(grad.contiguous(), qkv, prev if ctx.has_prev else None,
                                                  out, lse, start, valid_start, n, block)
        return dqkv, (dprev if ctx.has_prev else None), None, None, None, None


def local_attention(qkv, qkv_prev, start, valid_start, n, block, heads, backend="auto"):
    """Windowed causal attention of one block-aligned chunk; returns ``[B, n, H*D]``."""
    if qkv.is_cuda and backend != "torch" and qkv.dtype in (torch.bfloat16, torch.float32):
        ext = _native.native(qkv)
        if ext.local_attention_supported(block, qkv.shape[-1]):
            return _LocalAttentionNative.apply(qkv, qkv_prev, start, valid_start, n, block)
    return local_attention_reference(qkv, qkv_prev, start, valid_start, n, block, heads)


# ----------------------------------------------------------------------------
# token embedding
# ----------------------------------------------------------------------------


class _EmbeddingNative(torch.autograd.Function):
    """Row lookup; the weight gradient comes from ``embedding_bwd`` (per-vocabulary-row
    sums in token order: deterministic, no sort of the ids)."""

    @staticmethod
    def forward(ctx, ids, weight):
        ctx.save_for_backward(ids)
        ctx.vocab = weight.shape[0]
        return F.embedding(ids, weight)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        (ids,) = ctx.saved_tensors
        ext = _native.native(grad)
        return None, ext.embedding_bwd(ids, grad.float(), ctx.vocab)


def embedding(ids, table: torch.nn.Embedding, backend: str = "auto"):
    """``table(ids)``; on the native path its weight gradient avoids PyTorch's sort-based backward."""
    w = table.weight
    if (ids.is_cuda and backend != "torch" and w.dtype == torch.float32 and w.requires_grad
            and w.shape[1] % 4 == 0 and table.padding_idx is None and torch.is_grad_enabled()):
        return _EmbeddingNative.apply(ids, w)
    return table(ids)


# ----------------------------------------------------------------------------
# LM head + cross entropy
# ----------------------------------------------------------------------------


class _CrossEntropyNative(torch.autograd.Function):
    """Summed CE over rows with ``-100`` ignored, plus argmax hits, in one pass.

    The gradient ``softmax - onehot`` is produced in the same pass as the
    loss and only scaled in backward.
    """

    @staticmethod
    def forward(ctx, logits, targets):
        ext = _native.native(logits)
        loss, hits, dlogits = ext.cross_entropy_fwd(logits.contiguous(), targets.contiguous())
        ctx.save_for_backward(dlogits)
        ctx.mark_non_differentiable(hits)
        return loss, hits

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_loss, _grad_hits):
        (dlogits,) = ctx.saved_tensors
        return dlogits * grad_loss, None


def cross_entropy_sum(logits, targets, backend="auto"):
    """``(sum CE, hits)`` with ``hits`` true for correct or ignored (-100) rows."""
    if logits.is_cuda and backend != "torch" and logits.dtype == torch.float32:
        loss, hits = _CrossEntropyNative.apply(logits.reshape(-1, logits.shape[-1]),
                                               targets.reshape(-1))
        return loss, hits.view(targets.shape)
    loss = F.cross_entropy(logits.flatten(0, -2), targets.flatten(), ignore_index=-100,
                           reduction="sum")
    hits = (logits.argmax(-1) == targets) | (targets == -100)
    return loss, hits


def gelu_reference(x):
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))
