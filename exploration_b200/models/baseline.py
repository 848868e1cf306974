"""Dense causal Transformer baseline, parameter- and depth-matched to Stack.

Pre-norm causal attention with RoPE + FFN per block, a tied LM head, and the
same driver interface as :class:`StackModel` (reference:
st/models/baseline.py:22-158). ``--layers 3`` matches ``arch="Lx2,G"`` in
parameters (3 x 12 d^2 vs 24 d^2 local + 2 d^2 raw K/V + 10 d^2 read).

The baseline is the comparator, so its attention is PyTorch SDPA (the
reference's choice); its norms/FFN use the same fused ops as Stack.
"""
from __future__ import annotations

import math
from numbers import Integral

import torch
from torch import nn
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

from ..ops import fused
from ..ops.flash import flash_attention
from ..parallel.context import ParallelContext
from .blocks import FeedForward, RotaryEmbedding


class BaselineBlock(nn.Module):
    def __init__(self, dim, heads, rope, ffn_ratio, attention_backend="auto"):
        super().__init__()
        if attention_backend not in ("auto", "flash", "math"):
            raise ValueError("attention_backend must be auto, flash or math")
        self.heads, self.hd = heads, dim // heads
        self.rope = rope
        self.attention_backend = attention_backend
        self.attn_norm = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.out = nn.Linear(dim, dim, bias=False)
        self.ffn_norm = nn.LayerNorm(dim)
        self.ffn = FeedForward(dim, ffn_ratio)

    def _forward_impl(self, x, positions, parallel):
        parallel = parallel or ParallelContext()
        batch, n, dim = x.shape
        q, k, v = self.qkv(self.attn_norm(x)).reshape(batch, n, 3, self.heads, self.hd).unbind(2)
        q, k = self.rope(q, positions), self.rope(k, positions)
        q, k, v = (parallel.to_heads(t) for t in (q, k, v))
        ctx = flash_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                              is_causal=True, mode=self.attention_backend)
        ctx = parallel.to_sequence(ctx.transpose(1, 2)).reshape(batch, n, dim)
        y = x + self.out(ctx)
        return y + self.ffn(self.ffn_norm(y))

    def forward(self, x, positions, parallel=None, checkpoint_chunks=False):
        if checkpoint_chunks and torch.is_grad_enabled():
            return checkpoint(lambda h: self._forward_impl(h, positions, parallel), x,
                              use_reentrant=False, preserve_rng_state=False)
        return self._forward_impl(x, positions, parallel)


class BaselineModel(nn.Module):
    """``forward([B,N], sup=None) -> [B,N,vocab]`` with zero logits off ``sup``."""

    def __init__(self, vocab_size, dim=256, heads=4, layers=3, ffn_ratio=4, checkpoint_chunks=False,
                 loss_chunk=128, backend="auto"):
        super().__init__()
        for name, value in {"vocab_size": vocab_size, "dim": dim, "heads": heads,
                            "layers": layers}.items():
            if isinstance(value, bool) or not isinstance(value, Integral) or value < 1:
                raise ValueError(f"{name} must be a positive integer")
        if dim % heads or (dim // heads) % 2:
            raise ValueError("dim / heads must be an even integer for RoPE")
        if not math.isfinite(ffn_ratio) or ffn_ratio <= 0:
            raise ValueError("ffn_ratio must be finite and positive")
        if backend not in ("auto", "flash", "math"):
            raise ValueError("attention backend must be auto, flash or math")
        self.dim, self.heads, self.hd = dim, heads, dim // heads
        self.block_size = 1          # shard alignment only: no block semantics
        self.checkpoint_chunks, self.loss_chunk = checkpoint_chunks, loss_chunk
        self.attention_backend = backend
        self.embedding = nn.Embedding(vocab_size, dim)
        nn.init.normal_(self.embedding.weight, std=0.02)
        self.rope = RotaryEmbedding(self.hd)
        self.blocks = nn.ModuleList(BaselineBlock(dim, heads, self.rope, ffn_ratio, backend)
                                    for _ in range(layers))
        self.final_norm = nn.LayerNorm(dim)
        self.lm_head = nn.Linear(dim, vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight

    def encode(self, input_ids, parallel=None, offset=0):
        if input_ids.ndim != 2 or min(input_ids.shape) < 1:
            raise ValueError("input_ids must have nonempty shape [batch, sequence]")
        x = self.embedding(input_ids)
        positions = torch.arange(offset, offset + input_ids.shape[1], device=x.device)
        for block in self.blocks:
            x = block(x, positions, parallel, self.checkpoint_chunks)
        return x

    def iter_logits(self, input_ids, positions, parallel=None, offset=0):
        """Yield ``(slice, logits, None)`` per loss chunk of the requested positions."""
        x = self.encode(input_ids, parallel=parallel, offset=offset)
        rows = torch.arange(x.shape[0], device=x.device)[:, None]
        for lo in range(0, positions.shape[1], self.loss_chunk):
            sl = slice(lo, min(lo + self.loss_chunk, positions.shape[1]))
            yield sl, self.lm_head(self.final_norm(x[rows, positions[:, sl]])), None

    def forward_loss(self, input_ids, targets, sup=None, parallel=None, offset=0):
        if input_ids.shape != targets.shape:
            raise ValueError("input_ids and targets must have the same shape")
        if sup is not None and (sup.shape != targets.shape or sup.dtype != torch.bool):
            raise ValueError("sup must be bool [B,N]")
        valid = targets != -100
        if sup is not None:
            valid = valid & sup
        x = self.encode(input_ids, parallel, offset)
        where = valid.nonzero()
        # A rank with no supervised token still connects every parameter to
        # the loss, so its backward issues the same collectives as the others.
        loss = (x.sum() + self.final_norm.weight.sum() + self.final_norm.bias.sum()
                + self.lm_head.weight.sum()) * 0
        correct = torch.zeros((), device=x.device, dtype=torch.long)
        errors = torch.zeros(x.shape[0], device=x.device, dtype=torch.long)

        def head(hidden, labels):
            logits = self.lm_head(self.final_norm(hidden)).float()
            return F.cross_entropy(logits, labels, reduction="sum"), logits.argmax(-1).eq(labels)

        for lo in range(0, where.shape[0], self.loss_chunk):
            ix = where[lo:lo + self.loss_chunk]
            hidden, labels = x[ix[:, 0], ix[:, 1]], targets[ix[:, 0], ix[:, 1]]
            if self.checkpoint_chunks and torch.is_grad_enabled():
                part, hit = checkpoint(head, hidden, labels, use_reentrant=False,
                                       preserve_rng_state=False)
            else:
                part, hit = head(hidden, labels)
            loss = loss + part
            correct += hit.detach().sum()
            errors.scatter_add_(0, ix[:, 0], (~hit.detach()).long())
        return {"loss_sum": loss, "count": valid.sum(), "correct": correct, "row_errors": errors}

    def forward(self, input_ids, sup=None, *, targets=None, parallel=None, offset=0, compact=False):
        if targets is not None:
            return self.forward_loss(input_ids, targets, sup, parallel, offset)
        x = self.encode(input_ids, parallel, offset)
        if compact and sup is not None:
            counts = sup.sum(1)
            if int(counts.min()) < 1 or not bool((counts == counts[0]).all()):
                raise ValueError("compact logits require equal positive query counts per row")
            x = x[sup].reshape(input_ids.shape[0], int(counts[0]), self.dim)
        logits = self.lm_head(self.final_norm(x))
        if sup is not None and not compact:
            logits = logits * sup.unsqueeze(-1)
        return logits
