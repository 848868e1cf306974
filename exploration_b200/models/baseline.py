"""Dense causal Transformer: the comparator of the Stack model.

Same driver interface as :class:`StackModel` (``forward`` with or without
targets, ``iter_logits``, ``block_size``) and the same parameter names as the
reference's baseline (st/models/baseline.py:22-158), so checkpoints move
between the two frameworks: ``embedding``, ``blocks.i.{attn_norm, qkv, out,
ffn_norm, ffn.0, ffn.2}``, ``final_norm`` and ``lm_head`` (tied to the
embedding). Three layers match ``arch="Lx2,G"`` in parameters:
3 x 12 d^2 against 24 d^2 local + 2 d^2 raw K/V + 10 d^2 read.

A block is built from this package's fused layers, so on a B200 everything
except the attention itself runs on the native kernels:

* ``LayerNorm -> QKV``: the norm writes bf16 for the tcgen05 GEMM;
* rotary embedding on q and k, then causal attention through PyTorch's SDPA
  (the comparator keeps the library attention the reference uses);
* ``x + out(ctx)`` as one GEMM with a residual epilogue, then
  ``y + FFN(LayerNorm(y))`` as the two-GEMM bias+GELU / bias+residual pair.

Training reads the loss at every position of the shard with ``-100`` labels
where nothing is supervised, so every parameter and every collective of the
backward takes part on every rank whatever the mask (no data-dependent
compaction, no host synchronisation).
"""
from __future__ import annotations

import math
from numbers import Integral

import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

from ..ops import fused
from ..ops.flash import flash_attention
from ..parallel.context import ParallelContext
from .blocks import FeedForward, RotaryEmbedding
from .head import sliced_head_loss

ATTENTION_BACKENDS = ("auto", "flash", "math")
NATIVE_LOSS_SLICE = 65536       # positions per head slice on CUDA (vocab-sized fp32 logits per position)


def _check_sizes(vocab_size, dim, heads, layers, ffn_ratio, backend):
    for name, value in (("vocab_size", vocab_size), ("dim", dim), ("heads", heads), ("layers", layers)):
        if isinstance(value, bool) or not isinstance(value, Integral) or value < 1:
            raise ValueError(f"{name} must be a positive integer")
    if dim % heads or (dim // heads) % 2:
        raise ValueError("dim / heads must be an even integer for RoPE")
    if not math.isfinite(ffn_ratio) or ffn_ratio <= 0:
        raise ValueError("ffn_ratio must be finite and positive")
    if backend not in ATTENTION_BACKENDS:
        raise ValueError("attention backend must be auto, flash or math")


class BaselineBlock(nn.Module):
    """Pre-norm causal self-attention and FFN, both as residual updates."""

    def __init__(self, dim, heads, rope, ffn_ratio, attention_backend="auto"):
        super().__init__()
        if attention_backend not in ATTENTION_BACKENDS:
            raise ValueError("attention_backend must be auto, flash or math")
        self.heads, self.hd = heads, dim // heads
        self.rope = rope
        self.attention_backend = attention_backend
        self.attn_norm = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.out = nn.Linear(dim, dim, bias=False)
        self.ffn_norm = nn.LayerNorm(dim)
        self.ffn = FeedForward(dim, ffn_ratio)

    def context(self, x, positions, parallel):
        """Attention output in the sequence layout ``[B, N, D]``."""
        batch, n, dim = x.shape
        qkv = fused.linear(fused.layer_norm(x, self.attn_norm), self.qkv).view(batch, n, 3, self.heads, self.hd)
        q, k, v = qkv.unbind(2)
        q, k = self.rope(q, positions), self.rope(k, positions)
        # [B, N, H, d] -> this rank's heads over the whole sequence -> SDPA's [B, H, N, d].
        q, k, v = (parallel.to_heads(t).transpose(1, 2) for t in (q, k, v))
        ctx = flash_attention(q, k, v, is_causal=True, mode=self.attention_backend).transpose(1, 2)
        return parallel.to_sequence(ctx).reshape(batch, n, dim)

    def _residual_updates(self, x, positions, parallel):
        y = fused.linear_residual(self.context(x, positions, parallel), self.out, x)
        return fused.ffn_residual(fused.layer_norm(y, self.ffn_norm), y, self.ffn)

    def forward(self, x, positions, parallel=None, checkpoint_chunks=False):
        parallel = parallel or ParallelContext()
        if checkpoint_chunks and torch.is_grad_enabled():
            # The whole block is recomputed, so neither QKV nor the attention's
            # saved tensors stay alive across long layers.
            return checkpoint(self._residual_updates, x, positions, parallel, use_reentrant=False,
                              preserve_rng_state=False)
        return self._residual_updates(x, positions, parallel)


class BaselineModel(nn.Module):
    """``forward([B,N], sup=None) -> [B,N,vocab]`` with zero logits where ``sup`` is false."""

    def __init__(self, vocab_size, dim=256, heads=4, layers=3, ffn_ratio=4, checkpoint_chunks=False,
                 loss_chunk=128, backend="auto"):
        super().__init__()
        _check_sizes(vocab_size, dim, heads, layers, ffn_ratio, backend)
        self.dim, self.heads, self.hd = dim, heads, dim // heads
        self.block_size = 1          # sequence shards align to single tokens: no block semantics
        self.checkpoint_chunks, self.loss_chunk = checkpoint_chunks, loss_chunk
        self.attention_backend = backend
        self.embedding = nn.Embedding(vocab_size, dim)
        nn.init.normal_(self.embedding.weight, std=0.02)
        self.rope = RotaryEmbedding(self.hd)
        self.blocks = nn.ModuleList([BaselineBlock(dim, heads, self.rope, ffn_ratio, backend) for _ in range(layers)])
        self.final_norm = nn.LayerNorm(dim)
        self.lm_head = nn.Linear(dim, vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight

    def encode(self, input_ids, parallel=None, offset=0):
        """Residual stream ``[B, N, D]`` after every block (positions start at ``offset``)."""
        if input_ids.ndim != 2 or min(input_ids.shape) < 1:
            raise ValueError("input_ids must have nonempty shape [batch, sequence]")
        x = self.embedding(input_ids)
        positions = torch.arange(offset, offset + input_ids.shape[1], device=x.device)
        for block in self.blocks:
            x = block(x, positions, parallel, self.checkpoint_chunks)
        return x

    def _logits(self, x):
        return fused.linear(fused.layer_norm(x, self.final_norm), self.lm_head)

    def iter_logits(self, input_ids, positions, parallel=None, offset=0):
        """Encode once, then yield ``(slice, logits [B, s, V], None)`` for ``positions [B, S]``
        in slices of ``loss_chunk`` (the vocabulary projection stays bounded)."""
        x = self.encode(input_ids, parallel=parallel, offset=offset)
        picked = positions.to(x.device)
        for lo in range(0, picked.shape[1], self.loss_chunk):
            part = slice(lo, min(lo + self.loss_chunk, picked.shape[1]))
            rows = picked[:, part]
            yield part, self._logits(torch.gather(x, 1, rows[..., None].expand(-1, -1, x.shape[-1]))), None

    def forward_loss(self, input_ids, targets, sup=None, parallel=None, offset=0):
        if input_ids.shape != targets.shape:
            raise ValueError("input_ids and targets must have the same shape")
        if self.loss_chunk < 1:
            raise ValueError("loss_chunk must be positive")
        if sup is not None and (sup.shape != targets.shape or sup.dtype != torch.bool):
            raise ValueError("sup must be bool [B,N]")
        valid = targets != -100
        if sup is not None:
            valid &= sup
        labels = targets.masked_fill(~valid, -100)
        x = self.encode(input_ids, parallel, offset)
        native = x.is_cuda
        loss, hits = sliced_head_loss(x, labels, self.final_norm, self.lm_head,
                                      max(self.loss_chunk, NATIVE_LOSS_SLICE) if native else self.loss_chunk,
                                      recompute=self.checkpoint_chunks)
        return {"loss_sum": loss, "count": valid.sum(), "correct": (hits & valid).sum(),
                "row_errors": (~hits & valid).sum(1)}

    def forward(self, input_ids, sup=None, *, targets=None, parallel=None, offset=0, compact=False):
        if targets is not None:
            return self.forward_loss(input_ids, targets, sup, parallel, offset)
        x = self.encode(input_ids, parallel, offset)
        if sup is None:
            return self._logits(x)
        if not compact:
            return self._logits(x) * sup.unsqueeze(-1)
        counts = sup.sum(1)
        if int(counts.min()) < 1 or not bool((counts == counts[0]).all()):
            raise ValueError("compact logits require equal positive query counts per row")
        return self._logits(x[sup].view(input_ids.shape[0], int(counts[0]), self.dim))
