"""Building blocks of the Stack model: rotary embedding, FFN, the local halo
encoder block and the raw K/V projection.

Parameter names and shapes match the reference modules
(st/models/blocks.py:76-207) so state dicts load across frameworks.

Execution: every block runs through :mod:`exploration_b200.ops.fused`, so
CUDA tensors take the sm_100a kernels (fused LayerNorm, bias+GELU, the local
window attention with RoPE applied inside the kernel) and CPU tensors the
torch composition. Long inputs are streamed in block-aligned chunks; chunk
size never changes values (tests pin this), it only bounds peak memory. On
CUDA the chunk is at least ``NATIVE_MIN_CHUNK`` tokens, because a B200 holds
the activations of a whole 64k-token shard and larger GEMMs run closer to
peak.
"""
from __future__ import annotations

import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

from ..ops import fused

NATIVE_MIN_CHUNK = 16384


def _gather_heads(source, indices):
    """``source [B,H,S,D]``, ``indices [B,H,G,K]`` -> ``[B,H,G,K,D]`` gathered along S."""
    dim = source.shape[-1]
    expanded = source.unsqueeze(3).expand(-1, -1, -1, indices.shape[3], -1)
    return expanded.gather(2, indices.unsqueeze(-1).expand(-1, -1, -1, -1, dim))


class RotaryEmbedding(nn.Module):
    """Split-half RoPE with fp32 angles and an integer frequency index.

    The index is a non-persistent integer buffer, so casting the model to
    bf16 cannot round the frequencies (reference: st/models/blocks.py:76-93).
    """

    def __init__(self, head_dim: int, base: float = 10_000.0):
        super().__init__()
        self.head_dim, self.base = head_dim, base
        self.register_buffer("frequency_index", torch.arange(0, head_dim, 2), persistent=False)

    def tables(self, positions):
        with torch.autocast(device_type=positions.device.type, enabled=False):
            inv = self.base ** (-self.frequency_index.float() / self.head_dim)
            angles = positions.float().unsqueeze(-1) * inv
            return angles.cos(), angles.sin()

    def forward(self, x, positions):
        """Rotate ``x [..., H, D]``; ``positions`` broadcasts over the axes before H."""
        cos, sin = self.tables(positions)
        cos, sin = cos.unsqueeze(-2).to(x.dtype), sin.unsqueeze(-2).to(x.dtype)
        first, second = x.chunk(2, dim=-1)
        return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


class FeedForward(nn.Sequential):
    """``Linear(d, r*d) -> GELU -> Linear(r*d, d)`` (indices 0 and 2 hold weights)."""

    def __init__(self, dim: int, ratio: float):
        hidden = max(1, round(dim * ratio))
        super().__init__(nn.Linear(dim, hidden), nn.GELU(), nn.Linear(hidden, dim))


class HaloMemoryBlock(nn.Module):
    """Pre-norm causal attention over ``[previous block, current block]`` + FFN."""

    def __init__(self, dim, heads, block_size, rope, ffn_ratio, query_chunk_size,
                 checkpoint_chunks=False, backend="auto"):
        super().__init__()
        self.heads, self.hd = heads, dim // heads
        self.block_size, self.query_chunk_size = block_size, query_chunk_size
        self.rope = rope
        self.checkpoint_chunks = checkpoint_chunks
        self.backend = backend
        self.attn_norm = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.out = nn.Linear(dim, dim, bias=False)
        self.ffn_norm = nn.LayerNorm(dim)
        self.ffn = FeedForward(dim, ffn_ratio)

    def _project(self, x, link=None):
        return fused.linear(fused.layer_norm(x, self.attn_norm, self.backend, link), self.qkv, self.backend)

    def forward_chunk(self, x, previous=None, start=0):
        """Encode one block-aligned chunk given the previous layer-input block.

        ``previous`` is ``[B, b, dim]`` (the halo) or ``None`` for a sequence
        start, in which case the window's first half is masked. This is also
        the primitive for sequence-parallel halos and streamed prefill.
        """
        batch, n, dim = x.shape
        b = self.block_size
        if start % b:
            raise ValueError("halo chunk start must be block aligned")
        if previous is not None and tuple(previous.shape) != (batch, b, dim):
            raise ValueError("previous halo must contain exactly one block")
        valid_start = start if previous is None else max(0, start - b)
        # x and y each feed a LayerNorm and a residual add: the links let the
        # LayerNorm backward add the residual branch's gradient in its kernel.
        link_x, link_y = fused.ResidualLink(), fused.ResidualLink()
        qkv = self._project(x, link_x).view(batch, n, 3, self.heads, self.hd)
        halo = None if previous is None else \
            self._project(previous).view(batch, b, 3, self.heads, self.hd)
        context = fused.local_attention(qkv, halo, start, valid_start, n, b, self.heads, self.backend)
        y = fused.linear_residual(context, self.out, x, self.backend, link_x)
        return fused.ffn_residual(fused.layer_norm(y, self.ffn_norm, self.backend, link_y), y, self.ffn,
                                  self.backend, link_y)

    def chunk_tokens(self, x) -> int:
        step = self.query_chunk_size * self.block_size
        if x.is_cuda and self.backend != "torch":
            step = max(step, NATIVE_MIN_CHUNK // self.block_size * self.block_size)
        return step

    def forward(self, x, positions=None, previous=None, start=0):
        if positions is not None:
            start = int(positions[0])          # callers pass contiguous absolute positions
        b = self.block_size
        step = self.chunk_tokens(x)
        grad = torch.is_grad_enabled()
        parts = [] if grad else None
        result = None if grad else torch.empty_like(x)
        for lo in range(0, x.shape[1], step):
            hi = min(lo + step, x.shape[1])
            prev = previous if lo == 0 else x[:, lo - b:lo]
            if self.checkpoint_chunks and grad:
                y = checkpoint(self.forward_chunk, x[:, lo:hi], prev, start + lo,
                               use_reentrant=False, preserve_rng_state=False)
            else:
                y = self.forward_chunk(x[:, lo:hi], prev, start + lo)
            if grad:
                parts.append(y)
            else:
                result[:, lo:hi] = y
        if not grad:
            return result
        return parts[0] if len(parts) == 1 else torch.cat(parts, 1)


class KVProjection(nn.Module):
    """LayerNorm + Linear to ``(k, v)``, projected in token chunks."""

    def __init__(self, dim, heads, rope, use_rope=True, chunk_tokens=1 << 16, backend="auto"):
        super().__init__()
        self.heads, self.hd = heads, dim // heads
        self.norm = nn.LayerNorm(dim)
        self.proj = nn.Linear(dim, 2 * dim, bias=False)
        self.rope = rope
        self.use_rope = use_rope
        self.chunk_tokens = chunk_tokens
        self.backend = backend

    def forward(self, x, positions):
        n = x.shape[1]
        keys, values = [], []
        for lo in range(0, n, self.chunk_tokens):
            sl = slice(lo, lo + self.chunk_tokens)
            h = fused.layer_norm(x[:, sl], self.norm, self.backend)
            kv = fused.linear(h, self.proj, self.backend).view(x.shape[0], -1, 2, self.heads, self.hd)
            k, v = kv.unbind(2)
            if self.use_rope:
                k = self.rope(k, positions[sl])
            keys.append(k)
            values.append(v)
        if len(keys) == 1:
            return keys[0], values[0]
        return torch.cat(keys, 1), torch.cat(values, 1)
