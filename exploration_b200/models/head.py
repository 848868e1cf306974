"""Tied LM head with cross-entropy, shared by the models' training losses.

The head is ``final LayerNorm -> lm_head (fp32 logits) -> cross-entropy``.
On the native path the LayerNorm writes bf16 straight into the tcgen05 GEMM
and the loss kernel reads fp32 logits, so ``[rows, vocab]`` logits exist one
slice at a time only. Labels of unsupervised positions are ``-100``; they add
nothing to the loss and count as hits, so callers mask hits with their own
validity to count correct and wrong predictions.
"""
from __future__ import annotations

import torch
from torch.utils.checkpoint import checkpoint

from ..ops import fused


def head_loss(hidden, labels, norm, lm_head, backend="auto"):
    """``(sum of CE over labels != -100, hits)`` for one slice ``hidden [B, S, D]``."""
    logits = fused.linear(fused.layer_norm(hidden, norm, backend), lm_head, backend, out_f32=True)
    return fused.cross_entropy_sum(logits, labels, backend)


def sliced_head_loss(x, labels, norm, lm_head, slice_len, backend="auto", recompute=False):
    """Loss over every position of ``x [B, N, D]`` in slices of ``slice_len`` positions.

    Returns ``(loss_sum, hits [B, N])``. With ``recompute`` each slice's
    logits are rebuilt in backward instead of being kept.
    """
    losses, hits = [], []
    for lo in range(0, x.shape[1], slice_len):
        hidden, part_labels = x[:, lo:lo + slice_len], labels[:, lo:lo + slice_len]
        if recompute and torch.is_grad_enabled():
            loss, hit = checkpoint(head_loss, hidden, part_labels, norm, lm_head, backend, use_reentrant=False,
                                   preserve_rng_state=False)
        else:
            loss, hit = head_loss(hidden, part_labels, norm, lm_head, backend)
        losses.append(loss)
        hits.append(hit.detach())
    total = losses[0] if len(losses) == 1 else torch.stack(losses).sum()
    return total, torch.cat(hits, 1)
