"""Loop oracles: deliberately naive per-row implementations of the read ops.

They share no code with :mod:`exploration_b200.ops` and are used by the test
suite and the ``validate`` tool (reference oracle: tests/test_attention.py:11-44).
"""
from __future__ import annotations

import math

import torch


def eager_attention(q, k, v, positions, block_size, topk=None):
    """Gated (``topk=None``) or top-k sparse attention, one (batch, query, head) at a time."""
    batch, queries, heads, dim = q.shape
    b = block_size
    rows = []
    for bi in range(batch):
        per_query = []
        for qi in range(queries):
            p = int(positions[bi, qi])
            per_head = []
            for h in range(heads):
                if p < 0:
                    # Zero output that still depends (with zero weight) on every input.
                    per_head.append(q[bi, qi, h] * 0 + k[bi, :, h].sum(0) * 0 + v[bi, :, h].sum(0) * 0)
                    continue
                logits = k[bi, :p + 1, h] @ q[bi, qi, h] / math.sqrt(dim)
                remote_blocks = max(0, p // b - 1)
                chosen = list(range(remote_blocks))
                gate = None
                if remote_blocks:
                    scores = logits[:remote_blocks * b].reshape(remote_blocks, b).logsumexp(-1)
                    gate = scores.log_softmax(0)
                    if topk is not None and topk < remote_blocks:
                        chosen = scores.topk(topk).indices.tolist()
                keys, parts = [], []
                for j in chosen:
                    keys.extend(range(j * b, (j + 1) * b))
                    parts.append(logits[j * b:(j + 1) * b] + gate[j])
                keys.extend(range(remote_blocks * b, p + 1))
                parts.append(logits[remote_blocks * b:p + 1])
                weights = torch.cat(parts).softmax(0)
                per_head.append(weights @ v[bi, keys, h])
            per_query.append(torch.stack(per_head))
        rows.append(torch.stack(per_query))
    return torch.stack(rows)


def error_metrics(actual, expected) -> dict:
    actual, expected = actual.detach().float(), expected.detach().float()
    diff = (actual - expected).abs()
    scale = expected.square().mean().sqrt().clamp_min(1e-8)
    return {"max_abs": float(diff.max()), "relative_rms": float(diff.square().mean().sqrt() / scale)}
