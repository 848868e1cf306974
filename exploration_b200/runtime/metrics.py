"""Streaming evaluation metrics.

Long-context evaluation produces logits one query chunk at a time and must
never concatenate them. ``MetricAccumulator`` folds each chunk into running
sums: cross-entropy, argmax hits, per-row error counts and optional
absolute-position buckets (reference: st/runtime/metrics.py:47-117).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
from torch.nn import functional as F

_LN2 = math.log(2.0)


def tail_mask(shape_or_targets, tail_tokens: int) -> torch.Tensor:
    """Boolean ``[B, N]`` mask that supervises only the last ``tail_tokens`` columns."""
    has_shape = hasattr(shape_or_targets, "shape")
    shape = tuple(shape_or_targets.shape) if has_shape else tuple(shape_or_targets)
    if len(shape) != 2 or tail_tokens < 1:
        raise ValueError("tail supervision needs a [batch, length] shape and tail_tokens >= 1")
    device = shape_or_targets.device if has_shape else None
    mask = torch.zeros(shape, dtype=torch.bool, device=device)
    mask[:, max(0, shape[1] - int(tail_tokens)):] = True
    return mask


def default_bucket_edges(length: int, count: int = 4) -> tuple:
    if length < 1 or count < 1:
        raise ValueError("length and bucket count must be positive")
    inner = [round(length * i / count) for i in range(1, count)]
    return tuple(int(x) for x in sorted(set([0, length, *inner])))


def parse_bucket_edges(spec, length: int) -> tuple:
    """``'0,1024,4096'`` -> edges; ``None``/``''``/``'auto'`` -> four even buckets."""
    if spec in (None, "", "auto"):
        return default_bucket_edges(length)
    try:
        edges = tuple(int(tok.strip()) for tok in str(spec).split(",") if tok.strip())
    except ValueError as exc:
        raise ValueError("metric buckets must be comma-separated integers") from exc
    ordered = all(a < b for a, b in zip(edges, edges[1:]))
    if len(edges) < 2 or edges[0] != 0 or edges[-1] != length or not ordered:
        raise ValueError("metric buckets must increase from 0 to the evaluated length")
    return edges


def _summary(loss_sum: float, count: int, correct: int) -> dict:
    loss = loss_sum / count
    return {"loss": loss, "bpc": loss / _LN2, "ppl": math.exp(min(loss, 80.0)),
            "accuracy": correct / count}


@dataclass
class MetricAccumulator:
    bucket_edges: tuple | None = None
    loss_sum: float = 0.0
    count: int = 0
    correct: int = 0
    row_errors: torch.Tensor | None = None
    _bucket_loss: list = field(default_factory=list)
    _bucket_count: list = field(default_factory=list)
    _bucket_correct: list = field(default_factory=list)

    def start_rows(self, batch: int, device="cpu", track_rows: bool = True):
        self.row_errors = torch.zeros(batch, dtype=torch.long, device=device) if track_rows else None
        if self.bucket_edges is not None:
            slots = len(self.bucket_edges) - 1
            self._bucket_loss = [0.0] * slots
            self._bucket_count = [0] * slots
            self._bucket_correct = [0] * slots

    def update(self, logits: torch.Tensor, targets: torch.Tensor, positions: torch.Tensor | None = None):
        if logits.ndim != 3 or targets.shape != logits.shape[:2]:
            raise ValueError("expected logits [batch, queries, vocab] and targets [batch, queries]")
        token_loss = F.cross_entropy(logits.float().flatten(0, 1), targets.flatten(),
                                     reduction="none").view_as(targets)
        hits = logits.argmax(-1).eq(targets)
        self.loss_sum += float(token_loss.sum())
        self.count += targets.numel()
        self.correct += int(hits.sum())
        if self.row_errors is not None:
            self.row_errors += (~hits).sum(1).to(self.row_errors.device)
        if self.bucket_edges is None or positions is None:
            return
        if positions.shape != targets.shape:
            raise ValueError("positions must match targets for bucket metrics")
        inner = torch.tensor(self.bucket_edges[1:-1], device=positions.device)
        # right=True: every bucket is [lo, hi).
        slot = torch.bucketize(positions.contiguous(), inner, right=True)
        for i in range(len(self._bucket_count)):
            chosen = slot == i
            self._bucket_loss[i] += float(token_loss[chosen].sum())
            self._bucket_count[i] += int(chosen.sum())
            self._bucket_correct[i] += int(hits[chosen].sum())

    def finalize(self) -> dict:
        if self.count < 1:
            raise ValueError("cannot finalize metrics over zero tokens")
        result = _summary(self.loss_sum, self.count, self.correct)
        result["evaluated_tokens"] = self.count
        if self.row_errors is not None:
            result["exact"] = float((self.row_errors == 0).sum()) / max(1, self.row_errors.numel())
        if self.bucket_edges is not None:
            buckets = []
            for lo, hi, loss, count, correct in zip(self.bucket_edges, self.bucket_edges[1:],
                                                    self._bucket_loss, self._bucket_count,
                                                    self._bucket_correct):
                entry = {"start": lo, "end": hi, "count": count}
                if count:
                    entry.update(_summary(loss, count, correct))
                else:
                    entry.update({"loss": None, "bpc": None, "ppl": None, "accuracy": None})
                buckets.append(entry)
            result["buckets"] = buckets
        return result
