"""Evaluation metrics accumulated on the device while logits stream by.

Long-context evaluation yields logits one query chunk at a time. Each chunk is
folded into a small table of float64 sums that stays on the device where the
logits live: one row per absolute-position bucket (plus a row for the whole
evaluation) with columns (summed cross-entropy, token count, argmax hits), and
an optional per-row error count. A chunk costs a handful of kernels and no
host synchronisation; the table is read once, in :meth:`finalize`, which
reports loss, bits per character, perplexity, accuracy, exact match and the
per-bucket breakdown (the fields of st/runtime/metrics.py:47-117 in the
reference, whose accumulator reads every chunk back to the host).
"""
from __future__ import annotations

import math

import torch
from torch.nn import functional as F

_LOSS, _COUNT, _HITS = range(3)


def tail_mask(shape_or_targets, tail_tokens: int) -> torch.Tensor:
    """Boolean ``[B, N]`` mask that supervises only the last ``tail_tokens`` columns."""
    is_tensor = isinstance(shape_or_targets, torch.Tensor)
    shape = tuple(shape_or_targets.shape) if is_tensor else tuple(shape_or_targets)
    if len(shape) != 2 or tail_tokens < 1:
        raise ValueError("tail supervision needs a [batch, length] shape and tail_tokens >= 1")
    columns = torch.arange(shape[1], device=shape_or_targets.device if is_tensor else None)
    return (columns >= shape[1] - int(tail_tokens)).expand(shape).clone()


def default_bucket_edges(length: int, count: int = 4) -> tuple:
    """``count`` (about) equal position buckets over ``[0, length)``; duplicate edges collapse."""
    if length < 1 or count < 1:
        raise ValueError("length and bucket count must be positive")
    return tuple(sorted({0, length, *(round(length * i / count) for i in range(1, count))}))


def parse_bucket_edges(spec, length: int) -> tuple:
    """``'0,1024,4096'`` -> edges; ``None`` / ``''`` / ``'auto'`` -> four even buckets."""
    if spec in (None, "", "auto"):
        return default_bucket_edges(length)
    fields = [tok.strip() for tok in str(spec).split(",") if tok.strip()]
    if not all(tok.lstrip("-").isdigit() for tok in fields):
        raise ValueError("metric buckets must be comma-separated integers")
    edges = tuple(int(tok) for tok in fields)
    if len(edges) < 2 or edges[0] != 0 or edges[-1] != length or any(b <= a for a, b in zip(edges, edges[1:])):
        raise ValueError("metric buckets must increase from 0 to the evaluated length")
    return edges


def _rates(loss_sum: float, count: float, hits: float) -> dict:
    loss = loss_sum / count
    return {"loss": loss, "bpc": loss / math.log(2.0), "ppl": math.exp(min(loss, 80.0)), "accuracy": hits / count}


class MetricAccumulator:
    """Streaming token metrics with optional position buckets and per-row exact match."""

    def __init__(self, bucket_edges: tuple | None = None):
        self.bucket_edges = tuple(bucket_edges) if bucket_edges is not None else None
        self.table = None          # float64 [1 + buckets, 3] on the logits' device
        self.row_errors = None     # int64 [batch] when rows are tracked
        self._inner = None

    def start_rows(self, batch: int, device="cpu", track_rows: bool = True):
        """Reset; with ``track_rows`` count wrong predictions per row for exact match."""
        self.table = None
        self._inner = None
        self.row_errors = torch.zeros(batch, dtype=torch.long, device=device) if track_rows else None

    def _ensure(self, device):
        if self.table is None or self.table.device != device:
            slots = 1 + (len(self.bucket_edges) - 1 if self.bucket_edges is not None else 0)
            table = torch.zeros(slots, 3, dtype=torch.float64, device=device)
            if self.table is not None:
                table += self.table.to(device)
            self.table = table
            if self.bucket_edges is not None:
                self._inner = torch.tensor(self.bucket_edges[1:-1], device=device)

    def update(self, logits: torch.Tensor, targets: torch.Tensor, positions: torch.Tensor | None = None):
        """Fold one chunk: ``logits [B, Q, V]``, ``targets [B, Q]``, absolute ``positions [B, Q]``."""
        if logits.ndim != 3 or targets.shape != logits.shape[:2]:
            raise ValueError("expected logits [batch, queries, vocab] and targets [batch, queries]")
        if positions is not None and self.bucket_edges is not None and positions.shape != targets.shape:
            raise ValueError("positions must match targets for bucket metrics")
        self._ensure(logits.device)
        targets = targets.to(logits.device)
        token_loss = F.cross_entropy(logits.float().flatten(0, 1), targets.flatten(), reduction="none")
        hits = logits.argmax(-1).eq(targets)
        values = torch.stack((token_loss.double(), torch.ones_like(token_loss, dtype=torch.float64),
                              hits.flatten().double()), 1)
        self.table[0] += values.sum(0)
        if self.bucket_edges is not None and positions is not None:
            # right=True: bucket i covers [edge_i, edge_{i+1}).
            slot = torch.bucketize(positions.to(logits.device).flatten().contiguous(), self._inner, right=True)
            self.table.index_add_(0, slot + 1, values)
        if self.row_errors is not None:
            self.row_errors += (~hits).sum(1).to(self.row_errors.device)

    @property
    def count(self) -> int:
        return 0 if self.table is None else int(self.table[0, _COUNT])

    def finalize(self) -> dict:
        table = None if self.table is None else self.table.cpu().tolist()
        if not table or table[0][_COUNT] < 1:
            raise ValueError("cannot finalize metrics over zero tokens")
        total = table[0]
        result = _rates(total[_LOSS], total[_COUNT], total[_HITS])
        result["evaluated_tokens"] = int(total[_COUNT])
        if self.row_errors is not None:
            result["exact"] = float((self.row_errors == 0).sum()) / max(1, self.row_errors.numel())
        if self.bucket_edges is not None:
            buckets = []
            for (lo, hi), row in zip(zip(self.bucket_edges, self.bucket_edges[1:]), table[1:]):
                entry = {"start": lo, "end": hi, "count": int(row[_COUNT])}
                if row[_COUNT]:
                    entry.update(_rates(row[_LOSS], row[_COUNT], row[_HITS]))
                else:
                    entry.update(dict.fromkeys(("loss", "bpc", "ppl", "accuracy")))
                buckets.append(entry)
            result["buckets"] = buckets
        return result
