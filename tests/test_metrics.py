"""Streaming evaluation metrics: chunked accumulation equals one pass over all logits."""
import math

import pytest
import torch
from torch.nn import functional as F

from exploration_b200 import MetricAccumulator, parse_bucket_edges, tail_mask


def _one_pass(logits, targets, positions, edges):
    """Plain restatement over the concatenated logits."""
    loss = F.cross_entropy(logits.flatten(0, 1), targets.flatten(), reduction="none").view_as(targets)
    hits = logits.argmax(-1) == targets
    per_bucket = []
    for lo, hi in zip(edges, edges[1:]):
        sel = (positions >= lo) & (positions < hi)
        n = int(sel.sum())
        per_bucket.append((n, float(loss[sel].sum()) / n if n else None, float(hits[sel].sum()) / n if n else None))
    exact = float((~hits).sum(1).eq(0).double().mean())
    return float(loss.mean()), float(hits.double().mean()), per_bucket, exact


@pytest.mark.parametrize("chunk", [1, 3, 7, 16])
def test_chunked_updates_match_one_pass(chunk):
    g = torch.Generator().manual_seed(3)
    batch, queries, vocab, length = 3, 16, 11, 64
    logits = torch.randn(batch, queries, vocab, generator=g) * 3
    targets = torch.randint(vocab, (batch, queries), generator=g)
    targets[1] = logits[1].argmax(-1)                      # one row entirely right
    positions = torch.sort(torch.randint(length, (batch, queries), generator=g), 1).values
    edges = parse_bucket_edges("0,10,40,64", length)
    metric = MetricAccumulator(edges)
    metric.start_rows(batch)
    for lo in range(0, queries, chunk):
        sl = slice(lo, lo + chunk)
        metric.update(logits[:, sl], targets[:, sl], positions[:, sl])
    out = metric.finalize()
    loss, accuracy, buckets, exact = _one_pass(logits, targets, positions, edges)
    assert out["evaluated_tokens"] == batch * queries
    assert math.isclose(out["loss"], loss, rel_tol=1e-6)
    assert math.isclose(out["bpc"], loss / math.log(2), rel_tol=1e-6)
    assert math.isclose(out["ppl"], math.exp(loss), rel_tol=1e-6)
    assert math.isclose(out["accuracy"], accuracy)
    assert math.isclose(out["exact"], exact) and out["exact"] >= 1 / 3
    for got, (n, bucket_loss, bucket_acc) in zip(out["buckets"], buckets):
        assert got["count"] == n
        if n:
            assert math.isclose(got["loss"], bucket_loss, rel_tol=1e-6)
            assert math.isclose(got["accuracy"], bucket_acc)
        else:
            assert got["loss"] is None and got["accuracy"] is None


def test_no_rows_no_buckets_and_empty():
    metric = MetricAccumulator()
    metric.start_rows(0, track_rows=False)
    with pytest.raises(ValueError):
        metric.finalize()
    metric.update(torch.zeros(1, 2, 5), torch.tensor([[0, 4]]))
    out = metric.finalize()
    assert "exact" not in out and "buckets" not in out
    assert math.isclose(out["loss"], math.log(5), rel_tol=1e-6)
    with pytest.raises(ValueError):
        metric.update(torch.zeros(2, 5), torch.tensor([0, 1]))


def test_bucket_edges():
    assert parse_bucket_edges("auto", 8) == (0, 2, 4, 6, 8)
    assert parse_bucket_edges(None, 3) == (0, 1, 2, 3)
    assert parse_bucket_edges(" 0, 5 ,9", 9) == (0, 5, 9)
    for bad in ("1,9", "0,5", "0,5,5,9", "0,x,9", "0"):
        with pytest.raises(ValueError):
            parse_bucket_edges(bad, 9)


def test_tail_mask():
    mask = tail_mask((2, 5), 2)
    assert mask.dtype == torch.bool and mask.tolist() == [[False, False, False, True, True]] * 2
    assert bool(tail_mask(torch.zeros(1, 3), 10).all())
    with pytest.raises(ValueError):
        tail_mask((5,), 1)
