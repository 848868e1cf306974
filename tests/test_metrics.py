import math

import torch

from exploration_b200 import MetricAccumulator, parse_bucket_edges, tail_mask


def test_streaming_metrics_and_buckets():
    edges = parse_bucket_edges("0,2,4", 4)
    assert edges == (0, 2, 4)
    metric = MetricAccumulator(edges)
    metric.start_rows(2, track_rows=False)
    logits = torch.tensor([[[5., 0., 0.], [0., 5., 0.]], [[0., 5., 0.], [0., 0., 5.]]])
    metric.update(logits, torch.tensor([[0, 1], [1, 2]]), torch.tensor([[0, 1], [2, 3]]))
    out = metric.finalize()
    assert out["evaluated_tokens"] == 4 and out["accuracy"] == 1.0
    assert math.isclose(out["ppl"], math.exp(out["loss"]))
    assert [b["count"] for b in out["buckets"]] == [2, 2]


def test_row_errors_and_default_edges():
    metric = MetricAccumulator(parse_bucket_edges("auto", 8))
    metric.start_rows(2)
    logits = torch.zeros(2, 3, 4)
    logits[0, :, 1] = 1
    metric.update(logits, torch.tensor([[1, 1, 1], [1, 2, 1]]), torch.tensor([[0, 3, 7], [1, 2, 6]]))
    out = metric.finalize()
    assert out["exact"] == 0.5
    assert len(out["buckets"]) == 4


def test_tail_mask():
    assert tail_mask((2, 5), 2).tolist() == [[False, False, False, True, True]] * 2
