"""Flat parameter storage and the flat trainer on one CPU process."""
import torch

from exploration_b200 import ExecutionConfig, ParallelContext, build_model
from exploration_b200.runtime.flat import FlatParameters
from tests.dist_workers import _flat_vs_eager


def test_flat_parameters_are_views():
    model = build_model({"model": "stack", "vocab_size": 256, "dim": 64, "heads": 4, "block_size": 8,
                         "topk": 4, "arch": "Lx1,G", "ffn_ratio": 2.0}, execution=ExecutionConfig(backend="torch"))
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    flat = FlatParameters(model, torch.device("cpu"), shards=4)
    assert flat.split % (64 * 4) == 0 and (flat.total - flat.split) % (64 * 4) == 0
    names = {id(p): n for n, p in model.named_parameters()}
    assert len(flat.params) == len(names)
    for p, off in zip(flat.params, flat.offsets):
        assert torch.equal(p, before[names[id(p)]])
        assert p.data_ptr() == flat.data[off:].data_ptr()
        assert p.grad.data_ptr() == flat.grad[off:].data_ptr()
        assert off % 64 == 0
        # fp32-read parameters (norms, biases, embeddings) sit before the split
        assert (off < flat.split) == (p.dim() < 2 or p is model.embedding.weight)
    flat.data.add_(1.0)
    assert all(torch.equal(p, before[n] + 1) for n, p in model.named_parameters())
    flat.release()


def test_flat_trainer_matches_eager_single_process():
    assert _flat_vs_eager(ParallelContext(), shard=False) == 1
