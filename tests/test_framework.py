"""Engine-level invariants on CPU: the training loss, unsupervised rows, inference tiers, CP shards."""
from pathlib import Path

import pytest
import torch
from torch.nn import functional as F

from exploration_b200.models.stack import StackModel
from exploration_b200.parallel.context import ParallelContext
from exploration_b200.runtime.inference import InferenceSession


def stack(**overrides):
    options = dict(vocab_size=29, dim=16, heads=2, block_size=4, topk=2, arch="Lx2,(G)x2", backend="torch",
                   pos_chunk=3, encoder_chunk=8)
    options.update(overrides)
    return StackModel(**options).double()


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(2024)


@pytest.mark.parametrize("recompute,loss_chunk", [(False, 128), (True, 128), (True, 1), (False, 5)])
def test_training_loss_equals_cross_entropy_of_the_logits(recompute, loss_chunk):
    """``forward_loss`` (dense read, sliced head, optional recomputation) against the logits path."""
    m = stack(topk=64, loss_chunk=loss_chunk, checkpoint_chunks=recompute)
    for layer in m.local:
        layer.checkpoint_chunks = recompute
    ids, targets = torch.randint(29, (2, 22)), torch.randint(29, (2, 22))
    sup = torch.rand(2, 22) > 0.3
    logits = m(ids)
    # The loss path reads fp32 logits (as on the native path), whatever the model's dtype.
    want = F.cross_entropy(logits[sup].float(), targets[sup], reduction="sum")
    got = m(ids, targets=targets, sup=sup)
    assert int(got["count"]) == int(sup.sum())
    assert int(got["correct"]) == int((logits.argmax(-1) == targets)[sup].sum())
    torch.testing.assert_close(got["loss_sum"], want, rtol=1e-6, atol=1e-5)
    params = [p for p in m.parameters() if p.requires_grad]
    for g, w in zip(torch.autograd.grad(got["loss_sum"], params, allow_unused=True),
                    torch.autograd.grad(want, params, allow_unused=True)):
        if w is not None:
            torch.testing.assert_close(g, w, rtol=1e-5, atol=1e-6)


def test_a_row_without_targets_trains_with_finite_gradients():
    m = stack(checkpoint_chunks=True)
    ids = torch.randint(29, (2, 15))
    targets = torch.full_like(ids, -100)
    targets[1, -3:] = torch.tensor([1, 2, 3])
    result = m(ids, targets=targets)
    assert int(result["count"]) == 3 and result["row_errors"][0] == 0
    result["loss_sum"].backward()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


@pytest.mark.parametrize("tier,page", [("cpu", 12), ("cpu", 1000), ("disk", 8), ("disk", 12)])
def test_paged_session_matches_the_in_core_forward(tmp_path, tier, page):
    m = stack().eval()
    ids = torch.randint(29, (2, 57))
    pos = torch.tensor([[0, 9, 30, 56], [3, 8, 44, 55]])
    sup = torch.zeros_like(ids, dtype=torch.bool).scatter_(1, pos, True)
    with torch.no_grad():
        want = m(ids, sup=sup, compact=True)
    with InferenceSession(m, cache=tier, cache_dir=str(tmp_path), page_tokens=page, encoder_chunk=8,
                          query_chunk=3) as session:
        session.prefill(ids, pos)
        got = torch.cat([logits for _, logits, _ in session.iter_logits()], 1)
    torch.testing.assert_close(got, want, rtol=1e-9, atol=1e-10)
    assert list(Path(tmp_path).iterdir()) == []           # the disk tier removes its files


def test_query_states_spill_to_a_file_when_over_budget(tmp_path):
    m = stack().eval()
    ids = torch.randint(29, (1, 41))
    pos = torch.tensor([[2, 19, 40]])
    with torch.no_grad():
        want = m(ids, sup=torch.zeros_like(ids, dtype=torch.bool).scatter_(1, pos, True), compact=True)
    session = InferenceSession(m, cache="cpu", cache_dir=str(tmp_path), encoder_chunk=8, max_query_states_mb=0)
    session.max_query_bytes = 8
    with session:
        session.prefill(ids, pos)
        got = torch.cat([logits for _, logits, _ in session.iter_logits()], 1)
    torch.testing.assert_close(got, want, rtol=1e-9, atol=1e-10)
    assert list(tmp_path.iterdir()) == []


@pytest.mark.parametrize("start", [4, 4096, 1 << 20, 3 << 25])
def test_local_layer_depends_on_relative_positions_only(start):
    layer = stack(arch="L").eval().local[0]
    x, previous = torch.randn(2, 12, 16, dtype=torch.float64), torch.randn(2, 4, 16, dtype=torch.float64)
    with torch.no_grad():
        assert torch.equal(layer(x, previous=previous, start=start), layer(x, previous=previous, start=8))


@pytest.mark.parametrize("length,cp,block", [(13, 4, 4), (64, 8, 4), (7, 2, 16), (100, 3, 2)])
def test_sequence_shards_tile_the_sequence(length, cp, block):
    x = torch.arange(length)[None].expand(2, -1)
    shards = [ParallelContext(cp_size=cp, cp_rank=r).shard(x, block, -100) for r in range(cp)]
    width = shards[0][0].shape[1]
    assert width % block == 0 and all(s.shape[1] == width for s, _ in shards)
    assert [offset for _, offset in shards] == [r * width for r in range(cp)]
    joined = torch.cat([s for s, _ in shards], 1)
    assert torch.equal(joined[:, :length], x) and bool((joined[:, length:] == -100).all())
