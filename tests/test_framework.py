"""Engine-level invariants: chunked loss, unsupervised rows, streamed prefill tiers, CP shards."""
import copy
from pathlib import Path

import torch

from exploration_b200.models.stack import StackModel
from exploration_b200.parallel.context import ParallelContext
from exploration_b200.runtime.inference import InferenceSession


def make_model(**kw):
    args = dict(vocab_size=31, dim=16, heads=2, block_size=4, topk=2, arch="Lx2,(G)x2",
                backend="torch", pos_chunk=3, encoder_chunk=8)
    args.update(kw)
    return StackModel(**args).double()


def test_chunked_loss_and_parameter_gradients():
    torch.manual_seed(617)
    ref = make_model(topk=64)
    actual = copy.deepcopy(ref)
    actual.checkpoint_chunks = True
    for layer in actual.local:
        layer.checkpoint_chunks = True
    ids = torch.randint(31, (2, 21))
    targets = torch.randint(31, (2, 21))
    mask = torch.rand(2, 21) > 0.4
    expected = torch.nn.functional.cross_entropy(ref(ids)[mask].float(), targets[mask], reduction="sum")
    result = actual(ids, targets=targets, sup=mask)
    torch.testing.assert_close(result["loss_sum"], expected, atol=2e-5, rtol=1e-6)
    expected.backward()
    result["loss_sum"].backward()
    for (name, rp), (_, ap) in zip(ref.named_parameters(), actual.named_parameters()):
        if rp.grad is not None:
            torch.testing.assert_close(ap.grad, rp.grad, atol=3e-6, rtol=2e-5, msg=name)


def test_all_unsupervised_row_still_has_finite_gradients():
    torch.manual_seed(617)
    model = make_model(checkpoint_chunks=True)
    ids = torch.randint(31, (2, 13))
    targets = torch.full_like(ids, -100)
    targets[1, -2:] = 2
    result = model(ids, targets=targets)
    assert int(result["count"]) == 2
    result["loss_sum"].backward()
    assert all(torch.isfinite(p.grad).all() for p in model.parameters() if p.grad is not None)


def test_streamed_prefill_matches_in_core_and_cleans_disk(tmp_path):
    torch.manual_seed(617)
    model = make_model().eval()
    ids = torch.randint(31, (2, 53))
    pos = torch.tensor([[0, 7, 31, 52], [1, 8, 40, 51]])
    mask = torch.zeros_like(ids, dtype=torch.bool).scatter_(1, pos, True)
    with torch.no_grad():
        expected = model(ids, sup=mask, compact=True)
    for tier in ("cpu", "disk"):
        directory = tmp_path / tier
        directory.mkdir()
        with InferenceSession(model, cache=tier, cache_dir=str(directory), page_tokens=12,
                              encoder_chunk=8, query_chunk=2) as session:
            session.prefill(ids, pos)
            actual = torch.cat([logits for _, logits, _ in session.iter_logits()], 1)
            torch.testing.assert_close(actual, expected, atol=1e-10, rtol=1e-9)
        assert list(Path(directory).iterdir()) == []


def test_disk_query_states_when_over_budget(tmp_path):
    torch.manual_seed(5)
    model = make_model().eval()
    ids = torch.randint(31, (1, 40))
    pos = torch.tensor([[3, 17, 39]])
    mask = torch.zeros_like(ids, dtype=torch.bool).scatter_(1, pos, True)
    with torch.no_grad():
        expected = model(ids, sup=mask, compact=True)
    session = InferenceSession(model, cache="cpu", cache_dir=str(tmp_path), encoder_chunk=8,
                               max_query_states_mb=0)
    session.max_query_bytes = 8       # force the mapped-file query state tier
    with session:
        session.prefill(ids, pos)
        actual = torch.cat([logits for _, logits, _ in session.iter_logits()], 1)
    torch.testing.assert_close(actual, expected, atol=1e-10, rtol=1e-9)
    assert list(tmp_path.iterdir()) == []


def test_shifted_halo_has_no_long_position_aliasing():
    torch.manual_seed(617)
    layer = make_model(arch="L").eval().local[0]
    x = torch.randn(2, 12, 16, dtype=torch.float64)
    prev = torch.randn(2, 4, 16, dtype=torch.float64)
    with torch.no_grad():
        torch.testing.assert_close(layer(x, previous=prev, start=32 * 1024 * 1024),
                                   layer(x, previous=prev, start=4), atol=0, rtol=0)


def test_sequence_shards_cover_tail_and_preserve_targets():
    x = torch.arange(13)[None]
    parts = []
    for rank in range(4):
        local, offset = ParallelContext(cp_size=4, cp_rank=rank).shard(x, 4, -100)
        assert offset == rank * 4
        parts.append(local)
    joined = torch.cat(parts, 1)
    torch.testing.assert_close(joined[:, :13], x)
    assert bool((joined[:, 13:] == -100).all())
