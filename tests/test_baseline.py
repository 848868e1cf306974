"""Dense baseline: causality, supervision zeroing, recomputation parity, parameter match."""
import copy

import pytest
import torch

from exploration_b200.models.baseline import BaselineModel
from exploration_b200.models.stack import StackModel


def model(**overrides):
    args = dict(vocab_size=31, dim=16, heads=2, layers=2)
    args.update(overrides)
    return BaselineModel(**args)


def test_causal_and_prefix_invariance():
    torch.manual_seed(123)
    m = model().double().eval()
    ids = torch.randint(31, (2, 33))
    with torch.no_grad():
        full = m(ids)
        for cut in (1, 3, 8, 15, 16, 17, 31, 32):
            changed = ids.clone()
            changed[:, cut:] = (changed[:, cut:] + 7) % 31
            torch.testing.assert_close(m(changed)[:, :cut], full[:, :cut], rtol=1e-9, atol=1e-10)
            torch.testing.assert_close(m(ids[:, :cut]), full[:, :cut], rtol=1e-9, atol=1e-10)


def test_shapes_sup_zeroing_and_backward():
    torch.manual_seed(123)
    m = model()
    ids = torch.randint(31, (2, 17))
    sup = torch.zeros(2, 17, dtype=torch.bool)
    sup[:, -3:] = True
    logits = m(ids, sup=sup)
    assert logits.shape == (2, 17, 31) and logits[:, :-3].abs().max().item() == 0.0
    logits[sup].square().mean().backward()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


def test_full_block_checkpoint_matches_reference():
    torch.manual_seed(9)
    reference = model(backend="math").double()
    checkpointed = copy.deepcopy(reference)
    checkpointed.checkpoint_chunks = True
    ids = torch.randint(31, (2, 13))
    targets = torch.randint(31, ids.shape)
    sup = torch.zeros_like(ids, dtype=torch.bool)
    sup[:, -4:] = True
    expected = reference(ids, targets=targets, sup=sup)["loss_sum"]
    actual = checkpointed(ids, targets=targets, sup=sup)["loss_sum"]
    torch.testing.assert_close(actual, expected, atol=1e-10, rtol=1e-10)
    expected.backward()
    actual.backward()
    for left, right in zip(reference.parameters(), checkpointed.parameters()):
        if left.grad is not None:
            torch.testing.assert_close(left.grad, right.grad, atol=1e-9, rtol=1e-8)


def test_param_count_matches_stack_within_ten_percent():
    base = BaselineModel(256, dim=256, heads=4, layers=3)
    stack = StackModel(256, dim=256, heads=4, block_size=16, topk=64, arch="Lx2,G")
    pb = sum(p.numel() for p in base.parameters())
    ps = sum(p.numel() for p in stack.parameters())
    assert abs(pb - ps) / ps < 0.10


def test_validation():
    for kwargs in (dict(heads=3), dict(layers=0), dict(dim=0), dict(ffn_ratio=0), dict(vocab_size=0)):
        with pytest.raises(ValueError):
            model(**kwargs)
    with pytest.raises(ValueError):
        model()(torch.empty(4, dtype=torch.long))
