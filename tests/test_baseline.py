"""Dense baseline on CPU: a plain restatement of the network, the sliced loss, parameter parity."""
import math

import pytest
import torch
from torch.nn import functional as F

from exploration_b200.models.baseline import BaselineModel
from exploration_b200.models.stack import StackModel

VOCAB = 23


def make(**overrides):
    options = dict(vocab_size=VOCAB, dim=16, heads=2, layers=2)
    options.update(overrides)
    return BaselineModel(**options)


def restated_logits(m, ids):
    """Pre-norm causal transformer written out with torch ops on the model's weights."""
    batch, n = ids.shape
    x = m.embedding.weight[ids]
    half = m.hd // 2
    # Rotation angles in fp32, as the model computes them whatever its dtype.
    freq = 10000.0 ** (-torch.arange(0, m.hd, 2, dtype=torch.float32) / m.hd)
    angle = torch.arange(n, dtype=torch.float32)[:, None] * freq[None]
    cos, sin = (t.to(x.dtype)[None, :, None, :] for t in (angle.cos(), angle.sin()))

    def rotate(t):                       # rotary embedding on pairs (first half, second half)
        a, b = t[..., :half], t[..., half:]
        return torch.cat((a * cos - b * sin, a * sin + b * cos), -1)

    causal = torch.ones(n, n, dtype=torch.bool).tril()
    for blk in m.blocks:
        h = F.layer_norm(x, (m.dim,), blk.attn_norm.weight, blk.attn_norm.bias)
        q, k, v = (h @ blk.qkv.weight.t()).view(batch, n, 3, m.heads, m.hd).unbind(2)
        q, k = rotate(q), rotate(k)
        scores = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(m.hd)
        attn = scores.masked_fill(~causal, float("-inf")).softmax(-1)
        ctx = torch.einsum("bhqk,bkhd->bqhd", attn, v).reshape(batch, n, m.dim)
        x = x + ctx @ blk.out.weight.t()
        u = F.layer_norm(x, (m.dim,), blk.ffn_norm.weight, blk.ffn_norm.bias) @ blk.ffn[0].weight.t() + blk.ffn[0].bias
        x = x + F.gelu(u) @ blk.ffn[2].weight.t() + blk.ffn[2].bias
    return F.layer_norm(x, (m.dim,), m.final_norm.weight, m.final_norm.bias) @ m.embedding.weight.t()


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(99)


@pytest.mark.parametrize("backend", ["math", "auto"])
def test_logits_match_the_restated_network(backend):
    m = make(backend=backend).double().eval()
    ids = torch.randint(VOCAB, (2, 19))
    with torch.no_grad():
        torch.testing.assert_close(m(ids), restated_logits(m, ids), rtol=1e-9, atol=1e-10)


def test_supervision_masks_compact_logits_and_positions():
    m = make().double().eval()
    ids = torch.randint(VOCAB, (2, 17))
    sup = torch.zeros(2, 17, dtype=torch.bool)
    sup[:, [2, 9, 16]] = True
    with torch.no_grad():
        full = m(ids)
        masked = m(ids, sup=sup)
        compact = m(ids, sup=sup, compact=True)
        streamed = torch.cat([logits for _, logits, _ in m.iter_logits(ids, torch.tensor([[2, 9, 16]] * 2))], 1)
    assert masked[~sup].abs().max() == 0
    torch.testing.assert_close(masked[sup].view(2, 3, VOCAB), full[:, [2, 9, 16]])
    torch.testing.assert_close(compact, full[:, [2, 9, 16]])
    torch.testing.assert_close(streamed, compact)


@pytest.mark.parametrize("recompute,chunk", [(False, 128), (True, 3)])
def test_training_loss_and_gradients_follow_the_logits(recompute, chunk):
    m = make(checkpoint_chunks=recompute, loss_chunk=chunk).double()
    ids, targets = torch.randint(VOCAB, (2, 14)), torch.randint(VOCAB, (2, 14))
    sup = torch.rand(2, 14) > 0.5
    sup[0] = False                                        # a row with nothing to predict
    result = m(ids, targets=targets, sup=sup)
    logits = m(ids)
    want = F.cross_entropy(logits[sup].float(), targets[sup], reduction="sum")
    assert int(result["count"]) == int(sup.sum()) and int(result["row_errors"][0]) == 0
    torch.testing.assert_close(result["loss_sum"], want, rtol=1e-6, atol=1e-5)
    params = list(m.parameters())
    for g, w in zip(torch.autograd.grad(result["loss_sum"], params), torch.autograd.grad(want, params)):
        torch.testing.assert_close(g, w, rtol=1e-5, atol=1e-6)


def test_causality():
    m = make().double().eval()
    ids = torch.randint(VOCAB, (1, 24))
    with torch.no_grad():
        full = m(ids)
        for cut in (1, 7, 23):
            changed = ids.clone()
            changed[:, cut:] = (changed[:, cut:] + 3) % VOCAB
            torch.testing.assert_close(m(changed)[:, :cut], full[:, :cut], rtol=1e-10, atol=1e-11)


def test_three_layers_match_the_stack_parameter_budget():
    base = BaselineModel(256, dim=256, heads=4, layers=3)
    stack = StackModel(256, dim=256, heads=4, block_size=16, topk=64, arch="Lx2,G")
    count = lambda model: sum(p.numel() for p in model.parameters())  # noqa: E731
    assert abs(count(base) - count(stack)) / count(stack) < 0.10


def test_rejects_bad_sizes_and_inputs():
    for options in (dict(heads=3), dict(layers=0), dict(dim=0), dict(ffn_ratio=0), dict(vocab_size=0),
                    dict(backend="cudnn"), dict(dim=6, heads=2)):
        with pytest.raises(ValueError):
            make(**options)
    with pytest.raises(ValueError):
        make()(torch.empty(4, dtype=torch.long))
