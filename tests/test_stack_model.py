"""Stack model: loop oracle, causality, gradient paths, configuration."""
import math

import pytest
import torch
from torch.nn import functional as F

from exploration_b200.models.stack import StackModel


def model(**overrides):
    args = dict(vocab_size=31, dim=16, heads=2, block_size=2, topk=3, arch="Lx2,G", pos_chunk=3)
    args.update(overrides)
    return StackModel(**args)


def oracle_logits(m, ids, positions):
    """Per-position loop over the read path using the model's own sub-modules."""
    b = m.block_size
    batch, n = ids.shape
    x, raw_k, raw_v = m.encode(ids)
    groups = -(-n // b)
    padded = F.pad(raw_k, (0, 0, 0, 0, 0, groups * b - n))
    outs = []
    for t in positions:
        visible = [j for j in range(groups) if (j + 1) * b <= (t // b - 1) * b]
        z = x[:, t]
        for rd in m.reads:
            q = rd.wq(rd.q_norm(z)).reshape(batch, m.heads, m.hd)
            ctx = torch.zeros(batch, m.heads, m.hd, dtype=z.dtype)
            for bi in range(batch):
                for h in range(m.heads):
                    qh = q[bi, h]
                    scores = {j: (padded[bi, j * b:(j + 1) * b, h] @ qh / math.sqrt(m.hd)).logsumexp(0)
                              for j in visible}
                    keys, logits = [], []
                    if visible:
                        all_s = torch.stack([scores[j] for j in visible])
                        lz = all_s.logsumexp(0)
                        ranked = sorted(visible, key=lambda j: scores[j].item(), reverse=True)
                        for j in ranked[:m.topk]:
                            for i in range(j * b, min((j + 1) * b, t + 1)):
                                keys.append(i)
                                logits.append(raw_k[bi, i, h] @ qh / math.sqrt(m.hd) + scores[j] - lz)
                    lo = max((t // b - 1) * b, 0)
                    for i in range(lo, t + 1):
                        keys.append(i)
                        logits.append(raw_k[bi, i, h] @ qh / math.sqrt(m.hd))
                    w = torch.stack(logits).softmax(0)
                    ctx[bi, h] = w @ raw_v[bi, keys, h]
            z = z + rd.read_out(ctx.reshape(batch, m.dim))
            z = z + rd.ffn(rd.ffn_norm(z))
        outs.append(m.lm_head(m.final_norm(z)))
    return torch.stack(outs, 1)


@pytest.fixture(autouse=True)
def seed():
    torch.manual_seed(123)


def test_shapes_backward_and_tail_lengths():
    for n in (1, 3, 4, 5, 16, 17, 65):
        for use_sup in (False, True):
            m = model()
            ids = torch.randint(31, (2, n))
            sup = None
            if use_sup:
                sup = torch.zeros(2, n, dtype=torch.bool)
                sup[:, -2:] = True
            logits = m(ids, sup=sup)
            assert logits.shape == (2, n, 31) and torch.isfinite(logits).all()
            if use_sup and n > 2:
                assert logits[:, :-2].abs().max().item() == 0.0
                loss = logits[sup].square().mean()
            else:
                loss = logits.square().mean()
            loss.backward()
            for p in m.parameters():
                if p.grad is not None:
                    assert torch.isfinite(p.grad).all()


def test_sup_none_equals_all_positions():
    m = model().double().eval()
    ids = torch.randint(31, (2, 33))
    with torch.no_grad():
        torch.testing.assert_close(m(ids), m(ids, sup=torch.ones(2, 33, dtype=torch.bool)),
                                   rtol=1e-10, atol=1e-10)


def test_end_to_end_oracle_values_and_gradients():
    m = model().double()
    ids = torch.randint(31, (2, 21))
    sup = torch.zeros(2, 21, dtype=torch.bool)
    sup[:, -4:] = True
    positions = [17, 18, 19, 20]
    with torch.no_grad():
        m.eval()
        torch.testing.assert_close(m(ids, sup=sup)[:, -4:], oracle_logits(m, ids, positions),
                                   rtol=1e-9, atol=1e-10)
    m.train()
    probe = torch.randn(2, 4, 31, dtype=torch.double)
    params = [m.reads[0].wq.weight, m.reads[0].read_out.weight, m.raw_kv.proj.weight,
              m.local[0].qkv.weight, m.reads[0].ffn[0].weight, m.embedding.weight]
    out = m(ids, sup=sup)
    got = torch.autograd.grad((out[:, -4:] * probe).sum(), params, retain_graph=True)
    want = torch.autograd.grad((oracle_logits(m, ids, positions) * probe).sum(), params)
    for a, e in zip(got, want):
        torch.testing.assert_close(a, e, rtol=1e-8, atol=1e-9)


def test_dense_fast_path_matches_sparse_oracle():
    m = model(topk=64).double().eval()
    ids = torch.randint(31, (2, 21))
    sup = torch.zeros(2, 21, dtype=torch.bool)
    sup[:, -4:] = True
    with torch.no_grad():
        torch.testing.assert_close(m(ids, sup=sup)[:, -4:], oracle_logits(m, ids, [17, 18, 19, 20]),
                                   rtol=1e-9, atol=1e-10)
        torch.testing.assert_close(m(ids), oracle_logits(m, ids, list(range(21))), rtol=1e-9,
                                   atol=1e-10)
    m(ids, sup=sup).square().mean().backward()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


def test_shared_weight_cycling():
    shared, indep = model(arch="L,(G)x2"), model(arch="L,Gx2")
    assert shared.reads[0] is shared.reads[1] and indep.reads[0] is not indep.reads[1]
    assert sum(p.numel() for p in shared.parameters()) < sum(p.numel() for p in indep.parameters())
    m = model(arch="L,(G)x2", topk=3).double().eval()
    ids = torch.randint(31, (2, 21))
    sup = torch.zeros(2, 21, dtype=torch.bool)
    sup[:, -4:] = True
    with torch.no_grad():
        torch.testing.assert_close(m(ids, sup=sup)[:, -4:], oracle_logits(m, ids, [17, 18, 19, 20]),
                                   rtol=1e-9, atol=1e-10)


def test_arch_parser():
    for bad in ("", "G,L", "Lx0", "X", "(L)x0", "(G)", "L,", "Lx2,(G)x", "L,Gx2,Lx1"):
        with pytest.raises(ValueError):
            model(arch=bad)
    for good, passes in (("L", 1), ("Lx2,G", 3), ("(L)x3,(G)x2", 5), ("Gx2", 2)):
        m = model(arch=good)
        assert len(m.local) + len(m.reads) == passes


def test_future_perturbation_and_prefix_invariance():
    for arch in ("Lx2,G", "Lx2,(G)x2", "Lx2,Gx2"):
        m = model(arch=arch).double().eval()
        ids = torch.randint(31, (2, 33))
        with torch.no_grad():
            full = m(ids)
            for cut in (1, 3, 4, 5, 8, 15, 16, 17, 31, 32):
                changed = ids.clone()
                changed[:, cut:] = (changed[:, cut:] + 7) % 31
                torch.testing.assert_close(m(changed)[:, :cut], full[:, :cut], rtol=1e-9, atol=1e-10)
                torch.testing.assert_close(m(ids[:, :cut])[:, :cut], full[:, :cut], rtol=1e-9,
                                           atol=1e-10)


def test_no_gradient_to_future_inputs():
    m = model().double()
    ids = torch.randint(31, (1, 35))
    sup = torch.zeros(1, 35, dtype=torch.bool)
    sup[0, 20] = True
    captured = []

    def keep(module, inputs, output):
        output.retain_grad()
        captured.append(output)

    hook = m.embedding.register_forward_hook(keep)
    m(ids, sup=sup)[0, 20].square().sum().backward()
    hook.remove()
    grad = captured[0].grad
    assert grad[:, 21:].abs().max().item() == 0
    assert grad[:, :21].abs().sum().item() > 0


def test_gradient_highway_reaches_unselected_visible_blocks():
    m = model(block_size=4, topk=2)
    ids = torch.randint(31, (2, 65))
    x, raw_k, _ = m.encode(ids)
    n, b = 65, m.block_size
    groups = -(-n // b)
    pos = torch.arange(60, 65)[None].expand(2, 5)
    visible = ((torch.arange(groups) + 1) * b)[None, None, :] <= ((pos // b - 1) * b)[:, :, None]
    kb = F.pad(raw_k, (0, 0, 0, 0, 0, groups * b - n)).reshape(2, groups, b, m.heads, m.hd)
    q = m.reads[0].wq(m.reads[0].q_norm(x[torch.arange(2)[:, None], pos])).reshape(2, 5, m.heads, m.hd)
    s = m.push_scores(q, kb, visible)
    s.retain_grad()
    gate = torch.nan_to_num(s - s.logsumexp(-1, keepdim=True), nan=0.0, neginf=0.0)
    (s.logsumexp(-1).square().mean() + gate.sum()).backward()
    sg = s.grad[0, -1]
    _, sel = s[0, -1].detach().topk(min(m.topk, groups), dim=-1)
    chosen = set(sel.flatten().tolist())
    unselected = [j for j in range(15) if j not in chosen]
    assert unselected and sg[:, unselected].abs().sum().item() > 0
    assert sg[:, 15:].abs().sum().item() == 0.0
    named = dict(m.named_parameters())
    for name in ("reads.0.wq.weight", "raw_kv.proj.weight"):
        assert named[name].grad is not None and named[name].grad.norm().item() > 0


def test_push_scores_matches_manual():
    m = model().double()
    ids = torch.randint(31, (2, 33))
    x, raw_k, _ = m.encode(ids)
    b, n = m.block_size, 33
    groups = -(-n // b)
    kb = F.pad(raw_k, (0, 0, 0, 0, 0, groups * b - n)).reshape(2, groups, b, m.heads, m.hd)
    pos = torch.tensor([[7, 20, 32], [7, 20, 32]])
    visible = ((torch.arange(groups) + 1) * b)[None, None, :] <= ((pos // b - 1) * b)[:, :, None]
    q = m.reads[0].wq(m.reads[0].q_norm(x[torch.arange(2)[:, None], pos])).reshape(2, 3, m.heads, m.hd)
    s = m.push_scores(q, kb, visible)
    for row in range(2):
        for pi, t in enumerate((7, 20, 32)):
            for h in range(m.heads):
                for g in range(groups):
                    if (g + 1) * b <= (t // b - 1) * b:
                        toks = raw_k[row, g * b:(g + 1) * b, h]
                        ref = (q[row, pi, h] @ toks.T / math.sqrt(m.hd)).logsumexp(-1)
                        torch.testing.assert_close(s[row, pi, h, g], ref, rtol=1e-10, atol=1e-10)
                    else:
                        assert s[row, pi, h, g].item() == float("-inf")


def test_pos_chunk_invariance_and_cpu_bf16():
    m = model().eval()
    other = model(pos_chunk=1).eval()
    other.load_state_dict(m.state_dict())
    ids = torch.randint(31, (2, 33))
    sup = torch.zeros(2, 33, dtype=torch.bool)
    sup[:, -7:] = True
    with torch.no_grad():
        torch.testing.assert_close(m(ids, sup=sup), other(ids, sup=sup), rtol=1e-5, atol=1e-6)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        loss = m(ids).float().square().mean()
    assert torch.isfinite(loss)
    loss.backward()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


def test_diagnose():
    ids = torch.randint(31, (2, 33))
    with torch.no_grad():
        rec = model(topk=2).eval().diagnose(ids)
        dense = model(topk=64).eval().diagnose(ids)
    assert 0.0 <= rec["sel_cov"] <= 1.0
    assert abs(dense["sel_cov"] - 1.0) < 1e-3 and "gate_margin" not in dense


def test_configuration_and_empty_inputs():
    for kwargs in (dict(block_size=1), dict(heads=3), dict(topk=0), dict(ffn_ratio=0),
                   dict(pos_chunk=-1)):
        with pytest.raises(ValueError):
            model(**kwargs)
    m = model()
    for shape in ((0, 4), (1, 0), (4,)):
        with pytest.raises(ValueError):
            m(torch.empty(shape, dtype=torch.long))
    ragged = torch.zeros(2, 8, dtype=torch.bool)
    ragged[0, -3:] = True
    ragged[1, -2:] = True
    with pytest.raises(ValueError):
        m(torch.randint(31, (2, 8)), sup=ragged)
