"""Stack model on CPU: the read path against the loop oracle, causality, gradients, configuration.

The oracle composes the model's own encoder and projections with
``tools.oracle.eager_attention`` (a per-row loop that shares no code with the
operators), so a test fails when the model's read rounds, not its weights,
disagree with the definition.
"""
import math

import pytest
import torch

from exploration_b200.models.stack import StackModel, parse_arch
from exploration_b200.ops.gated_reference import block_log_mass
from exploration_b200.tools.oracle import eager_attention

VOCAB = 29


def make(**overrides):
    options = dict(vocab_size=VOCAB, dim=16, heads=2, block_size=2, topk=3, arch="Lx2,G", pos_chunk=3)
    options.update(overrides)
    return StackModel(**options)


def oracle_logits(m, ids, positions):
    """Logits at ``positions`` (a list) through the model's layers and the loop oracle."""
    batch = ids.shape[0]
    x, raw_k, raw_v = m.encode(ids)
    pos = torch.tensor(positions)[None].expand(batch, -1)
    z = x[:, positions]
    for rd in m.reads:
        q = rd.wq(rd.q_norm(z)).view(batch, len(positions), m.heads, m.hd)
        topk = None if m.topk >= -(-ids.shape[1] // m.block_size) else m.topk
        ctx = eager_attention(q, raw_k, raw_v, pos, m.block_size, topk=topk)
        z = z + rd.read_out(ctx.reshape(batch, len(positions), m.dim))
        z = z + rd.ffn(rd.ffn_norm(z))
    return m.lm_head(m.final_norm(z))


def tail(n, count, batch=2):
    sup = torch.zeros(batch, n, dtype=torch.bool)
    sup[:, -count:] = True
    return sup


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(7)


@pytest.mark.parametrize("topk,arch", [(3, "Lx2,G"), (64, "Lx2,G"), (2, "L,(G)x2"), (1, "Lx2,Gx2")])
def test_logits_match_the_loop_oracle(topk, arch):
    m = make(topk=topk, arch=arch).double().eval()
    ids = torch.randint(VOCAB, (2, 23))
    positions = [0, 3, 9, 18, 21, 22]
    sup = torch.zeros(2, 23, dtype=torch.bool)
    sup[:, positions] = True
    with torch.no_grad():
        want = oracle_logits(m, ids, positions)
        torch.testing.assert_close(m(ids, sup=sup, compact=True), want, rtol=1e-9, atol=1e-10)
        full = m(ids, sup=sup)
        torch.testing.assert_close(full[:, positions], want, rtol=1e-9, atol=1e-10)
        others = [i for i in range(23) if i not in positions]
        assert full[:, others].abs().max().item() == 0.0


@pytest.mark.parametrize("topk", [3, 64])
def test_gradients_match_the_loop_oracle(topk):
    """Autograd through the top-k read (materialising reference) and the dense read."""
    m = make(topk=topk).double()
    ids = torch.randint(VOCAB, (2, 19))
    positions = list(range(15, 19))
    probe = torch.randn(2, len(positions), VOCAB, dtype=torch.double)
    params = [m.reads[0].wq.weight, m.reads[0].read_out.weight, m.raw_kv.proj.weight, m.local[1].qkv.weight,
              m.reads[0].ffn[2].weight, m.embedding.weight]
    got = torch.autograd.grad((m(ids, sup=tail(19, 4), compact=True) * probe).sum(), params)
    want = torch.autograd.grad((oracle_logits(m, ids, positions) * probe).sum(), params)
    for g, w in zip(got, want):
        torch.testing.assert_close(g, w, rtol=1e-8, atol=1e-9)


def test_gate_gradient_reaches_unselected_remote_blocks():
    """The gate normalises over every remote block, so blocks the top-k drops still get gradient."""
    m = make(block_size=4, topk=2)
    ids = torch.randint(VOCAB, (1, 64))
    x, raw_k, _ = m.encode(ids)
    pos = torch.tensor([[63]])
    q = m.reads[0].wq(m.reads[0].q_norm(x[:, 63:64])).view(1, 1, m.heads, m.hd)
    scores = block_log_mass(q, raw_k, pos, 4)
    scores.retain_grad()
    gate = torch.nan_to_num(scores - scores.logsumexp(-1, keepdim=True), nan=0.0, neginf=0.0)
    kept = scores.detach().topk(2, -1).indices
    gate.gather(-1, kept).sum().backward()
    remote = torch.isfinite(scores.detach())
    dropped = remote.clone().scatter_(-1, kept, False)
    assert dropped.any() and scores.grad[dropped].abs().sum() > 0
    assert scores.grad[~remote].abs().sum() == 0


def test_block_log_mass_is_the_blockwise_logsumexp():
    g = torch.Generator().manual_seed(1)
    b, n = 4, 30
    q = torch.randn(2, 3, 2, 8, generator=g, dtype=torch.double)
    k = torch.randn(2, n, 2, 8, generator=g, dtype=torch.double)
    pos = torch.tensor([[3, 13, 29], [8, 9, 27]])
    scores = block_log_mass(q, k, pos, b)
    assert scores.shape == (2, 3, 2, -(-n // b))
    for row in range(2):
        for qi in range(3):
            p = int(pos[row, qi])
            for h in range(2):
                for j in range(scores.shape[-1]):
                    if j < p // b - 1:
                        keys = k[row, j * b:(j + 1) * b, h]
                        want = (keys @ q[row, qi, h] / math.sqrt(8)).logsumexp(0)
                        torch.testing.assert_close(scores[row, qi, h, j], want)
                    else:
                        assert scores[row, qi, h, j] == float("-inf")


@pytest.mark.parametrize("n", [1, 2, 3, 5, 16, 17, 40])
def test_odd_lengths_run_forward_and_backward(n):
    m = make()
    ids = torch.randint(VOCAB, (2, n))
    for sup in (None, tail(n, min(2, n))):
        logits = m(ids, sup=sup)
        assert logits.shape == (2, n, VOCAB) and torch.isfinite(logits).all()
        logits.square().mean().backward()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


def test_causality_and_prefix_invariance():
    for arch in ("Lx2,G", "Lx2,(G)x2"):
        m = make(arch=arch).double().eval()
        ids = torch.randint(VOCAB, (2, 30))
        with torch.no_grad():
            full = m(ids)
            assert torch.equal(m(ids, sup=torch.ones(2, 30, dtype=torch.bool)), full)
            for cut in (1, 2, 5, 12, 13, 29):
                later_changed = ids.clone()
                later_changed[:, cut:] = (later_changed[:, cut:] + 5) % VOCAB
                torch.testing.assert_close(m(later_changed)[:, :cut], full[:, :cut], rtol=1e-9, atol=1e-10)
                torch.testing.assert_close(m(ids[:, :cut]), full[:, :cut], rtol=1e-9, atol=1e-10)


def test_loss_at_one_position_sends_no_gradient_to_later_tokens():
    m = make().double()
    ids = torch.randint(VOCAB, (1, 33))
    embedded = []

    def keep(module, inputs, output):
        output.retain_grad()
        embedded.append(output)

    hook = m.embedding.register_forward_hook(keep)
    sup = torch.zeros(1, 33, dtype=torch.bool)
    sup[0, 19] = True
    m(ids, sup=sup, compact=True).square().sum().backward()
    hook.remove()
    grad = embedded[0].grad[0]
    assert grad[20:].abs().max() == 0 and grad[:20].abs().sum() > 0


def test_query_chunking_and_cpu_autocast():
    m, one_at_a_time = make().eval(), make(pos_chunk=1).eval()
    one_at_a_time.load_state_dict(m.state_dict())
    ids = torch.randint(VOCAB, (2, 27))
    with torch.no_grad():
        torch.testing.assert_close(m(ids, sup=tail(27, 9)), one_at_a_time(ids, sup=tail(27, 9)), rtol=1e-5, atol=1e-6)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        loss = m(ids).float().square().mean()
    loss.backward()
    assert torch.isfinite(loss) and all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)


def test_diagnose_reports_selection_quality():
    ids = torch.randint(VOCAB, (2, 40))
    with torch.no_grad():
        narrow = make(topk=2).eval().diagnose(ids)
        wide = make(topk=64).eval().diagnose(ids)
        needle = make(block_size=4, topk=64).eval().diagnose(ids, sup=tail(40, 1), needle_pos=torch.tensor([3, 5]))
    assert 0.0 < narrow["sel_cov"] < 1.0 and narrow["gate_margin"] >= 0.0
    assert wide["sel_cov"] == pytest.approx(1.0, abs=1e-4) and "gate_margin" not in wide
    assert needle["needle_block_hit"] == 1.0


def test_arch_grammar_and_weight_sharing():
    assert parse_arch("Lx2,(G)x3,G") == [("L", 2, False), ("G", 3, True), ("G", 1, False)]
    for bad in ("", " ", "G,L", "Lx0", "X", "L2", "(L)x0", "(G)", "L,", "Lx2,(G)x", "L,Gx2,Lx1"):
        with pytest.raises(ValueError):
            make(arch=bad)
    shared, separate = make(arch="L,(G)x2"), make(arch="L,Gx2")
    assert shared.reads[0] is shared.reads[1] and separate.reads[0] is not separate.reads[1]
    assert sum(p.numel() for p in shared.parameters()) < sum(p.numel() for p in separate.parameters())


def test_configuration_and_input_errors():
    for options in (dict(block_size=1), dict(heads=3), dict(topk=0), dict(ffn_ratio=0), dict(pos_chunk=-1)):
        with pytest.raises(ValueError):
            make(**options)
    m = make()
    for shape in ((0, 4), (1, 0), (4,)):
        with pytest.raises(ValueError):
            m(torch.empty(shape, dtype=torch.long))
    ragged = tail(8, 3)
    ragged[1, -3] = False
    with pytest.raises(ValueError):
        m(torch.randint(VOCAB, (2, 8)), sup=ragged)
