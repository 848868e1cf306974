"""Gated dense attention reference and paged sparse attention vs the loop oracle (fp64)."""
import torch

from exploration_b200.ops.attention import dense_attention
from exploration_b200.ops.gated_reference import eager_gated
from exploration_b200.ops.sparse import TensorPages, sparse_attention
from exploration_b200.tools.oracle import eager_attention


def test_forward_and_all_input_gradients():
    torch.manual_seed(981)
    for n, b in ((1, 2), (7, 3), (17, 4), (33, 8)):
        q = torch.randn(2, 5, 2, 6, dtype=torch.float64, requires_grad=True)
        k = torch.randn(2, n, 2, 6, dtype=torch.float64, requires_grad=True)
        v = torch.randn_like(k, requires_grad=True)
        pos = torch.tensor([[0, min(3, n - 1), n - 1, -1, n // 2], [n - 1, -1, 0, n // 2, n - 1]])
        expected = eager_attention(q, k, v, pos, b)
        actual = dense_attention(q, k, v, pos, b, "torch", q_chunk=2, kv_chunk=2 * b)
        torch.testing.assert_close(actual, expected, atol=1e-11, rtol=1e-10)
        probe = torch.randn_like(actual)
        want = torch.autograd.grad((expected * probe).sum(), (q, k, v))
        got = torch.autograd.grad((actual * probe).sum(), (q, k, v))
        for a, e in zip(got, want):
            torch.testing.assert_close(a, e, atol=1e-10, rtol=1e-9)


def test_eager_vectorised_form_matches_oracle():
    torch.manual_seed(3)
    q = torch.randn(1, 4, 2, 8, dtype=torch.float64)
    k = torch.randn(1, 29, 2, 8, dtype=torch.float64)
    v = torch.randn_like(k)
    pos = torch.tensor([[28, 3, 17, 9]])
    torch.testing.assert_close(eager_gated(q, k, v, pos, 4), eager_attention(q, k, v, pos, 4),
                               atol=1e-12, rtol=1e-10)


def test_gate_gradient_finite_difference():
    torch.manual_seed(4)
    q = torch.randn(1, 2, 1, 4, dtype=torch.float64, requires_grad=True)
    k = torch.randn(1, 13, 1, 4, dtype=torch.float64, requires_grad=True)
    v = torch.randn_like(k, requires_grad=True)
    pos = torch.tensor([[9, 12]])
    assert torch.autograd.gradcheck(lambda q, k, v: dense_attention(q, k, v, pos, 2, "torch", 2, 6),
                                    (q, k, v), eps=1e-6, atol=1e-5, rtol=1e-4)


def test_sparse_pages_and_dense_degenerate():
    torch.manual_seed(124)
    q = torch.randn(2, 4, 3, 8, dtype=torch.float64)
    k = torch.randn(2, 45, 3, 8, dtype=torch.float64)
    v = torch.randn_like(k)
    pos = torch.tensor([[0, 7, 44, 22], [13, 44, 1, 43]])
    for keep in (1, 2, 64):
        expected = eager_attention(q, k, v, pos, 4, keep)
        for page in (4, 12, 64):
            actual = sparse_attention(q, TensorPages(k, v, page), pos, 4, keep, "torch",
                                      score_page_tokens=8)
            torch.testing.assert_close(actual, expected, rtol=1e-10, atol=1e-11)


def test_sparse_selection_is_returned_and_padding_rows_are_zero():
    torch.manual_seed(5)
    q = torch.randn(1, 3, 2, 8, dtype=torch.float64)
    k = torch.randn(1, 40, 2, 8, dtype=torch.float64)
    v = torch.randn_like(k)
    pos = torch.tensor([[39, -1, 20]])
    out, sel = sparse_attention(q, TensorPages(k, v, 16), pos, 4, 2, "torch", return_selection=True)
    assert sel["indices"].shape == (1, 3, 2, 2)
    assert bool((sel["indices"][0, 1] == -1).all())
    assert float(out[0, 1].abs().max()) == 0.0
