"""Bitwise determinism of the native kernels (no atomics in any reduction).

Each op runs twice on identical inputs; outputs and gradients must be equal
bit for bit. This is the determinism half of the race-detection substitute
(compute-sanitizer is not available on the GPU pool).
"""
import pytest
import torch

from exploration_b200.ops import fused
from exploration_b200.ops.attention import dense_attention
from exploration_b200.ops.sparse import TensorPages, sparse_attention

pytestmark = pytest.mark.gpu


def _twice(fn):
    a = fn()
    b = fn()
    for x, y in zip(a, b):
        assert torch.equal(x, y), "outputs differ between two identical runs"


def test_gated_attention_is_deterministic():
    torch.manual_seed(0)
    n, h, d, b = 2048, 4, 64, 16
    q, k, v = (torch.randn(1, n, h, d, device="cuda").to(torch.bfloat16) for _ in range(3))
    pos = torch.arange(n, device="cuda")[None]
    g = torch.randn(1, n, h, d, device="cuda").to(torch.bfloat16)

    def run():
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        out = dense_attention(qq, kk, vv, pos, b, "cuda")
        grads = torch.autograd.grad(out, (qq, kk, vv), g)
        return (out, *grads)

    _twice(run)


def test_local_attention_is_deterministic():
    torch.manual_seed(1)
    n, h = 2048, 16
    qkv = torch.randn(1, n, 3, h, 64, device="cuda").to(torch.bfloat16)
    g = torch.randn(1, n, h * 64, device="cuda").to(torch.bfloat16)

    def run():
        x = qkv.clone().requires_grad_()
        out = fused.local_attention(x, None, 0, 0, n, 16, h, "cuda")
        (dx,) = torch.autograd.grad(out, (x,), g)
        return out, dx

    _twice(run)


def test_sparse_read_is_deterministic():
    torch.manual_seed(2)
    keys, h = 70000, 4
    q = torch.randn(1, 16, h, 64, device="cuda").to(torch.bfloat16)
    k = torch.randn(1, keys, h, 64, device="cuda").to(torch.bfloat16)
    v = torch.randn_like(k)
    pos = torch.linspace(keys - 16, keys - 1, 16, device="cuda").long()[None]

    def run():
        out, sel = sparse_attention(q, TensorPages(k, v), pos, 16, 64, "cuda", return_selection=True)
        return out, sel["indices"], sel["scores"], sel["log_zr"]

    _twice(run)


def test_layer_norm_and_gemm_layers_are_deterministic():
    from exploration_b200.ops import gemm as G
    torch.manual_seed(3)
    rows, d, hidden = 4096, 1024, 4096
    norm = torch.nn.LayerNorm(d).cuda()
    up, down = torch.nn.Linear(d, hidden).cuda(), torch.nn.Linear(hidden, d).cuda()
    x = torch.randn(rows, d, device="cuda")
    probe = torch.randn(rows, d, device="cuda")

    def run():
        xx = x.clone().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            h = fused.layer_norm(xx, norm, "cuda")
            out = G.FFNResidual.apply(h, xx, up.weight, up.bias, down.weight, down.bias)
        params = [xx, norm.weight, norm.bias, up.weight, up.bias, down.weight, down.bias]
        grads = torch.autograd.grad((out * probe).sum(), params)
        return (out, *grads)

    _twice(run)
