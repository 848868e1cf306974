"""tcgen05 GEMM and the fused linear layers against fp32 torch references (B200 only)."""
import pytest
import torch
from torch.nn import functional as F

from exploration_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean(native):
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert native.device_errors(torch.cuda.current_device()) == (0, 0)


def _operand(rows, cols, mn, seed):
    """Logical [rows, cols] operand; stored transposed when ``mn``."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    logical = torch.randn(rows, cols, device="cuda", generator=g).to(torch.bfloat16)
    stored = logical.t().contiguous() if mn else logical
    return logical, stored


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (304, 200, 136), (1024, 768, 512), (264, 520, 1000)])
def test_gemm_layouts(m, n, k, a_mn, b_mn):
    a, a_st = _operand(m, k, a_mn, 1)
    b, b_st = _operand(n, k, b_mn, 2)
    out = torch.empty(m, n, device="cuda", dtype=torch.float32)
    G.gemm(a_st, a_mn, b_st, b_mn, out, G.STORE_F32)
    ref = a.float() @ b.float().t()
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-3)


@pytest.mark.parametrize("m,n,k", [(512, 4096, 1024), (8192, 3072, 1024)])
def test_gemm_large_bf16(m, n, k):
    a, _ = _operand(m, k, False, 3)
    b, _ = _operand(n, k, False, 4)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    G.gemm(a, False, b, False, out, G.STORE_BF16)
    ref = a.float() @ b.float().t()
    torch.testing.assert_close(out.float(), ref, atol=0.25, rtol=2e-2)


def test_gemm_epilogues():
    m, n, k = 384, 320, 256
    a, _ = _operand(m, k, False, 5)
    b, _ = _operand(n, k, False, 6)
    bias = torch.randn(n, device="cuda")
    acc = a.float() @ b.float().t()
    dgelu = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    post = torch.empty_like(dgelu)
    G.gemm(a, False, b, False, post, G.BIAS_GELU, bias=bias, aux=dgelu)
    z = (acc + bias).requires_grad_()
    want_dgelu = torch.autograd.grad(F.gelu(z).sum(), z)[0]
    torch.testing.assert_close(dgelu.float(), want_dgelu, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(post.float(), F.gelu(acc + bias), atol=0.1, rtol=1e-2)
    res = torch.randn(m, n, device="cuda")
    out = torch.empty(m, n, device="cuda")
    G.gemm(a, False, b, False, out, G.BIAS_RESIDUAL, bias=bias, residual=res)
    torch.testing.assert_close(out, res + acc + bias, atol=2e-2, rtol=2e-3)
    accum = torch.randn(m, n, device="cuda")
    start = accum.clone()
    G.gemm(a, False, b, False, accum, G.ACCUM_F32, alpha=0.5)
    torch.testing.assert_close(accum, start + 0.5 * acc, atol=2e-2, rtol=2e-3)
    dgrad = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    partial = torch.empty(-(-m // G.TILE_M), n, device="cuda")
    G.gemm(a, False, b, False, dgrad, G.GELU_BACK, aux=dgelu, partial=partial)
    want = acc * dgelu.float()
    torch.testing.assert_close(dgrad.float(), want, atol=0.1, rtol=2e-2)
    torch.testing.assert_close(partial.sum(0), dgrad.float().sum(0), atol=0.5, rtol=1e-2)


def test_fused_layers_match_torch():
    torch.manual_seed(0)
    rows, d, hidden = 300, 256, 1024
    up, down = torch.nn.Linear(d, hidden).cuda(), torch.nn.Linear(hidden, d).cuda()
    proj = torch.nn.Linear(d, d, bias=False).cuda()
    h = torch.randn(rows, d, device="cuda").to(torch.bfloat16).requires_grad_()
    y = torch.randn(rows, d, device="cuda", requires_grad=True)
    out = G.FFNResidual.apply(h, y, up.weight, up.bias, down.weight, down.bias)
    out = G.LinearResidual.apply(h, proj.weight, None, out)
    hr, yr = h.detach().float().requires_grad_(), y.detach().clone().requires_grad_()
    ref = yr + down(F.gelu(up(hr)))
    ref = ref + proj(hr)
    torch.testing.assert_close(out, ref, atol=0.1, rtol=2e-2)
    probe = torch.randn_like(ref)
    params = [up.weight, up.bias, down.weight, down.bias, proj.weight]
    got = torch.autograd.grad((out * probe).sum(), [h, y, *params])
    want = torch.autograd.grad((ref * probe).sum(), [hr, yr, *params])
    for a, e in zip(got, want):
        scale = max(1.0, e.abs().max().item())
        torch.testing.assert_close(a.float(), e, atol=5e-2 * scale, rtol=5e-2)
