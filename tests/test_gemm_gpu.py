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


@pytest.mark.parametrize("shape", [G.AUTO, G.NARROW, G.WIDE, G.PAIR])
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (304, 200, 136), (1024, 768, 512), (264, 520, 1000),
                                   (600, 640, 4160)])
def test_gemm_layouts(m, n, k, a_mn, b_mn, shape):
    """Every tile shape (the CTA pair included) and operand layout, ragged edges in M, N and K."""
    a, a_st = _operand(m, k, a_mn, 1)
    b, b_st = _operand(n, k, b_mn, 2)
    out = torch.empty(m, n, device="cuda", dtype=torch.float32)
    G.gemm(a_st, a_mn, b_st, b_mn, out, G.STORE_F32, shape=shape)
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


@pytest.mark.parametrize("shape", [G.AUTO, G.WIDE, G.PAIR])
def test_gemm_epilogues(shape):
    m, n, k = 640, 520, 256
    a, _ = _operand(m, k, False, 5)
    b, _ = _operand(n, k, False, 6)
    bias = torch.randn(n, device="cuda")
    acc = a.float() @ b.float().t()
    dgelu = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    post = torch.empty_like(dgelu)
    G.gemm(a, False, b, False, post, G.BIAS_GELU, bias=bias, aux=dgelu, shape=shape)
    z = (acc + bias).requires_grad_()
    want_dgelu = torch.autograd.grad(F.gelu(z).sum(), z)[0]
    torch.testing.assert_close(dgelu.float(), want_dgelu, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(post.float(), F.gelu(acc + bias), atol=0.1, rtol=1e-2)
    res = torch.randn(m, n, device="cuda")
    out = torch.empty(m, n, device="cuda")
    G.gemm(a, False, b, False, out, G.BIAS_RESIDUAL, bias=bias, residual=res, shape=shape)
    torch.testing.assert_close(out, res + acc + bias, atol=2e-2, rtol=2e-3)
    accum = torch.randn(m, n, device="cuda")
    start = accum.clone()
    G.gemm(a, False, b, False, accum, G.ACCUM_F32, alpha=0.5, shape=shape)
    torch.testing.assert_close(accum, start + 0.5 * acc, atol=2e-2, rtol=2e-3)
    dgrad = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    partial = torch.empty(-(-m // G.TILE_M), n, device="cuda")
    G.gemm(a, False, b, False, dgrad, G.GELU_BACK, aux=dgelu, partial=partial, shape=shape)
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


@pytest.mark.parametrize("n_out,k_in", [(1024, 1024), (256, 1024), (3072, 1024), (200, 136)])
@pytest.mark.parametrize("splits", [0, 1, 5])
@pytest.mark.parametrize("shape", [G.AUTO, G.PAIR])
def test_weight_grad_accumulates_over_long_reductions(n_out, k_in, splits, shape):
    """``dW += g^T x`` at the training reduction length (8,192 tokens), both operands MN-major."""
    tokens = 8192
    g, _ = _operand(tokens, n_out, False, 7)
    x, _ = _operand(tokens, k_in, False, 8)
    grad = torch.randn(n_out, k_in, device="cuda")
    start = grad.clone()
    G.plain(g, True, x, True, grad, accumulate=True, splits=splits, shape=shape)
    want = start + g.float().t() @ x.float()
    torch.testing.assert_close(grad, want, atol=5e-2, rtol=2e-3)


def test_weight_grad_split_k_is_deterministic(native):
    g, _ = _operand(8192, 1024, False, 9)
    x, _ = _operand(8192, 1024, False, 10)
    assert native.gemm_plain_plan(1024, 1024, 8192, torch.cuda.get_device_properties(0).multi_processor_count)[1] > 1
    first = G.weight_grad(g, x)
    for _ in range(3):
        assert torch.equal(G.weight_grad(g, x), first)


@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("shape", [G.AUTO, G.PAIR])
@pytest.mark.parametrize("m,n,k", [(8192, 1024, 3072), (1000, 256, 1024), (384, 520, 4096)])
def test_forward_and_input_grad(m, n, k, splits, shape):
    """``x W^T`` (bf16 / fp32 out) and ``dy W`` (W read MN-major) against fp32 torch."""
    x, _ = _operand(m, k, False, 11)
    w, _ = _operand(n, k, False, 12)
    ref = x.float() @ w.float().t()
    out32 = torch.empty(m, n, device="cuda")
    G.plain(x, False, w, False, out32, splits=splits, shape=shape)
    torch.testing.assert_close(out32, ref, atol=5e-2, rtol=2e-3)
    out16 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    G.plain(x, False, w, False, out16, splits=splits, shape=shape)
    torch.testing.assert_close(out16.float(), ref, atol=0.25, rtol=2e-2)
    dy, _ = _operand(m, n, False, 13)
    w2, _ = _operand(n, k, False, 14)
    dx = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
    G.plain(dy, False, w2, True, dx, splits=splits, shape=shape)
    torch.testing.assert_close(dx.float(), dy.float() @ w2.float(), atol=0.25, rtol=2e-2)


def test_linear_layer_runs_no_library_gemm():
    """The no-bias linear layer (QKV, projections, LM head) runs forward and backward on gemm_tc."""
    from torch.profiler import ProfilerActivity, profile
    torch.manual_seed(1)
    layer = torch.nn.Linear(1024, 3072, bias=False).cuda()
    x = torch.randn(4096, 1024, device="cuda").to(torch.bfloat16).requires_grad_()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        y = G.Linear.apply(x, layer.weight, False)
        y.float().square().sum().backward()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("gemm_tc_kernel" in n for n in names)
    library = [n for n in names if n.startswith(("nvjet", "cutlass", "sm90_", "sm100_"))
               or ("gemm" in n.lower() and "gemm_tc" not in n)]
    assert not library, library
    xr = x.detach().float().requires_grad_()
    want = xr @ layer.weight.t()
    torch.testing.assert_close(y.float(), want, atol=0.25, rtol=2e-2)
    (want.square().sum()).backward()
    torch.testing.assert_close(x.grad.float(), xr.grad, atol=1.0, rtol=3e-2)
