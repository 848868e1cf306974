"""sm_100a kernels against fp32 torch references of the same ops (B200 only)."""
import copy
import math

import pytest
import torch

from exploration_b200.models.stack import StackModel
from exploration_b200.ops import fused
from exploration_b200.ops.attention import dense_attention
from exploration_b200.ops.sparse import TensorPages, sparse_attention
from exploration_b200.tools.oracle import eager_attention

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 2e-4), torch.bfloat16: (3e-2, 5e-2)}


@pytest.fixture(autouse=True)
def _no_tf32_and_clean_errors(native):
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert native.device_errors(torch.cuda.current_device()) == (0, 0)


def _dense_inputs(n, b, d, dtype, queries=5, heads=2, seed=772):
    torch.manual_seed(seed)
    q = torch.randn(2, queries, heads, d, device="cuda", dtype=dtype, requires_grad=True)
    k = torch.randn(2, n, heads, d, device="cuda", dtype=dtype, requires_grad=True)
    v = torch.randn_like(k, requires_grad=True)
    if queries == 5:
        pos = torch.tensor([[0, b - 1, min(2 * b + 1, n - 1), n - 1, -1], [n - 1, 0, n // 2, -1, n - 2]],
                           device="cuda")
    else:
        pos = torch.randint(0, n, (2, queries), device="cuda")
        pos[0, -1] = -1
    return q, k, v, pos


CASES = [(17, 2, 16), (129, 16, 32), (257, 32, 64), (193, 64, 96), (385, 128, 128), (131, 16, 256),
         (385, 128, 256), (300, 16, 64), (520, 16, 128), (400, 64, 64)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,b,d", CASES)
def test_gated_attention_matches_oracle(n, b, d, dtype):
    q, k, v, pos = _dense_inputs(n, b, d, dtype)
    rq, rk, rv = (t.detach().float().requires_grad_() for t in (q, k, v))
    expected = eager_attention(rq, rk, rv, pos, b)
    actual = dense_attention(q, k, v, pos, b, "cuda")
    probe = torch.randn_like(actual)
    got = torch.autograd.grad((actual * probe).sum(), (q, k, v))
    want = torch.autograd.grad((expected * probe.float()).sum(), (rq, rk, rv))
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(actual.float(), expected, atol=atol, rtol=rtol)
    for a, e in zip(got, want):
        torch.testing.assert_close(a.float(), e, atol=atol, rtol=rtol)


@pytest.mark.parametrize("b,d", [(16, 64), (16, 128), (32, 64), (128, 128), (64, 128)])
def test_gated_tc_many_query_tiles(b, d):
    """Several 128-row query tiles, causal positions, padding rows: tcgen05 path vs fp32 reference."""
    torch.manual_seed(5)
    n, queries = 700, 300
    q = torch.randn(1, queries, 3, d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, n, 3, d, device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    pos = torch.sort(torch.randint(0, n, (1, queries), device="cuda"), 1).values
    pos[0, 7] = -1
    q, k, v = (t.requires_grad_() for t in (q, k, v))
    out = dense_attention(q, k, v, pos, b, "cuda")
    rq, rk, rv = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = dense_attention(rq, rk, rv, pos, b, "torch")
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=5e-2)
    probe = torch.randn_like(ref)
    got = torch.autograd.grad((out.float() * probe).sum(), (q, k, v))
    want = torch.autograd.grad((ref * probe).sum(), (rq, rk, rv))
    for name, a, e in zip("qkv", got, want):
        scale = e.abs().max().item()
        torch.testing.assert_close(a.float(), e, atol=3e-2 * max(1.0, scale), rtol=5e-2, msg=name)


@pytest.mark.parametrize("b", [16, 32])
def test_gated_tc_at_the_training_length(b):
    """8,192 keys at head dim 64 (the stack_100m read): long key loops, the stale-max rescale,
    sorted positions with padding rows; forward and all three gradients against the fp32 reference."""
    torch.manual_seed(8)
    n, heads, d = 8192, 2, 64
    q = (torch.randn(1, n, heads, d, device="cuda") * 2).to(torch.bfloat16)
    k = (torch.randn(1, n, heads, d, device="cuda") * 2).to(torch.bfloat16)
    v = torch.randn(1, n, heads, d, device="cuda").to(torch.bfloat16)
    pos = torch.arange(n, device="cuda")[None].clone()
    pos[0, 4000:4100] = -1                                  # padding rows inside the sequence
    q, k, v = (t.requires_grad_() for t in (q, k, v))
    out = dense_attention(q, k, v, pos, b, "cuda")
    rq, rk, rv = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = dense_attention(rq, rk, rv, pos, b, "torch")
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=5e-2)
    probe = torch.randn_like(ref)
    got = torch.autograd.grad((out.float() * probe).sum(), (q, k, v))
    want = torch.autograd.grad((ref * probe).sum(), (rq, rk, rv))
    for name, a, e in zip("qkv", got, want):
        scale = e.abs().max().item()
        torch.testing.assert_close(a.float(), e, atol=3e-2 * max(1.0, scale), rtol=5e-2, msg=name)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,b,d,prev", [(37, 16, 64, False), (64, 16, 64, True), (100, 32, 32, True),
                                        (5, 8, 16, False), (130, 16, 128, True), (300, 16, 64, True),
                                        (1000, 16, 64, False), (129, 16, 64, True)])
def test_local_attention_matches_reference(n, b, d, prev, dtype):
    torch.manual_seed(3)
    heads, start = 3, 4 * b
    qkv = torch.randn(2, n, 3, heads, d, device="cuda", dtype=dtype, requires_grad=True)
    halo = torch.randn(2, b, 3, heads, d, device="cuda", dtype=dtype, requires_grad=True) if prev else None
    valid = start - b if prev else start
    out = fused.local_attention(qkv, halo, start, valid, n, b, heads, "cuda")
    r_qkv = qkv.detach().double().requires_grad_()
    r_halo = halo.detach().double().requires_grad_() if prev else None
    ref = fused.local_attention_reference(r_qkv, r_halo, start, valid, n, b, heads)
    probe = torch.randn_like(out)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(out.double(), ref, atol=atol, rtol=rtol)
    inputs = (qkv, halo) if prev else (qkv,)
    r_inputs = (r_qkv, r_halo) if prev else (r_qkv,)
    got = torch.autograd.grad((out * probe).sum(), inputs)
    want = torch.autograd.grad((ref * probe.double()).sum(), r_inputs)
    for a, e in zip(got, want):
        torch.testing.assert_close(a.double(), e, atol=atol * 4, rtol=rtol)


@pytest.mark.parametrize("prev", [False, True])
def test_local_tc_many_units_per_cta(prev):
    """The tensor-core local forward is persistent: with ~1,000 units of 128 rows every
    CTA runs several, so shared-memory stages and TMEM buffers are reused."""
    torch.manual_seed(11)
    b, d, heads, n, start = 16, 64, 16, 4100, 32
    qkv = torch.randn(2, n, 3, heads, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    halo = torch.randn(2, b, 3, heads, d, device="cuda", dtype=torch.bfloat16, requires_grad=True) if prev else None
    valid = start - b if prev else start
    out = fused.local_attention(qkv, halo, start, valid, n, b, heads, "cuda")
    r_qkv = qkv.detach().float().requires_grad_()
    r_halo = halo.detach().float().requires_grad_() if prev else None
    ref = fused.local_attention_reference(r_qkv, r_halo, start, valid, n, b, heads)
    atol, rtol = TOL[torch.bfloat16]
    torch.testing.assert_close(out.float(), ref, atol=atol, rtol=rtol)
    probe = torch.randn_like(out)
    inputs = (qkv, halo) if prev else (qkv,)
    r_inputs = (r_qkv, r_halo) if prev else (r_qkv,)
    got = torch.autograd.grad((out * probe).sum(), inputs)
    want = torch.autograd.grad((ref * probe.float()).sum(), r_inputs)
    for a, e in zip(got, want):
        torch.testing.assert_close(a.float(), e, atol=atol * 4, rtol=rtol)


@pytest.mark.parametrize("cols,rows", [(1000, 300), (1024, 517), (768, 64), (128, 3), (1536, 200)])
@pytest.mark.parametrize("dtype,out", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                       (torch.bfloat16, torch.bfloat16)])
def test_layer_norm(dtype, out, cols, rows, native):
    torch.manual_seed(0)
    x = torch.randn(rows, cols, device="cuda", dtype=dtype) * 3 + 1
    norm = torch.nn.LayerNorm(cols).cuda()
    torch.nn.init.normal_(norm.weight)
    torch.nn.init.normal_(norm.bias)
    xr = x.detach().float().requires_grad_()
    xn = x.detach().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=out == torch.bfloat16):
        y = fused.layer_norm(xn, norm, "cuda")
    assert y.dtype == out
    ref = torch.nn.functional.layer_norm(xr, (cols,), norm.weight, norm.bias, norm.eps)
    atol = 2e-5 if out == torch.float32 and dtype == torch.float32 else 3e-2
    torch.testing.assert_close(y.float(), ref, atol=atol, rtol=1e-2)
    g = torch.randn_like(ref)
    gx, gw, gb = torch.autograd.grad((y.float() * g).sum(), (xn, norm.weight, norm.bias))
    rx, rw, rb = torch.autograd.grad((ref * g).sum(), (xr, norm.weight, norm.bias))
    torch.testing.assert_close(gx.float(), rx, atol=atol * 10, rtol=2e-2)
    torch.testing.assert_close(gw, rw, atol=0.5 if out == torch.bfloat16 else 1e-3, rtol=2e-2)
    torch.testing.assert_close(gb, rb, atol=0.3 if out == torch.bfloat16 else 1e-3, rtol=1e-3)


def test_bias_gelu_and_cross_entropy(native):
    torch.manual_seed(1)
    h = torch.randn(257, 300, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    bias = torch.randn(300, device="cuda", requires_grad=True)
    out = fused._BiasGeluNative.apply(h, bias)
    hr, br = h.detach().float().requires_grad_(), bias.detach().clone().requires_grad_()
    ref = torch.nn.functional.gelu(hr + br)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    g = torch.randn_like(ref)
    a = torch.autograd.grad((out.float() * g).sum(), (h, bias))
    e = torch.autograd.grad((ref * g).sum(), (hr, br))
    torch.testing.assert_close(a[0].float(), e[0], atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(a[1], e[1], atol=0.3, rtol=2e-2)
    logits = torch.randn(77, 256, device="cuda", requires_grad=True)
    targets = torch.randint(256, (77,), device="cuda")
    targets[3] = -100
    loss, hits = fused.cross_entropy_sum(logits, targets, "cuda")
    ref = torch.nn.functional.cross_entropy(logits, targets, ignore_index=-100, reduction="sum")
    torch.testing.assert_close(loss, ref, atol=1e-4, rtol=1e-5)
    want_hits = (logits.argmax(-1) == targets) | (targets == -100)
    assert torch.equal(hits, want_hits)
    torch.testing.assert_close(torch.autograd.grad(loss * 0.5, logits)[0],
                               torch.autograd.grad(ref * 0.5, logits)[0], atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("tokens, vocab, dim", [(8192, 256, 1024), (8193 + 8192, 31, 64), (37, 300, 1028)])
def test_embedding_gradient_matches_torch(tokens, vocab, dim):
    torch.manual_seed(5)
    table = torch.nn.Embedding(vocab, dim, device="cuda")
    ids = torch.randint(vocab, (1, tokens), device="cuda")
    ids[0, : tokens // 3] = 3                      # one very frequent id
    g = torch.randn(1, tokens, dim, device="cuda")
    fused.embedding(ids, table, "cuda").backward(g)
    ours = table.weight.grad.clone()
    table.weight.grad = None
    table(ids).backward(g)
    torch.testing.assert_close(ours, table.weight.grad, atol=1e-4, rtol=1e-5)


def test_fused_adamw_matches_torch(native):
    from exploration_b200.runtime.optim import FusedAdamW
    torch.manual_seed(2)
    params = [torch.randn(s, device="cuda", requires_grad=True) for s in ((33, 17), (5000,), (3,))]
    clones = [p.detach().clone().requires_grad_() for p in params]
    ours = FusedAdamW(params, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    ref = torch.optim.AdamW(clones, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for _ in range(4):
        for p, c in zip(params, clones):
            g = torch.randn_like(p)
            p.grad, c.grad = g, g.clone()
        ours.step()
        ref.step()
    for p, c in zip(params, clones):
        torch.testing.assert_close(p, c, atol=1e-6, rtol=1e-5)
    norm = native.grad_sq_norm([p.grad for p in params])
    torch.testing.assert_close(norm, sum((p.grad ** 2).sum() for p in params), rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,b,d", [(129, 16, 32), (257, 32, 64), (385, 128, 128), (1000, 16, 64)])
def test_sparse_attention_matches_topk_oracle(n, b, d, dtype):
    q, k, v, pos = _dense_inputs(n, b, d, dtype)
    with torch.no_grad():
        expected = eager_attention(q.float(), k.float(), v.float(), pos, b, 2)
        actual = sparse_attention(q.detach(), TensorPages(k.detach(), v.detach(), 4 * b), pos, b, 2, "cuda",
                                  score_page_tokens=2 * b)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(actual.float(), expected, atol=atol, rtol=rtol)


def test_model_native_matches_torch_backend_bf16():
    torch.manual_seed(42)
    model = StackModel(128, 64, 4, 16, 64, "Lx2,(G)x2", backend="cuda", checkpoint_chunks=True,
                       encoder_chunk=32, pos_chunk=7).cuda()
    ref = copy.deepcopy(model)
    ref.set_backend("torch")
    ids = torch.randint(128, (2, 131), device="cuda")
    targets = torch.randint(128, ids.shape, device="cuda")
    sup = torch.rand(ids.shape, device="cuda") > 0.75
    with torch.autocast("cuda", dtype=torch.bfloat16):
        actual = model(ids, sup=sup, targets=targets)["loss_sum"]
        expected = ref(ids, sup=sup, targets=targets)["loss_sum"]
    torch.testing.assert_close(actual, expected, atol=0.1, rtol=0.003)
    actual.backward()
    expected.backward()
    for (name, a), (_, e) in zip(model.named_parameters(), ref.named_parameters()):
        if a.grad is not None:
            torch.testing.assert_close(a.grad, e.grad, atol=0.08, rtol=0.06, msg=name)


def test_model_fp32_native_matches_reference_tightly():
    torch.manual_seed(7)
    model = StackModel(64, 32, 2, 16, 64, "Lx2,G", backend="cuda", encoder_chunk=32).cuda()
    ref = copy.deepcopy(model)
    ref.set_backend("torch")
    ids = torch.randint(64, (2, 77), device="cuda")
    targets = torch.randint(64, ids.shape, device="cuda")
    a = model(ids, targets=targets)["loss_sum"]
    e = ref(ids, targets=targets)["loss_sum"]
    torch.testing.assert_close(a, e, atol=1e-3, rtol=1e-5)
    a.backward()
    e.backward()
    for (name, pa), (_, pe) in zip(model.named_parameters(), ref.named_parameters()):
        if pa.grad is not None:
            torch.testing.assert_close(pa.grad, pe.grad, atol=1e-4, rtol=1e-3, msg=name)


@pytest.mark.parametrize("keys,b,d,queries,topk,first", [(70000, 16, 64, 16, 64, 0), (4144, 32, 128, 5, 16, 64),
                                                          (1000, 16, 64, 32, 200, 32), (300, 16, 64, 3, 512, 0), (200000, 32, 64, 16, 64, 0)])
def test_block_scores_tc_matches_reference(native, keys, b, d, queries, topk, first):
    from exploration_b200.ops.sparse import block_scores_reference
    torch.manual_seed(5)
    heads = 3
    q = torch.randn(1, queries, heads, d, device="cuda").to(torch.bfloat16)
    k = torch.randn(1, keys, heads, d, device="cuda").to(torch.bfloat16)
    pos = torch.randint(first, first + keys + 3 * b, (1, queries), device="cuda")
    pos[0, 0] = -1
    pos = pos.to(torch.int32)
    assert native.block_scores_tc_supported(q, k, b, topk)
    scores, ids, zr = native.block_scores_topk_tc(q, k, pos, b, first, topk)
    ref = block_scores_reference(q.float(), k.float(), pos.long(), b, first)      # [B, Q, H, G]
    want_zr = ref.logsumexp(-1)
    count = min(topk, ref.shape[-1])
    want = ref.topk(count, -1).values
    finite = torch.isfinite(want)
    assert torch.equal(torch.isfinite(scores), finite)
    torch.testing.assert_close(scores[finite], want[finite], atol=2e-3, rtol=1e-4)
    got_at_ids = ref.gather(-1, ids - first // b)
    torch.testing.assert_close(got_at_ids[finite], scores[finite], atol=2e-3, rtol=1e-4)
    assert torch.equal(torch.isfinite(zr), torch.isfinite(want_zr))
    ok = torch.isfinite(want_zr)
    torch.testing.assert_close(zr[ok], want_zr[ok], atol=2e-3, rtol=1e-4)
    # descending order, ties by ascending block id
    assert bool((scores[..., 1:] <= scores[..., :-1]).all())


@pytest.mark.parametrize("tier", ["cuda", "cpu"])
def test_bf16_cast_model_inference_native(tier, tmp_path):
    """Evaluation casts the model to bf16 (norm/bias parameters included); the
    native inference path must accept it and agree with the fp32 model."""
    from exploration_b200 import ExecutionConfig, build_model
    from exploration_b200.runtime.inference import InferenceSession
    torch.manual_seed(11)
    options = {"model": "stack", "vocab_size": 128, "dim": 256, "heads": 4, "block_size": 16, "topk": 8,
               "arch": "Lx2,G", "ffn_ratio": 4.0}
    model = build_model(options, execution=ExecutionConfig(backend="cuda"), device="cuda").eval()
    ids = torch.randint(128, (1, 3000))
    pos = torch.tensor([[100, 1500, 2999]])
    mask = torch.zeros_like(ids, dtype=torch.bool).scatter_(1, pos, True)
    with torch.no_grad():
        expected = model(ids.cuda(), sup=mask.cuda(), compact=True).float()
        model.to(torch.bfloat16)
        with InferenceSession(model, cache=tier, cache_dir=str(tmp_path), page_tokens=1024) as session:
            session.prefill(ids, pos)
            actual = torch.cat([logits for _, logits, _ in session.iter_logits()], 1).float()
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual.cpu(), expected.cpu(), atol=0.3, rtol=0.1)


def test_native_backward_as_first_cuda_work_of_the_autograd_thread():
    """A fresh process whose first backward node is a native op: the autograd
    engine's device thread has no CUDA context yet when the op encodes its TMA
    tensor maps (which needs one). Runs in a subprocess so the thread is new."""
    import subprocess
    import sys
    code = (
        "import torch\n"
        "from exploration_b200.ops import fused\n"
        "qkv = torch.randn(1, 1024, 3, 16, 64, device='cuda').to(torch.bfloat16).requires_grad_()\n"
        "out = fused.local_attention(qkv, None, 0, 0, 1024, 16, 16, 'cuda')\n"
        "out.backward(torch.randn_like(out))\n"
        "torch.cuda.synchronize()\n"
        "print('ok', float(qkv.grad.float().abs().sum()) > 0)\n")
    for _ in range(3):
        proc = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
        assert proc.returncode == 0, proc.stderr[-2000:]
        assert "ok True" in proc.stdout
