"""Fused Ulysses GEMMs (peer scatter / peer gather) and the peer barrier.

The kernels take one pointer per rank. Here every "rank" buffer lives on the
one visible GPU and the ranks run one after another: the GEMMs never wait on
each other, so this checks the layout arithmetic for 2/4/8 ranks against an
fp32 torch reference of ``to_heads(x W^T)`` and ``to_sequence(h) W^T``.
The barrier test gives a two-rank barrier a peer that never arrives and
checks that the bounded wait reports the timeout and the context stays usable.
"""
import pytest
import torch

from exploration_b200.ops import gemm as G

pytestmark = pytest.mark.gpu

SITE_PEER = 9


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("world,parts,batch,n_local,hpr,hd", [
    (2, 1, 1, 256, 2, 64), (4, 2, 1, 128, 1, 64), (8, 2, 2, 128, 2, 64), (2, 3, 1, 200, 3, 32)])
@pytest.mark.parametrize("b_mn", [False, True])
def test_scatter_gemm(native, world, parts, batch, n_local, hpr, hd, b_mn):
    C = hpr * hd
    dim = world * C
    k = 192
    w = _rand((parts * dim, k), 1, 0.1)
    w_st = w.t().contiguous() if b_mn else w
    bufs = [torch.zeros(parts, batch, world * n_local, C, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    xs = [_rand((batch * n_local, k), 10 + r) for r in range(world)]
    for r in range(world):
        native.gemm_scatter(xs[r], w_st, b_mn, [b.data_ptr() for b in bufs], r, parts, batch, n_local, C)
    torch.cuda.synchronize()
    for r in range(world):
        y = (xs[r].float() @ w.float().t()).view(batch, n_local, parts, world, C)
        for s in range(world):
            got = bufs[s][:, :, r * n_local:(r + 1) * n_local].float()
            want = y[:, :, :, s].permute(2, 0, 1, 3)
            torch.testing.assert_close(got, want, atol=3e-2, rtol=2e-2)
    assert native.device_errors(0) == (0, 0)


@pytest.mark.parametrize("world,parts,batch,n_local,hpr", [(2, 1, 1, 256, 1), (4, 2, 2, 128, 2), (8, 1, 1, 128, 2)])
@pytest.mark.parametrize("b_mn", [False, True])
def test_gather_gemm(native, world, parts, batch, n_local, hpr, b_mn):
    hd = 64
    C = hpr * hd
    kdim = parts * world * C
    n_out = 320
    bufs = [_rand((parts, batch, world * n_local, C), 20 + s) for s in range(world)]
    w = _rand((n_out, kdim), 3, 0.05)
    w_st = w.t().contiguous() if b_mn else w
    bias = torch.randn(n_out, device="cuda")
    for r in range(world):
        a = torch.stack([b[:, :, r * n_local:(r + 1) * n_local] for b in bufs], 0)      # [world, parts, B, n, C]
        a = a.permute(2, 3, 1, 0, 4).reshape(batch * n_local, kdim).float()             # k = (part, owner, c)
        ref = a @ w.float().t()
        out = torch.empty(batch * n_local, n_out, device="cuda", dtype=torch.bfloat16)
        native.gemm_gather([b.data_ptr() for b in bufs], r, parts, batch, n_local, C, w_st, b_mn, out,
                           G.STORE_BF16, None, None)
        torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=2e-2)
        res = torch.randn(batch * n_local, n_out, device="cuda")
        out32 = torch.empty_like(res)
        native.gemm_gather([b.data_ptr() for b in bufs], r, parts, batch, n_local, C, w_st, b_mn, out32,
                           G.BIAS_RESIDUAL, bias, res)
        torch.testing.assert_close(out32, ref + bias + res, atol=2e-2, rtol=2e-3)
        seq = torch.empty(batch * n_local, kdim, device="cuda", dtype=torch.bfloat16)
        native.gather_rows([b.data_ptr() for b in bufs], r, parts, batch, n_local, C, seq)
        torch.testing.assert_close(seq.float(), a, atol=0, rtol=0)
    assert native.device_errors(0) == (0, 0)


def test_heap_views_and_single_rank_barrier(native):
    base = native.heap_alloc(1 << 20, 0)
    try:
        start = native.heap_signal_bytes()
        view = native.heap_tensor(base, start, [4, 8], torch.bfloat16, 0)
        view.fill_(3.0)
        again = native.heap_tensor(base, start, [32], torch.bfloat16, 0)
        assert float(again.float().sum()) == 96.0
        for _ in range(3):
            native.heap_barrier([base], 0, 1.0)
        torch.cuda.synchronize()
        assert native.device_errors(0) == (0, 0)
    finally:
        native.heap_free(base, 0)


def test_barrier_times_out_without_peer(native):
    """Rank 1 never arrives: the wait runs out, reports the peer site and returns."""
    bases = [native.heap_alloc(1 << 16, 0), native.heap_alloc(1 << 16, 0)]
    try:
        native.heap_barrier(bases, 0, 0.2)
        torch.cuda.synchronize()
        code, _ = native.device_errors(0)
        assert code == SITE_PEER
        # The context stays usable and the slot was cleared by the read.
        x = torch.ones(1024, device="cuda")
        assert float(x.sum()) == 1024.0
        assert native.device_errors(0) == (0, 0)
    finally:
        for b in bases:
            native.heap_free(b, 0)
