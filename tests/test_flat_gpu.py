"""Flat AdamW kernels and the CUDA-graph training step on a B200."""
import copy

import pytest
import torch

from exploration_b200 import ExecutionConfig, ParallelContext, build_model
from exploration_b200.cli import parse_args
from exploration_b200.runtime.engine import Trainer, lr_factor, make_batch
from exploration_b200.runtime.flat import GraphTrainer, _TorchFlat

pytestmark = pytest.mark.gpu


def test_flat_adamw_matches_torch_formula(native):
    n = 4096 * 37
    g = torch.Generator(device="cuda").manual_seed(0)
    p = torch.randn(n, device="cuda", generator=g)
    grad = torch.randn(n, device="cuda", generator=g)
    m = torch.randn(n, device="cuda", generator=g).abs() * 0.1
    v = torch.rand(n, device="cuda", generator=g) * 0.01
    shadow = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    hyper = torch.tensor([1e-3, 7.0, 0.5, 0.0], device="cuda")
    native.flat_sq_norm(grad, hyper)
    torch.testing.assert_close(hyper[3], grad.double().pow(2).sum().float(), rtol=1e-5, atol=0)
    ref = [t.cpu().clone() for t in (p, grad, m, v)]
    ref_hyper = hyper.cpu().clone()
    check = torch.tensor(1.0, device="cuda")
    native.flat_adamw(p, grad, m, v, shadow, hyper, check, 0.9, 0.95, 1e-8, 0.1)
    _TorchFlat.flat_adamw(ref[0], ref[1], ref[2], ref[3], None, ref_hyper, torch.tensor(1.0), 0.9, 0.95, 1e-8, 0.1)
    torch.testing.assert_close(p.cpu(), ref[0], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m.cpu(), ref[2], rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(v.cpu(), ref[3], rtol=1e-5, atol=1e-9)
    torch.testing.assert_close(shadow.float(), p.to(torch.bfloat16).float(), rtol=0, atol=0)
    # A non-finite loss skips the update entirely.
    before = p.clone()
    native.flat_adamw(p, grad, m, v, shadow, hyper, torch.tensor(float("nan"), device="cuda"),
                      0.9, 0.95, 1e-8, 0.1)
    assert torch.equal(p, before)


def _args(length):
    return parse_args(["train", "--dim", "256", "--heads", "4", "--block-size", "16", "--arch", "Lx2,G",
                       "--task", "random", "--length", str(length), "--batch-size", "1", "--precision", "bf16",
                       "--backend", "cuda", "--steps", "6", "--save", "", "--no-checkpoint-chunks",
                       "--clip-grad", "1.0"])


def test_graph_trainer_matches_eager(native):
    args = _args(1024)
    torch.manual_seed(0)
    options = {"model": "stack", "vocab_size": 256, "dim": 256, "heads": 4, "block_size": 16, "topk": 8,
               "arch": "Lx2,G", "ffn_ratio": 4.0}
    base = build_model(options, execution=ExecutionConfig(backend="cuda"), device="cuda")
    eager_model, graph_model = copy.deepcopy(base), copy.deepcopy(base)
    parallel = ParallelContext()
    eager = Trainer(args, eager_model, parallel)
    graph = GraphTrainer(args, graph_model, parallel)
    gen_a, gen_b = torch.Generator().manual_seed(3), torch.Generator().manual_seed(3)
    try:
        for step in range(args.steps):
            lr = args.lr * lr_factor(step, args.steps)
            eager.optimizer.zero_grad(set_to_none=True)
            for group in eager.optimizer.param_groups:
                group["lr"] = lr
            ids, target, mask, _ = make_batch(args, gen_a)
            a = eager.micro_step(ids, target, mask, last=True).cpu()
            eager.finish_step()
            ids, target, mask, _ = make_batch(args, gen_b)
            b, norm = graph.step(ids, target, mask, lr)
            assert norm > 0
            torch.testing.assert_close(b[0] / b[1], a[0] / a[1], rtol=2e-2, atol=2e-2)
        assert graph.graph is not None and graph.graph_launches > 0
        for p, q in zip(eager_model.parameters(), graph_model.parameters()):
            torch.testing.assert_close(q, p, rtol=5e-2, atol=5e-3)
    finally:
        graph.close()
    assert native.device_errors(0) == (0, 0)


def test_peer_reduction_kernels_single_rank(native):
    """The peer-memory reduction kernels on one rank: scale, norm partials, epochs, shadow stores."""
    from exploration_b200.parallel.symmetric import SymmetricHeap
    n, ctas = 64 * 1000, 32
    heap = SymmetricHeap(None, torch.device("cuda", 0), n * 6 + native.grad_flag_bytes() + (1 << 16))
    try:
        goff = heap.alloc(n * 4)
        soff = heap.alloc(n * 2)
        foff = heap.alloc(native.grad_flag_bytes())
        grad = heap.tensor(goff, [n], torch.float32)
        shadow = heap.tensor(soff, [n], torch.bfloat16)
        g = torch.Generator(device="cuda").manual_seed(1)
        partial = torch.zeros(2 * ctas, device="cuda")
        hyper = torch.tensor([1e-3, 1.0, 0.0, 0.0], device="cuda")
        for step in range(3):                      # epochs advance on every exchange
            src = torch.randn(n, device="cuda", generator=g)
            grad.copy_(src)
            bounds = [(0, 64 * 400), (64 * 400, n)]
            for b in (1, 0):
                lo, hi = bounds[b]
                native.grad_reduce_bucket([heap.base + goff], [heap.base + foff], 0, b, lo, hi, hi - lo, b == 0,
                                          0.5, partial[b * ctas:(b + 1) * ctas], 5.0)
            native.grad_norm_exchange(partial, [heap.base + foff], 0, hyper, 5.0)
            torch.cuda.synchronize()
            torch.testing.assert_close(grad, src * 0.5, rtol=0, atol=0)
            torch.testing.assert_close(hyper[3], (src * 0.5).double().pow(2).sum().float(), rtol=1e-5, atol=0)
        # AdamW with the shadow stored through the peer table equals the local kernel.
        p = torch.randn(n, device="cuda", generator=g)
        m = torch.zeros(n, device="cuda")
        v = torch.zeros(n, device="cuda")
        p2, m2, v2 = p.clone(), m.clone(), v.clone()
        local_shadow = torch.empty(n, device="cuda", dtype=torch.bfloat16)
        native.flat_adamw_peer(p, grad, m, v, [heap.base + soff], 0, hyper, None, 0.9, 0.95, 1e-8, 0.1)
        native.flat_adamw(p2, grad, m2, v2, local_shadow, hyper, None, 0.9, 0.95, 1e-8, 0.1)
        torch.cuda.synchronize()
        assert torch.equal(p, p2) and torch.equal(m, m2) and torch.equal(v, v2)
        assert torch.equal(shadow, local_shadow)
        assert native.device_errors(0) == (0, 0)
    finally:
        heap.close()
