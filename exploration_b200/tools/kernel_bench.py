"""Kernel-level timings of the attention and GEMM paths at training shapes.

``python -m exploration_b200.tools.kernel_bench`` prints CUDA-event timings
(median of ``--iterations`` after ``--warmup``) of the local window
attention, the gated dense attention and the fused-epilogue FFN GEMMs
(bias+GELU, bias+residual, GELU backward; dim = heads * head_dim, hidden
4 * dim) for one
sequence of the chosen shape (default: stack_100m, 8192 tokens, 16 heads of
64). ``--once`` runs every op exactly once (forward and backward) and
prints a marker after each: the small, short-lived program to put under a
profiler with a kernel filter.
"""
from __future__ import annotations

import argparse
import faulthandler
import json
import os

import torch

from ..ops import _native, fused
from ..ops.attention import dense_attention


def _time(fn, warmup, iterations):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    samples = []
    for _ in range(iterations):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end))
    samples.sort()
    return samples[len(samples) // 2]


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--length", type=int, default=8192)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--head-dim", type=int, default=64)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iterations", type=int, default=10)
    p.add_argument("--once", action="store_true", help="run each op once (profiling) instead of timing")
    args = p.parse_args(argv)
    if not torch.cuda.is_available():
        p.error("kernel_bench needs a CUDA device")
    faulthandler.enable()
    ext = _native.load()
    torch.manual_seed(0)
    n, H, D, b = args.length, args.heads, args.head_dim, args.block_size
    qkv = torch.randn(1, n, 3, H, D, device="cuda").to(torch.bfloat16).requires_grad_()
    g_local = torch.randn(1, n, H * D, device="cuda").to(torch.bfloat16)
    q, k, v = (torch.randn(1, n, H, D, device="cuda").to(torch.bfloat16).requires_grad_() for _ in range(3))
    pos = torch.arange(n, device="cuda")[None]
    g_gated = torch.randn(1, n, H, D, device="cuda").to(torch.bfloat16)

    def local_fwd():
        with torch.no_grad():
            return fused.local_attention(qkv, None, 0, 0, n, b, H, "cuda")

    def local_fwd_bwd():
        return torch.autograd.grad(fused.local_attention(qkv, None, 0, 0, n, b, H, "cuda"), qkv, g_local)

    def gated_fwd():
        with torch.no_grad():
            return dense_attention(q, k, v, pos, b, "cuda")

    def gated_fwd_bwd():
        return torch.autograd.grad(dense_attention(q, k, v, pos, b, "cuda"), (q, k, v), g_gated)

    from ..ops import gemm as G
    dim = H * D
    ffn = torch.nn.Sequential(torch.nn.Linear(dim, 4 * dim), torch.nn.GELU(), torch.nn.Linear(4 * dim, dim)).cuda()
    h_in = torch.randn(1, n, dim, device="cuda").to(torch.bfloat16).requires_grad_()
    y_in = torch.randn(1, n, dim, device="cuda", requires_grad=True)
    g_ffn = torch.randn(1, n, dim, device="cuda")

    def ffn_fwd():
        with torch.no_grad():
            return G.FFNResidual.apply(h_in, y_in, ffn[0].weight, ffn[0].bias, ffn[2].weight, ffn[2].bias)

    def ffn_fwd_bwd():
        out = G.FFNResidual.apply(h_in, y_in, ffn[0].weight, ffn[0].bias, ffn[2].weight, ffn[2].bias)
        return torch.autograd.grad(out, (h_in, y_in, ffn[0].weight, ffn[2].weight), g_ffn)

    ops = {"local_fwd": local_fwd, "local_fwd_bwd": local_fwd_bwd, "gated_fwd": gated_fwd,
           "gated_fwd_bwd": gated_fwd_bwd, "ffn_fwd": ffn_fwd, "ffn_fwd_bwd": ffn_fwd_bwd}
    if args.once:
        for name, fn in ops.items():
            fn()
            torch.cuda.synchronize()
            print(f"{name} ok errors={ext.device_errors(torch.cuda.current_device())}", flush=True)
        return
    result = {name + "_ms": round(_time(fn, args.warmup, args.iterations), 4) for name, fn in ops.items()}
    result["shape"] = {"length": n, "heads": H, "head_dim": D, "block": b}
    print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
