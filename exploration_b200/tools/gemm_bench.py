"""GEMM timings at the training shapes: the tcgen05 kernel per tile shape against cuBLAS.

``python -m exploration_b200.tools.gemm_bench`` times, for each GEMM of one
stack_100m layer at 8,192 tokens (forward ``x W^T``, input gradient ``dy W``
and weight gradient ``dy^T x`` of the QKV, output and FFN projections), the
kernel with each tile shape (128 x 128, 128 x 256, 256 x 256 on a CTA pair,
and the cost model's choice with its K split) and ``torch.mm`` (cuBLAS) on
the same operands. Each sample is one launch between CUDA events with a
256 MB buffer written before it, so operands come from HBM as they do inside
a training step; the median of ``--iterations`` samples is reported in
microseconds and TFLOP/s. ``--once SHAPE`` runs one GEMM once (for a profiler
with a kernel filter).
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops import _native
from ..ops import gemm as G

SHAPE_NAMES = {G.NARROW: "128x128", G.WIDE: "128x256", G.PAIR: "256x256 pair", G.AUTO: "auto"}


def cases(tokens: int, dim: int, hidden: int):
    """(name, M, N, K, a_mn, b_mn, fp32 accumulate) of the training GEMMs."""
    out = []
    for layer, n_out, n_in in (("qkv", 3 * dim, dim), ("out", dim, dim), ("ffn1", hidden, dim), ("ffn2", dim, hidden)):
        out.append((f"{layer}.fwd", tokens, n_out, n_in, False, False, False))
        out.append((f"{layer}.dgrad", tokens, n_in, n_out, False, True, False))
        out.append((f"{layer}.wgrad", n_out, n_in, tokens, True, True, True))
    return out


def operands(M, N, K, a_mn, b_mn, accumulate):
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn((K, M) if a_mn else (M, K), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), device="cuda", generator=g).to(torch.bfloat16)
    out = torch.zeros(M, N, device="cuda", dtype=torch.float32 if accumulate else torch.bfloat16)
    return a, b, out


def library(a, a_mn, b, b_mn, out, accumulate):
    lhs = a.t() if a_mn else a
    rhs = b if b_mn else b.t()
    if accumulate:
        torch.addmm(out, lhs, rhs, out_dtype=torch.float32, out=out)
    else:
        torch.mm(lhs, rhs, out=out)


def timed(fn, flush, warmup, iterations):
    for _ in range(warmup):
        fn()
    samples = []
    for _ in range(iterations):
        flush.add_(1)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1e3)
    samples.sort()
    return samples[len(samples) // 2]


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--dim", type=int, default=1024)
    p.add_argument("--hidden", type=int, default=4096)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iterations", type=int, default=20)
    p.add_argument("--once", default="", help="run this case (e.g. qkv.fwd) once with the planned shape")
    p.add_argument("--shape", type=int, default=G.AUTO, help="tile shape for --once (0 auto, 1, 2, 3)")
    args = p.parse_args(argv)
    ext = _native.load(required=True)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    flush = torch.empty(64 << 20, device="cuda", dtype=torch.float32)
    for name, M, N, K, a_mn, b_mn, acc in cases(args.tokens, args.dim, args.hidden):
        if args.once and name != args.once:
            continue
        a, b, out = operands(M, N, K, a_mn, b_mn, acc)
        if args.once:
            G.plain(a, a_mn, b, b_mn, out, accumulate=acc, shape=args.shape)
            torch.cuda.synchronize()
            print(f"{name} ok errors={ext.device_errors(0)}", flush=True)
            return
        flops = 2.0 * M * N * K
        row = {"case": name, "M": M, "N": N, "K": K, "plan": ext.gemm_plain_plan(M, N, K, sms)}
        for shape in (G.AUTO, G.NARROW, G.WIDE, G.PAIR):
            us = timed(lambda: G.plain(a, a_mn, b, b_mn, out, accumulate=acc, shape=shape), flush, args.warmup,
                       args.iterations)
            row[SHAPE_NAMES[shape]] = {"us": round(us, 1), "tflops": round(flops / us / 1e6, 1)}
        us = timed(lambda: library(a, a_mn, b, b_mn, out, acc), flush, args.warmup, args.iterations)
        row["cublas"] = {"us": round(us, 1), "tflops": round(flops / us / 1e6, 1)}
        print(json.dumps(row), flush=True)
    print(json.dumps({"device_errors": list(ext.device_errors(0))}))


if __name__ == "__main__":
    main()
