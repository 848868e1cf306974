"""Operator latency and memory: ``python -m st benchmark``.

``dense`` times the gated attention forward + backward over all (or
``--queries``) positions; ``sparse`` times paged exact scoring + top-k +
pop, forward only. Inputs are N(0,1) from seed 42, TF32 is off, positions
are evenly spaced (dense from 0, sparse over the last ``queries`` tokens).
Each iteration is timed with CUDA events on the launching stream after
warm-up; the report holds the median/min, all samples, peak memory and the
native kernel record (reference: st/tools/benchmark.py:73-172).

Backends: ``cuda`` (native sm_100a kernels; ``triton`` is accepted as a
synonym for command compatibility), ``torch`` (bounded reference) and
``eager`` (materialises Q x N; small sizes only).
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import torch

from ..ops.attention import dense_attention
from ..ops.gated_reference import eager_gated
from ..ops.launch import launch_report
from ..ops.sparse import TensorPages, sparse_attention
from ..runtime.memory import GiB

ROLES = {"eager": "Q x N algebra (materialises the full score matrix)",
         "torch": "bounded-memory fp32 reference / oracle",
         "cuda": "native sm_100a kernels"}


def parser():
    p = argparse.ArgumentParser(prog="python -m st benchmark", description=__doc__, allow_abbrev=False,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--compare", action="store_true", help="same inputs through every backend")
    p.add_argument("--operation", choices=["dense", "sparse"], default="dense")
    p.add_argument("--backend", choices=["cuda", "triton", "torch", "eager"], default="cuda")
    p.add_argument("--length", type=int, default=512)
    p.add_argument("--queries", type=int, default=0, help="0 = all for dense, 16 for sparse")
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--heads", type=int, default=4)
    p.add_argument("--head-dim", type=int, default=64)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--topk", type=int, default=64)
    p.add_argument("--q-chunk", type=int, default=0, help="torch-reference query tile (0 = default)")
    p.add_argument("--kv-chunk", type=int, default=0, help="torch-reference KV tile (0 = default)")
    p.add_argument("--precision", choices=["fp32", "bf16"], default="bf16")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--iterations", type=int, default=10)
    p.add_argument("--page-tokens", type=int, default=65536)
    p.add_argument("--output", default="", help="JSON path (default runs/benchmarks/...)")
    return p


def measure(args) -> dict:
    p = parser()
    if not torch.cuda.is_available():
        p.error("benchmark requires an NVIDIA GPU")
    backend = "cuda" if args.backend == "triton" else args.backend
    if min(args.length, args.batch_size, args.heads, args.head_dim, args.block_size, args.iterations,
           args.topk) < 1 or args.warmup < 1 or min(args.queries, args.q_chunk, args.kv_chunk) < 0 \
            or args.page_tokens < args.block_size:
        p.error("sizes/iterations/warmup must be positive, queries/chunks >= 0, "
                "page_tokens >= block_size")
    queries = args.queries or (args.length if args.operation == "dense" else min(16, args.length))
    if queries > args.length:
        p.error("queries must not exceed length")
    if args.operation == "sparse" and backend == "eager":
        p.error("use torch as the paged sparse reference")
    if backend == "eager":
        free, _ = torch.cuda.mem_get_info()
        if args.batch_size * queries * args.heads * args.length * 4 * 12 > free * 0.7:
            p.error("eager Q x N estimate exceeds the GPU budget; reduce length/queries")
    torch.manual_seed(42)
    torch.backends.cuda.matmul.allow_tf32 = False
    dtype = torch.bfloat16 if args.precision == "bf16" else torch.float32
    grad = args.operation == "dense"
    q = torch.randn(args.batch_size, queries, args.heads, args.head_dim, device="cuda", dtype=dtype,
                    requires_grad=grad)
    k = torch.randn(args.batch_size, args.length, args.heads, args.head_dim, device="cuda",
                    dtype=dtype, requires_grad=grad)
    v = torch.randn_like(k, requires_grad=grad)
    first = 0 if args.operation == "dense" else args.length - queries
    positions = torch.linspace(first, args.length - 1, queries, device="cuda").round().long()
    positions = positions[None].expand(args.batch_size, -1).contiguous()
    probe = torch.randn_like(q)
    pages = TensorPages(k, v, max(args.block_size, args.page_tokens // args.block_size * args.block_size))
    chunks = {name: size for name, size in (("q_chunk", args.q_chunk), ("kv_chunk", args.kv_chunk))
              if size}

    def iteration():
        if args.operation == "dense":
            q.grad = k.grad = v.grad = None
            if backend == "eager":
                out = eager_gated(q, k, v, positions, args.block_size)
            else:
                out = dense_attention(q, k, v, positions, args.block_size, backend, **chunks)
            out.backward(probe)
            return out
        return sparse_attention(q, pages, positions, args.block_size, args.topk, backend)

    for _ in range(args.warmup):
        iteration()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    samples = []
    for _ in range(args.iterations):
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record()
        iteration()
        end.record()
        end.synchronize()
        samples.append(begin.elapsed_time(end))
    ordered = sorted(samples)
    flops = None
    if args.operation == "dense":
        visible = float(positions.float().add(1).sum()) * args.heads      # (query, key) pairs
        flops = visible * args.head_dim * 2 * 2 * 3.5                     # fwd (2 GEMMs) + bwd (5)
    from .validate import environment
    return {"environment": environment(), "config": vars(args), "queries": queries,
            "role": ROLES[backend], "includes_backward": grad,
            "latency_ms_median": ordered[len(ordered) // 2], "latency_ms_min": ordered[0],
            "latency_ms_samples": samples,
            "model_tflops_per_s": (flops / (ordered[len(ordered) // 2] * 1e-3) / 1e12) if flops else None,
            "peak_allocated_gib": torch.cuda.max_memory_allocated() / GiB,
            "peak_reserved_gib": torch.cuda.max_memory_reserved() / GiB,
            "kernel_launches": launch_report()}


def main(argv=None):
    args = parser().parse_args(argv)
    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        parser().error("the operator benchmark runs on one GPU; use train for distributed throughput")
    if args.compare:
        backends = ["eager", "torch", "cuda"] if args.operation == "dense" else ["torch", "cuda"]
    else:
        backends = [args.backend]
    reports = []
    for backend in backends:
        case = argparse.Namespace(**{**vars(args), "backend": backend})
        torch.cuda.empty_cache() if torch.cuda.is_available() else None
        report = measure(case)
        reports.append(report)
        print(f"{backend}: median={report['latency_ms_median']:.3f} ms, "
              f"peak allocated={report['peak_allocated_gib']:.3f} GiB", flush=True)
    result = {"comparison": reports} if args.compare else reports[0]
    label = "compare" if args.compare else args.backend
    path = Path(args.output or f"runs/benchmarks/{args.operation}-{label}.json")
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(result, indent=2, default=str) + "\n")
    print(f"Report: {path}", flush=True)
    return result

