"""Device timing of the NVLink-fused Ulysses exchange against its NCCL baseline.

``torchrun --nproc-per-node N -m exploration_b200.tools.ulysses_bench
[--config configs/stack_500m.json] [--length 65536]`` (one rank per GPU).

Every rank holds ``n_local = length / N`` tokens of width ``dim``; the ops are
the Stack G-round projections around the gated attention:

* ``q_scatter`` / ``kv_scatter``: the projection GEMM ``x W^T`` (``dim`` or
  ``2 dim`` outputs) whose epilogue stores each tile into the head owner's
  buffer over NVLink (``gemm_scatter``), followed by the heap barrier that
  publishes it: sequence layout in, head layout out.
* ``out_gather``: the output projection with the residual epilogue whose A
  operand is read tile by tile from the owners' head buffers (``gemm_gather``)
  after the barrier that makes them ready: head layout in, sequence layout out.
* ``out_landed``: the same direction as two kernels, the default in
  training: ``gather_rows`` pulls each remote row over NVLink once into a
  local buffer, then the tcgen05 GEMM with the residual epilogue reads it.
* ``*_nccl``: the baseline of each: the same GEMM (cuBLAS) plus
  ``all_to_all_single`` and the layout permutes (the reference's path,
  st/runtime/parallel.py:16-27).

Timing: CUDA events on the launching stream around ``--iterations`` calls
after ``--warmup``, median per call, max over ranks. Roofline per fused op
= max(FLOPs / measured bf16 GEMM peak, bytes this rank sends to (scatter)
or reads from (gather) other ranks / 770 GB/s, the measured peer-copy
bandwidth per direction); ``frac`` = roofline time / measured time.
Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

from ..ops import _native
from ..ops import gemm as G
from ..parallel.context import exchange
from ..parallel.ulysses import UlyssesFused

ROOT = Path(__file__).resolve().parents[2]
PEER_BYTES_PER_S = 770e9
FALLBACK_TFLOPS = 1590.0


def measured_tflops() -> float:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return FALLBACK_TFLOPS


def _time(fn, warmup: int, iterations: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    samples = []
    for _ in range(iterations):
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
    p.add_argument("--config", default=str(ROOT / "configs" / "stack_500m.json"))
    p.add_argument("--length", type=int, default=65536)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iterations", type=int, default=20)
    args = p.parse_args(argv)
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device)
    model = json.loads(Path(args.config).read_text())["model"]
    dim, heads = int(model["dim"]), int(model["heads"])
    hd = dim // heads
    n_local = args.length // world
    hpr = heads // world
    C = hpr * hd
    ext = _native.load(required=True)
    need = (3 * args.length * C + args.length * C) * 2 + (8 << 20)
    U = UlyssesFused(dist.group.WORLD, rank, world, device, need)
    heap = U.heap
    g = torch.Generator(device=device).manual_seed(rank)
    x = torch.randn(n_local, dim, device=device, generator=g).to(torch.bfloat16)
    w_q = (torch.randn(dim, dim, device=device, generator=g) * dim ** -0.5).to(torch.bfloat16)
    w_kv = (torch.randn(2 * dim, dim, device=device, generator=g) * dim ** -0.5).to(torch.bfloat16)
    w_o = (torch.randn(dim, dim, device=device, generator=g) * dim ** -0.5).to(torch.bfloat16)
    residual = torch.randn(n_local, dim, device=device, generator=g)
    out = torch.empty(n_local, dim, device=device)
    q_slot = heap.alloc(args.length * C * 2)
    kv_slot = heap.alloc(2 * args.length * C * 2)
    heads_slot = heap.alloc(args.length * C * 2)
    heap.tensor(heads_slot, [args.length * C]).normal_()
    heap.barrier()
    torch.cuda.synchronize()

    def q_scatter():
        ext.gemm_scatter(x, w_q, False, heap.peer_ptrs(q_slot), rank, 1, 1, n_local, C)
        heap.barrier()

    def kv_scatter():
        ext.gemm_scatter(x, w_kv, False, heap.peer_ptrs(kv_slot), rank, 2, 1, n_local, C)
        heap.barrier()

    def out_gather():
        heap.barrier()
        ext.gemm_gather(heap.peer_ptrs(heads_slot), rank, 1, 1, n_local, C, w_o, False, out,
                        G.BIAS_RESIDUAL, None, residual)

    landed = torch.empty(n_local, dim, device=device, dtype=torch.bfloat16)

    def out_landed():
        heap.barrier()
        ext.gather_rows(heap.peer_ptrs(heads_slot), rank, 1, 1, n_local, C, landed)
        G.gemm(landed, False, w_o, False, out, G.BIAS_RESIDUAL, residual=residual)

    def q_nccl():
        y = torch.mm(x, w_q.t()).view(1, n_local, heads, hd)
        return exchange(y, dist.group.WORLD, True)

    def kv_nccl():
        y = torch.mm(x, w_kv.t()).view(1, n_local, 2 * heads, hd)
        return exchange(y, dist.group.WORLD, True)

    heads_local = torch.randn(1, args.length, hpr, hd, device=device, generator=g).to(torch.bfloat16)

    def out_nccl():
        seq = exchange(heads_local, dist.group.WORLD, False).reshape(n_local, dim)
        return torch.mm(seq, w_o.t(), out_dtype=torch.float32) + residual

    def gemm_q_local():
        return torch.mm(x, w_q.t())

    ops = {"q_scatter": q_scatter, "q_nccl": q_nccl, "kv_scatter": kv_scatter, "kv_nccl": kv_nccl,
           "out_gather": out_gather, "out_landed": out_landed, "out_nccl": out_nccl,
           "q_gemm_local": gemm_q_local}
    times = {name: _time(fn, args.warmup, args.iterations) for name, fn in ops.items()}
    t = torch.tensor([times[k] for k in ops], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    times = dict(zip(ops, (float(v) for v in t)))
    peak = measured_tflops() * 1e12
    remote = (world - 1) / world

    def roofline(flops, bytes_remote):
        return max(flops / peak, bytes_remote / PEER_BYTES_PER_S) * 1e6      # us

    proj = {"q_scatter": (2 * n_local * dim * dim, n_local * dim * 2 * remote),
            "kv_scatter": (2 * n_local * dim * 2 * dim, n_local * 2 * dim * 2 * remote),
            "out_gather": (2 * n_local * dim * dim, n_local * dim * 2 * remote),
            "out_landed": (2 * n_local * dim * dim, n_local * dim * 2 * remote)}
    report = {"config": Path(args.config).stem, "length": args.length, "world": world, "n_local": n_local,
              "dim": dim, "heads": heads, "peak_tflops": peak / 1e12, "peer_gbs": PEER_BYTES_PER_S / 1e9,
              "us_max_over_ranks": {k: round(v, 1) for k, v in times.items()}}
    for name, (flops, nbytes) in proj.items():
        roof = roofline(flops, nbytes)
        base = name.split("_")[0] + "_nccl"
        report[name] = {"roofline_us": round(roof, 1), "frac": round(roof / times[name], 3),
                        "speedup_vs_nccl": round(times[base] / times[name], 2),
                        "gflop": round(flops / 1e9, 2), "remote_mb": round(nbytes / 1e6, 2)}
    report["device_errors"] = list(ext.device_errors(device.index))
    if rank == 0:
        print(json.dumps(report), flush=True)
    U.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
