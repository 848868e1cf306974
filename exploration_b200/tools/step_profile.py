"""Where a training step's device time goes, per phase, at N GPUs (max over ranks).

Run as one process per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m exploration_b200.tools.step_profile --steps 5 --warmup 3

It trains the benchmark workload (stack_100m, 8,192 tokens, CP = N, CUDA-graph
step, NVLink exchange and peer gradient reduction when N > 1) and records the
timed steps with the CUDA profiler (kernels replayed from the graph
included). Every kernel is put in one phase by its name:

* ``ulysses_scatter``: projection GEMMs whose epilogue stores head shards to their owners;
* ``ulysses_gather``: remote rows landed for the output projection (and the in-GEMM gather);
* ``heap_barrier``: symmetric-heap barriers between exchange phases (also counted);
* ``grad_reduce``: the peer-memory gradient reduction and norm exchange;
* ``gemm``: every other tcgen05 GEMM (and the split-K reduce);
* ``gated_attention``, ``local_attention``, ``norm`` (LayerNorm, column sums), ``loss``,
  ``optimizer``, ``nccl``, ``other``.

Rank 0 prints one JSON line: the step time (CUDA events, max over ranks) and,
per phase, kernel microseconds per step and launches per step (max over
ranks). Kernels of the gradient reduction run on a side stream under the
backward, so phase times add up to more than the step time.
"""
from __future__ import annotations

import argparse
import json
import os
import re
from pathlib import Path

import torch
import torch.distributed as dist

PHASES = ("ulysses_scatter", "ulysses_gather", "heap_barrier", "grad_reduce", "gemm", "gated_attention",
          "local_attention", "norm", "loss", "optimizer", "nccl", "other")
_GEMM_ARGS = re.compile(r"gemm_tc_kernel<(\d+), (\w+), (\w+), (\d+), (\w+)(?:, (\d))?>")


def phase_of(name: str) -> str:
    gemm = _GEMM_ARGS.search(name)
    if gemm:
        epilogue, gather = int(gemm.group(4)), gemm.group(5) in ("1", "true")
        if epilogue == 6:
            return "ulysses_scatter"
        return "ulysses_gather" if gather else "gemm"
    table = (("gather_rows", "ulysses_gather"), ("heap_barrier", "heap_barrier"), ("grad_reduce", "grad_reduce"),
             ("grad_norm_exchange", "grad_reduce"), ("splitk_reduce", "gemm"), ("gated_", "gated_attention"),
             ("delta_rho", "gated_attention"), ("tile_bounds", "gated_attention"), ("local", "local_attention"),
             ("ln_", "norm"), ("layer_norm", "norm"), ("column_", "norm"), ("cast_colsum", "norm"),
             ("cross_entropy", "loss"), ("adamw", "optimizer"), ("flat_", "optimizer"), ("nccl", "nccl"))
    for key, phase in table:
        if key in name:
            return phase
    return "other"


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--length", type=int, default=8192)
    p.add_argument("--config", default=str(Path(__file__).resolve().parents[2] / "configs" / "stack_100m.json"))
    p.add_argument("--top", type=int, default=0, help="also print this rank-0 count of the costliest kernels")
    args = p.parse_args(argv)

    from .. import ExecutionConfig, ParallelContext, build_model
    from ..cli import parse_args as cli_args
    from ..runtime.engine import lr_factor, make_batch
    from ..runtime.flat import GraphTrainer

    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local_rank)
    targs = cli_args(["train", "--config", args.config, "--task", "random", "--length", str(args.length),
                      "--batch-size", "1", "--precision", "bf16", "--backend", "cuda", "--context-parallel",
                      str(world), "--steps", str(args.warmup + args.steps), "--save", "", "--log-every",
                      "1000000", "--no-checkpoint-chunks"])
    parallel = ParallelContext.initialize(world, "cuda")
    device = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    options = {k: getattr(targs, k) for k in ("vocab_size", "dim", "heads", "block_size", "topk", "arch", "ffn_ratio")}
    execution = ExecutionConfig(backend="cuda", checkpoint_chunks=False, encoder_chunk=targs.encoder_chunk,
                                query_chunk=targs.query_chunk, loss_chunk=targs.loss_chunk)
    model = build_model({"model": "stack", **options}, execution=execution, device=device)
    model.train()
    parallel.attach_fused(device, max(512 << 20, parallel.fused_heap_bytes(model, 1, args.length)))
    trainer = GraphTrainer(targs, model, parallel)
    generator = torch.Generator().manual_seed(100 + parallel.dp_rank)

    def step(index):
        ids, target, mask, _ = make_batch(targs, generator)
        trainer.step(ids, target, mask, targs.lr * lr_factor(index, targs.steps))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        start.record()
        for i in range(args.steps):
            step(args.warmup + i)
        end.record()
        torch.cuda.synchronize()
    step_ms = start.elapsed_time(end) / args.steps
    totals = {name: [0.0, 0] for name in PHASES}
    kernels = {}
    for event in prof.events():
        if event.device_type != torch.autograd.DeviceType.CUDA:
            continue
        us = event.device_time_total if hasattr(event, "device_time_total") else event.cuda_time_total
        slot = totals[phase_of(event.name)]
        slot[0] += us
        slot[1] += 1
        entry = kernels.setdefault(event.name[:100], [0.0, 0])
        entry[0] += us
        entry[1] += 1
    values = torch.tensor([step_ms] + [totals[n][0] / args.steps for n in PHASES]
                          + [totals[n][1] / args.steps for n in PHASES], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(values, op=dist.ReduceOp.MAX)
    values = values.tolist()
    if parallel.rank == 0:
        phases = {name: {"us_per_step": round(values[1 + i], 1), "launches_per_step": round(values[1 + len(PHASES) + i], 1)}
                  for i, name in enumerate(PHASES) if values[1 + len(PHASES) + i] > 0}
        print(json.dumps({"n_gpus": world, "step_ms_max_over_ranks": round(values[0], 3),
                          "tokens_per_s": round(args.length * parallel.dp_size / values[0] * 1e3, 1),
                          "phases_max_over_ranks": phases}), flush=True)
        ranked = sorted(kernels.items(), key=lambda kv: -kv[1][0])[:args.top]
        for name, (us, count) in ranked:
            print(json.dumps({"kernel": name, "us_per_step": round(us / args.steps, 1),
                              "launches_per_step": count / args.steps}), flush=True)
    trainer.close()
    parallel.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
