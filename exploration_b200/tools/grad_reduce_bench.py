"""Device time of the peer-memory gradient reduction, per bucket, at N GPUs.

Run as one process per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m exploration_b200.tools.grad_reduce_bench --reps 10

It builds the benchmark model (stack_100m by default), lays its parameters
out in the flat buffers of the training step (gradient and bf16 shadow in
the symmetric heap, ZeRO-1 sharding over all ranks) and runs the gradient
reduction of one step on its own, with no backward to hide it: every bucket
kernel (``grad_reduce_bucket``) back to back on the side stream, then the
norm exchange. CUDA events bracket each bucket and the whole reduction;
every figure is the median over ``--reps`` repetitions of the maximum over
ranks.

Bytes that cross NVLink per rank and bucket: the rank pulls its slice
(``q`` fp32 elements) from each of the other ``N - 1`` ranks; an all-reduce
bucket also stores the sum into those ranks' buffers (the other direction of
the link). The roofline of a bucket is therefore ``(N - 1) * q * 4`` bytes
over the measured 770 GB/s peer bandwidth per direction.

Rank 0 prints one JSON line per bucket and one summary line. The reference
reduces gradients with DDP's NCCL all-reduce buckets
(st/runtime/engine.py:85-87).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

LINK_GBS = 770.0     # measured peer copy bandwidth per direction on this pool's B200 nodes


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--bucket-mb", type=int, default=32)
    p.add_argument("--config", default=str(Path(__file__).resolve().parents[2] / "configs" / "stack_100m.json"))
    args = p.parse_args(argv)

    from .. import ExecutionConfig, build_model
    from ..cli import parse_args as cli_args
    from ..runtime.flat import FlatParameters, PeerGradBuckets

    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world < 2:
        raise SystemExit("grad_reduce_bench needs at least two ranks (torch.distributed.run)")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=60))
    rank = dist.get_rank()
    targs = cli_args(["train", "--config", args.config, "--backend", "cuda", "--save", ""])
    options = {k: getattr(targs, k) for k in ("vocab_size", "dim", "heads", "block_size", "topk", "arch", "ffn_ratio")}
    torch.manual_seed(0)
    model = build_model({"model": "stack", **options}, execution=ExecutionConfig(backend="cuda"), device=device)
    flat = FlatParameters(model, device, shards=world, peer_group=dist.group.WORLD)
    buckets = PeerGradBuckets(flat, shard=True, bucket_bytes=args.bucket_mb << 20)
    hyper = torch.zeros(4, device=device)
    n_buckets = len(buckets.bounds)

    # Events around every bucket launch (on the side stream, where the kernels run).
    marks: list[tuple[int, torch.cuda.Event, torch.cuda.Event]] = []
    launch = buckets._launch

    def timed_launch(index: int) -> None:
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record(buckets.stream)
        launch(index)
        end.record(buckets.stream)
        marks.append((index, begin, end))

    buckets._launch = timed_launch
    per_bucket = [[] for _ in range(n_buckets)]
    totals = []
    for rep in range(args.warmup + args.reps):
        flat.grad.normal_()
        marks.clear()
        torch.cuda.synchronize()
        dist.barrier()
        first, last = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        first.record(buckets.stream)
        buckets.start()
        buckets.finish(hyper)
        last.record(buckets.stream)
        torch.cuda.synchronize()
        times = torch.zeros(n_buckets + 1, device=device, dtype=torch.float64)
        for index, begin, end in marks:
            times[index] = begin.elapsed_time(end)
        times[n_buckets] = first.elapsed_time(last)
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        if rep >= args.warmup:
            values = times.tolist()
            for b in range(n_buckets):
                per_bucket[b].append(values[b])
            totals.append(values[n_buckets])
    errors = buckets.ext.device_errors(local_rank)

    if rank == 0:
        link_bytes = 0
        bucket_us = 0.0
        for b, (lo, hi) in enumerate(buckets.bounds):
            q, all_reduce = buckets.slices[b]
            pulled = (world - 1) * q * 4
            us = statistics.median(per_bucket[b]) * 1e3
            link_bytes += pulled
            bucket_us += us
            print(json.dumps({"bucket": b, "elements": hi - lo, "slice": q, "all_reduce": bool(all_reduce),
                              "pulled_bytes_per_rank": pulled, "us": round(us, 1),
                              "link_gbs": round(pulled / us / 1e3, 1),
                              "of_770": round(pulled / us / 1e3 / LINK_GBS, 3)}), flush=True)
        total_us = statistics.median(totals) * 1e3
        print(json.dumps({"n_gpus": world, "buckets": n_buckets, "gradient_elements": flat.total,
                          "pulled_bytes_per_rank": link_bytes, "bucket_kernels_us": round(bucket_us, 1),
                          "reduction_us": round(total_us, 1), "link_gbs": round(link_bytes / total_us / 1e3, 1),
                          "of_770": round(link_bytes / total_us / 1e3 / LINK_GBS, 3),
                          "device_errors": list(errors)}), flush=True)
    buckets.remove()
    flat.release()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
