"""Headline benchmark: Stack training throughput (tokens/s) on B200.

Workload: configs/stack_100m.json (d=1024, 16 heads, block 16,
``Lx7,G``), random-token task (next-token loss on every position), sequence
length 8192, batch 1 per data-parallel replica, bf16 autocast with fp32
master weights and AdamW, Ulysses context parallelism over all N ranks
(``cpN``). Synthetic data, random-init weights.

Usage::

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        # N > 1

One JSON line from rank 0. ``value`` is the whole-job tokens/s over the K
timed steps: W untimed warm-up steps, then a barrier + synchronize, CUDA
events around exactly K steps on every rank, the maximum elapsed time over
ranks. Every step copies its inputs from pinned host memory and reads its
loss back; ``e2e`` is the same K steps timed by the host clock (barrier +
synchronize on both sides), i.e. through the public training API end to
end. Inputs per step (ids/targets/mask, ~0.14 MB) are smaller than L2, but
each step streams ~1.3 GB of activations and weights, far larger than the
126 MB L2, so no explicit flush is needed (``l2`` in the config says so).
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
BASELINE_TOKENS_PER_S = None          # the reference publishes no B200 number for this config
METRIC = "train_tokens_per_second"
CONFIG = ROOT / "configs" / "stack_100m.json"
L2_NOTE = "no flush: ~1.3 GB of activations/weights stream per step (> 126 MB L2)"
LOG_WINDOW = 10                       # the reference's default --log-every: its throughput records cover 10 steps


def common_config(args, dp, cp):
    """The workload description both arms print, key for key."""
    return {"model": Path(args.config).stem, "global_batch": dp, "seq_len": args.length,
            "parallelism": f"cp{cp}" + (f"xdp{dp}" if dp > 1 else ""),
            "activation_recompute": bool(args.recompute), "l2": L2_NOTE}


def last_window(steps: int) -> int:
    """Size of the reference's last throughput window over ``steps`` timed steps."""
    return (steps - 1) % LOG_WINDOW + 1


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--length", type=int, default=8192)
    p.add_argument("--config", default=str(CONFIG))
    p.add_argument("--cp", type=int, default=0, help="context parallel size (default: all ranks)")
    p.add_argument("--recompute", action="store_true", help="activation recomputation (same on both arms)")
    p.add_argument("--cuda-graph", dest="cuda_graph", action=argparse.BooleanOptionalAction, default=True,
                   help="our arm: replay each training step from a CUDA graph")
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """``nvidia-smi`` clock and throttle-reason samples every 50 ms, kept for the timed window.

    The sampler starts before the warm-up steps (the process needs a moment to
    produce its first line) and ``mark(start, end)`` sets the timed window in
    wall-clock time; ``summary()`` reports the samples inside the window, or,
    when the window is shorter than the sampling interval, the nearest sample
    on each side of it (``"window": "adjacent"``).
    """

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, indices, interval_ms: int = 50):
        self.indices = set(indices)
        self.interval_ms = interval_ms
        self.proc = None
        self.lines = []
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", str(self.interval_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self, start: float, end: float) -> None:
        """The timed window, as ``time.time()`` values."""
        self.window = (start, end)

    def stop(self):
        if self.proc is not None:
            time.sleep(2 * self.interval_ms / 1e3)        # one more sample after the window
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.proc = None

    @staticmethod
    def _when(stamp: str):
        from datetime import datetime
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.strptime(stamp, fmt).timestamp()
            except ValueError:
                continue
        return None

    def samples(self):
        out = []
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10 or not parts[1].isdigit() or int(parts[1]) not in self.indices:
                continue
            try:
                sm, mx = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            reasons = {name for name, flag in zip(self.REASONS, parts[6:10]) if flag.lower() == "active"}
            out.append((self._when(parts[0]), sm, mx, reasons))
        return out

    def summary(self):
        samples = self.samples()
        chosen, window = samples, "unbounded"
        if self.window is not None and samples and all(t is not None for t, *_ in samples):
            t0, t1 = self.window
            inside = [s for s in samples if t0 <= s[0] <= t1]
            if inside:
                chosen, window = inside, "timed"
            else:
                before = [s for s in samples if s[0] < t0][-1:]
                after = [s for s in samples if s[0] > t1][:1]
                chosen, window = before + after, "adjacent"
        if not chosen:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = set().union(*(r for *_, r in chosen))
        return {"sm_mhz": statistics.median(s[1] for s in chosen), "sm_max_mhz": max(s[2] for s in chosen),
                "reasons": sorted(reasons), "samples": len(chosen), "window": window,
                "interval_ms": self.interval_ms}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from exploration_b200 import ExecutionConfig, ParallelContext, build_model
    from exploration_b200.cli import parse_args as cli_args
    from exploration_b200.ops import _native
    from exploration_b200.runtime.engine import Trainer, make_batch

    torch.cuda.set_device(local_rank)
    cp = args.cp or world
    argv = ["train", "--config", args.config, "--task", "random", "--length", str(args.length),
            "--batch-size", "1", "--precision", "bf16", "--backend", "cuda", "--context-parallel", str(cp),
            "--steps", str(args.warmup + args.steps), "--save", "", "--log-every", "1000000"]
    argv.append("--checkpoint-chunks" if args.recompute else "--no-checkpoint-chunks")
    targs = cli_args(argv)
    parallel = ParallelContext.initialize(cp, "cuda")
    device = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    options = {k: getattr(targs, k) for k in ("vocab_size", "dim", "heads", "block_size", "topk", "arch",
                                               "ffn_ratio")}
    execution = ExecutionConfig(backend="cuda", checkpoint_chunks=targs.checkpoint_chunks,
                                encoder_chunk=targs.encoder_chunk, query_chunk=targs.query_chunk,
                                loss_chunk=targs.loss_chunk)
    model = build_model({"model": "stack", **options}, execution=execution, device=device)
    model.train()
    fused_exchange = parallel.attach_fused(
        device, max(512 << 20, parallel.fused_heap_bytes(model, 1, args.length)))
    graphed = args.cuda_graph
    if graphed:
        from exploration_b200.runtime.engine import lr_factor
        from exploration_b200.runtime.flat import GraphTrainer
        trainer = GraphTrainer(targs, model, parallel)
    else:
        trainer = Trainer(targs, model, parallel)
    ext = _native.load()
    generator = torch.Generator().manual_seed(100 + parallel.dp_rank)
    h2d = d2h = 0

    def step(index):
        nonlocal h2d, d2h
        ids, target, mask, _ = make_batch(targs, generator)
        shard = -(-ids.shape[1] // (model.block_size * cp)) * model.block_size
        h2d = shard * ids.shape[0] * (ids.element_size() + target.element_size() + mask.element_size())
        if graphed:
            # Pinned inputs are copied to the device and the statistics back to
            # pinned memory inside the replayed graph; reading them is the D2H.
            trainer.step(ids, target, mask, targs.lr * lr_factor(index, targs.steps))
            d2h = 6 * 8
            stats = trainer.last_stats
            return float(stats[4] / stats[5])        # global mean loss per supervised token
        trainer.optimizer.zero_grad(set_to_none=True)
        trainer.set_lr(index)
        ids, target, mask = ids.pin_memory(), target.pin_memory(), mask.pin_memory()
        stats = trainer.micro_step(ids, target, mask, last=True)
        trainer.finish_step()
        loss = float(stats[0] / stats[1])          # device -> host read of the step's result (this rank's mean)
        d2h = stats.element_size() * stats.numel()
        return loss

    sampler = ClockSampler([local_rank]).start() if rank == 0 else None
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ext.launch_count()
    window0 = time.time()
    wall0 = time.perf_counter()
    start.record()
    losses = [step(args.warmup + i) for i in range(args.steps)]
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if sampler is not None:
        sampler.mark(window0, time.time())
        sampler.stop()
    launches = ext.launch_count() - launches0
    if graphed:
        launches += trainer.graph_launches * args.steps          # kernels replayed from the graph
    elapsed = torch.tensor([start.elapsed_time(end) / 1e3, wall], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    device_s, wall_s = (float(x) for x in elapsed)
    tokens = args.steps * parallel.dp_size * args.length          # batch 1 per DP replica
    result = None
    if rank == 0:
        value = tokens / device_s
        result = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(device_s * 1e3 / args.steps, 3),
            "higher_is_better": True, "scaling": "strong" if cp > 1 or world == 1 else "weak",
            "vs_baseline": None if BASELINE_TOKENS_PER_S is None else round(value / BASELINE_TOKENS_PER_S, 4),
            "dtype": "bf16", "data": "synthetic (uniform random token ids), random-init weights",
            "config": common_config(args, parallel.dp_size, cp),
            "details": {"optimizer": "fused AdamW fp32 master",
                        "ulysses_exchange": "nvlink-fused" if fused_exchange else ("nccl" if cp > 1 else "none"),
                        "cuda_graph": bool(graphed), "optimizer_shard": bool(targs.optimizer_shard),
                        "final_loss_over": f"mean of the last {last_window(args.steps)} steps"},
            "clocks": sampler.summary() if sampler is not None else None,
            "e2e": {"value": round(tokens / wall_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": int(launches),
            "final_loss": round(sum(losses[-last_window(args.steps):]) / last_window(args.steps), 4),
        }
    if graphed:
        trainer.close()
    parallel.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ---------------------------------------------------------------------------
# reference arm (unmodified reference from baseline/_ref, its own public CLI)
# ---------------------------------------------------------------------------

def run_reference(args, rank, world, local_rank):
    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "st" / "__init__.py").exists():
        return {"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}
    # Import the reference's `st` package, not this repository's alias of it.
    sys.path = [str(ref_root)] + [p for p in sys.path if Path(p or ".").resolve() != ROOT]
    for name in list(sys.modules):
        if name == "st" or name.startswith("st."):
            del sys.modules[name]
    import st  # noqa: F401  (the reference)
    from st.cli import main as reference_main
    cp = args.cp or world
    # The reference reports throughput once per 10-step window (its default
    # --log-every), timed by its host clock after cuda.synchronize and maxed
    # over ranks. Its warm-up is rounded up to whole windows so that the
    # windows after it cover exactly the K timed steps.
    warmup = max(LOG_WINDOW, -(-args.warmup // LOG_WINDOW) * LOG_WINDOW)
    argv = ["train", "--config", str(args.config), "--task", "random", "--length", str(args.length),
            "--batch-size", "1", "--precision", "bf16", "--backend", "auto", "--context-parallel", str(cp),
            "--steps", str(warmup + args.steps), "--save", "", "--eval-every", "0",
            "--checkpoint-chunks" if args.recompute else "--no-checkpoint-chunks"]
    buffer = io.StringIO()
    wall0 = time.perf_counter()
    with contextlib.redirect_stdout(buffer):
        reference_main(argv)
    wall = time.perf_counter() - wall0
    if rank != 0:
        return None
    records = [json.loads(line) for line in buffer.getvalue().splitlines() if line.startswith("{")]
    train = [r for r in records if r.get("event") == "train" and r["step"] > warmup]
    dp = world // cp
    tokens_per_step = dp * args.length
    steps, seconds, previous = 0, 0.0, warmup
    for r in train:
        window = r["step"] - previous
        previous = r["step"]
        steps += window
        seconds += window * tokens_per_step / r["tokens_per_second"]
    value = tokens_per_step * steps / seconds
    # Each step's batch is built on the host and copied to the device (ids and
    # targets int64, mask bool, this rank's shard); the loop reads the token
    # count, a finiteness flag and the clip norm's finiteness check back.
    shard = -(-args.length // cp)
    return {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": round(seconds * 1e3 / steps, 3),
            "higher_is_better": True, "scaling": "strong" if cp > 1 or world == 1 else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform random token ids), random-init weights",
            "config": common_config(args, dp, cp),
            "details": {"timing": "reference's own per-window host clock after cuda.synchronize, max over ranks",
                        "final_loss_over": f"its last window ({last_window(steps)} steps)",
                        "process_wall_s": round(wall, 2)},
            "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": shard * 17 * world,
                    "d2h_bytes_per_step": 10 * world,
                    "how": "the reference's host-clock windows, which include its pageable H2D input copies "
                           "and per-step device-to-host reads"},
            "final_loss": train[-1]["loss"] if train else None,
            "peak_allocated_gib": train[-1].get("peak_allocated_gib") if train else None}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    runner = run_reference if args.impl == "reference" else run_ours
    try:
        result = runner(args, rank, world, local_rank)
    except Exception as exc:
        if args.impl == "reference":
            result = {"impl": "reference", "unavailable": f"{type(exc).__name__}: {str(exc)[:200]}"}
        else:
            raise
    if rank == 0 and result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
