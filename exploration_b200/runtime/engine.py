"""Train / evaluate / plan engine behind the CLI and ``bench.py``.

One training step (reference: st/runtime/engine.py:79-208), per micro-batch:
build the CPU batch from this DP replica's generator, shard it over the CP
group, run the dense loss under bf16 autocast, normalise by the *global*
supervised-token count (times ``world_size`` to cancel DDP's averaging),
refuse a non-finite loss on any rank, backward; then clip with
``error_if_nonfinite`` and step the optimizer. The learning rate warms up
linearly for ``steps/20`` steps, then follows a cosine down to 10%.

B200 choices: the optimizer is the fused multi-tensor AdamW of
:mod:`exploration_b200.runtime.optim` (one kernel per step for all
parameters, fp32 master weights), wrapped in ZeRO-1 when sharding is on;
throughput windows are timed as the max over ranks.
"""
from __future__ import annotations

import contextlib
import json
import math
import os
import random
import time
from pathlib import Path

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

from .. import data
from ..api import build_model
from ..config import ExecutionConfig, ModelConfig
from ..data.tokens import TokenDataset, enwik8_dataset
from ..ops import fused
from ..models.baseline import BaselineModel
from ..models.stack import StackModel
from ..parallel.context import ParallelContext, init_distributed, sum_all
from . import checkpoint as ckpt
from . import trace
from .faults import maybe_fail
from .inference import InferenceSession
from .memory import GiB, training_estimate
from .metrics import MetricAccumulator, parse_bucket_edges, tail_mask
from .optim import build_optimizer

RESUME_KEYS = ("task", "tokens", "token_dtype", "length", "batch_size", "grad_accum", "precision",
               "steps", "lr", "weight_decay", "clip_grad", "npairs", "npairs_density", "nqueries",
               "nkeytoks", "supervision", "tail_tokens")


def model_options(args) -> dict:
    return ModelConfig(model=args.model, vocab_size=args.vocab_size, dim=args.dim, heads=args.heads,
                       block_size=args.block_size, arch=args.arch, ffn_ratio=args.ffn_ratio,
                       topk=args.topk or 64, layers=args.layers).to_dict()


def emit(record: dict, args, rank: int = 0) -> None:
    """Rank-0 JSONL record to stdout and, optionally, the ``--log`` file."""
    if rank:
        return
    line = json.dumps(record, ensure_ascii=False)
    print(line, flush=True)
    if getattr(args, "log", ""):
        Path(args.log).parent.mkdir(parents=True, exist_ok=True)
        with open(args.log, "a") as handle:
            handle.write(line + "\n")


def make_batch(args, generator, dataset=None):
    """One CPU micro-batch ``(ids, targets, mask, extra)`` for ``args.task``."""
    if args.task in ("tokens", "enwik8"):
        batch = dataset.batch(args.batch_size, args.length, generator)
    elif args.task == "random":
        batch = data.random_batch(args.batch_size, args.length, generator, args.vocab_size)
    elif args.task == "mqar":
        pairs = data.resolve_npairs(args.length, args.npairs, args.npairs_density)
        batch = data.mqar_batch(args.batch_size, args.length, generator, "cpu", n_pairs=pairs,
                                n_queries=args.nqueries, key_tokens=args.nkeytoks)
    else:
        batch = getattr(data, f"{args.task}_batch")(args.batch_size, args.length, generator, "cpu")
    ids, targets, mask, extra = batch
    if args.supervision == "all":
        mask = torch.ones_like(mask)
    elif args.supervision == "tail":
        if args.tail_tokens < 1:
            raise ValueError("--tail-tokens must be positive with --supervision tail")
        mask = tail_mask(mask, min(args.tail_tokens, mask.shape[1]))
    return ids, targets, mask, extra


def choose_cp(args, model, world, capacity) -> int:
    """Explicit CP, or the smallest CP dividing world and heads whose estimate fits."""
    if args.context_parallel != "auto":
        cp = int(args.context_parallel)
        if cp < 1 or world % cp or model.heads % cp:
            raise ValueError("context_parallel must divide both WORLD_SIZE and heads")
        return cp
    options = [c for c in range(1, world + 1) if world % c == 0 and model.heads % c == 0]
    for cp in options:
        estimate = training_estimate(model, args.batch_size, args.length, cp, args.checkpoint_chunks)
        if estimate["estimated_total_bytes"] < capacity * args.memory_fraction:
            return cp
    return options[-1]


def lr_factor(step: int, steps: int) -> float:
    warm = max(1, steps // 20)
    if step < warm:
        return (step + 1) / warm
    return 0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * (step - warm) / max(1, steps - warm)))


class Trainer:
    """Owns the wrapped model, the optimizer and one optimizer step."""

    def __init__(self, args, model, parallel):
        self.args, self.model, self.parallel = args, model, parallel
        self.device = next(model.parameters()).device
        if self.device.type == "cuda" and args.precision == "bf16" and not torch.cuda.is_bf16_supported():
            raise ValueError("this GPU does not support bf16; choose fp32")
        if args.activation_offload and self.device.type != "cuda":
            raise ValueError("activation offload requires CUDA")
        if parallel.world_size > 1:
            unused = isinstance(model, StackModel) and not bool(model.reads)
            self.wrapped = DDP(model, device_ids=[self.device.index] if self.device.type == "cuda" else None,
                               broadcast_buffers=False, gradient_as_bucket_view=True,
                               find_unused_parameters=unused)
        else:
            self.wrapped = model
        self.optimizer = build_optimizer(model, args, parallel, self.device)

    def set_lr(self, step: int) -> None:
        factor = lr_factor(step, self.args.steps)
        for group in self.optimizer.param_groups:
            group["lr"] = self.args.lr * factor

    def micro_step(self, ids, target, mask, last: bool):
        """Forward/backward of one micro-batch; returns detached (loss_sum, count, correct)."""
        args, parallel = self.args, self.parallel
        ids, offset = parallel.shard(ids, self.model.block_size)
        target, _ = parallel.shard(target, self.model.block_size, -100)
        mask, _ = parallel.shard(mask, self.model.block_size, False)
        ids, target, mask = (t.to(self.device, non_blocking=True) for t in (ids, target, mask))
        sync = self.wrapped.no_sync() if isinstance(self.wrapped, DDP) and not last \
            else contextlib.nullcontext()
        amp = torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=args.precision == "bf16")
        offload = torch.autograd.graph.save_on_cpu(pin_memory=True) if args.activation_offload \
            else contextlib.nullcontext()
        with sync:
            with amp, offload, trace.phase("forward"):
                result = self.wrapped(ids, sup=mask, targets=target, parallel=parallel, offset=offset)
                count = sum_all(result["count"])
                if int(count) == 0:
                    raise ValueError("global batch has no supervised tokens")
                scaled = result["loss_sum"] * parallel.world_size / count / args.grad_accum
            maybe_fail("before_backward")
            if not bool(torch.isfinite(sum_all(scaled.detach()))):
                raise FloatingPointError("non-finite loss across ranks; optimizer step was not applied")
            with trace.phase("backward"):
                scaled.backward()
        return torch.stack((result["loss_sum"].detach().double(), result["count"].double(),
                            result["correct"].double()))

    def finish_step(self):
        norm = torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.args.clip_grad,
                                              error_if_nonfinite=True)
        with trace.phase("optimizer"):
            self.optimizer.step()
        # Parameters changed (locally, or by a ZeRO broadcast that bypasses the
        # version counters): drop the per-step low-precision weight copies.
        fused.clear_cast_cache()
        return norm


def use_graph_trainer(args, model, device) -> bool:
    """The CUDA-graph step applies to Stack models on CUDA with one micro-step and no offload."""
    return (getattr(args, "cuda_graph", False) and device.type == "cuda" and isinstance(model, StackModel)
            and args.grad_accum == 1 and not args.activation_offload)


def train(args, model, parallel, ck, dataset, validation_dataset=None):
    device = next(model.parameters()).device
    graphed = use_graph_trainer(args, model, device)
    if graphed:
        from .flat import GraphTrainer
        trainer = GraphTrainer(args, model, parallel)
    else:
        trainer = Trainer(args, model, parallel)
    opt, device = trainer.optimizer, trainer.device
    generator = torch.Generator().manual_seed(args.seed + 100 + parallel.dp_rank)
    start = 0
    if ck is not None and not args.weights_only:
        topology = ck.get("topology", {})
        if topology and topology != {"world_size": parallel.world_size, "cp_size": parallel.cp_size}:
            raise ValueError("exact resume needs the saved topology; use --weights-only to change it")
        saved = ck.get("config", {}).get("runtime", {})
        for key in RESUME_KEYS:
            if key in saved and getattr(args, key) != saved[key]:
                raise ValueError(f"exact resume requires {key}={saved[key]!r}; use --weights-only "
                                 "to change the experiment")
        opt.load_state_dict(ck["opt"])
        start = ck["step"] + 1
        if "rng_by_rank" in ck:
            ckpt.restore_rng(ck["rng_by_rank"][parallel.rank], generator)
        else:
            emit({"event": "warning", "message": "legacy checkpoint has no RNG state; "
                  "the data stream restarts"}, args, parallel.rank)
    if ck is not None:
        ck.clear()
    model_keys = set(ModelConfig.__dataclass_fields__)
    config = {"model": model_options(args),
              "runtime": {k: v for k, v in vars(args).items()
                          if k not in model_keys and k not in ("command", "config")}}
    if start >= args.steps:
        raise ValueError("--steps is the total target step count and must exceed the resumed step")
    model.train()
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)
    stats = torch.zeros(3, device=device, dtype=torch.float64)
    window_start, window_steps = time.perf_counter(), 0
    profiler = None
    if getattr(args, "profile", ""):
        from .trace import StepProfiler
        profiler = StepProfiler(args.profile, parallel.rank)
    for step in range(start, args.steps):
        if graphed:
            ids, target, mask, _ = make_batch(args, generator, dataset)
            host, norm = trainer.step(ids, target, mask, args.lr * lr_factor(step, args.steps))
            stats += host.to(device)
        else:
            opt.zero_grad(set_to_none=True)
            trainer.set_lr(step)
            for micro in range(args.grad_accum):
                ids, target, mask, _ = make_batch(args, generator, dataset)
                stats += trainer.micro_step(ids, target, mask, last=micro == args.grad_accum - 1).to(device)
            norm = trainer.finish_step()
        window_steps += 1
        if profiler is not None:
            profiler.step()
        if (step + 1) % args.log_every == 0 or step == args.steps - 1:
            totals = sum_all(stats)
            if device.type == "cuda":
                torch.cuda.synchronize(device)
            elapsed = torch.tensor(time.perf_counter() - window_start, device=device)
            if parallel.world_size > 1:
                dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
            tokens = window_steps * args.grad_accum * args.batch_size * parallel.dp_size * args.length
            emit({"event": "train", "step": step + 1,
                  "loss": round(float(totals[0] / totals[1]), 6),
                  "accuracy": round(float(totals[2] / totals[1]), 4),
                  "grad_norm": round(float(norm), 4),
                  "tokens_per_second": round(tokens / float(elapsed)),
                  "peak_allocated_gib": round(torch.cuda.max_memory_allocated(device) / GiB, 3)
                  if device.type == "cuda" else None,
                  "peak_reserved_gib": round(torch.cuda.max_memory_reserved(device) / GiB, 3)
                  if device.type == "cuda" else None}, args, parallel.rank)
            stats.zero_()
            window_start, window_steps = time.perf_counter(), 0
        stop = False
        if args.eval_every and ((step + 1) % args.eval_every == 0 or step == args.steps - 1):
            began = time.perf_counter()
            record = evaluate(args, model, parallel, validation_dataset, during_training=True,
                              step=step + 1)
            model.train()
            stop = args.stop_exact is not None and record["exact"] >= args.stop_exact
            window_start += time.perf_counter() - began      # evaluation is not training time
        final = step == args.steps - 1
        if args.save and (stop or final or (args.save_every and (step + 1) % args.save_every == 0)):
            ckpt.save(args.save, model, opt, config, step, generator, parallel)
        if stop:
            emit({"event": "early_stop", "step": step + 1, "exact": round(record["exact"], 4)},
                 args, parallel.rank)
            break
    if profiler is not None:
        emit({"event": "profile", **profiler.summary()}, args, parallel.rank)
    if graphed:
        trainer.close()


def _query_positions(args, mask):
    """``[B, S]`` absolute positions whose next token is scored."""
    if args.eval_positions:
        # A fixed, evenly spread set that always includes the last position.
        width = min(args.eval_positions, args.length)
        return torch.linspace(0, args.length - 1, width).round().long()[None].expand(args.batch_size, -1)
    counts = mask.sum(1)
    if int(counts.max()) != int(counts.min()) or int(counts.min()) == 0:
        raise ValueError("inference task masks must have equal nonzero counts per row")
    return mask.nonzero()[:, 1].view(args.batch_size, -1)


@contextlib.contextmanager
def _logit_stream(args, model, parallel, ids, positions, first: bool):
    """Yields an iterator of ``(slice, logits)`` over ``positions``.

    Stack models run the paged sparse session (prefill into the tiered K/V
    cache, then the read rounds chunk by chunk); the dense baseline encodes
    once and projects the requested positions slice by slice.
    """
    if not isinstance(model, StackModel):
        device = next(model.parameters()).device
        yield ((sl, logits) for sl, logits, _ in model.iter_logits(ids.to(device), positions.to(device),
                                                                    parallel=parallel))
        return
    group = dist.group.WORLD if parallel.world_size > 1 else None
    with InferenceSession(model, group=group, cache=args.cache, cache_dir=args.cache_dir or None,
                          memory_fraction=args.memory_fraction, page_tokens=args.page_tokens,
                          encoder_chunk=args.encoder_chunk, query_chunk=args.inference_query_chunk,
                          workspace_mb=args.workspace_mb, max_query_states_mb=args.max_query_states_mb) as session:
        session.prefill(ids, positions)
        if first:
            emit({"event": "inference_plan", "batch": 0, **session.plan.to_dict()}, args, parallel.rank)
        yield ((sl, logits) for sl, logits, _ in session.iter_logits())


@torch.no_grad()
def evaluate(args, model, parallel, dataset, during_training=False, step=None):
    """Score ``eval_batches`` batches; token metrics and exact match stay on the device until the end."""
    model.eval()
    if args.precision == "bf16" and not during_training:
        model.to(torch.bfloat16)
    on_gpu = next(model.parameters()).is_cuda
    if on_gpu and not during_training:
        torch.cuda.reset_peak_memory_stats()
    generator = torch.Generator().manual_seed(args.seed + 200)
    metrics = MetricAccumulator(parse_bucket_edges(getattr(args, "metric_buckets", "auto"), args.length))
    metrics.start_rows(0, track_rows=False)
    exact_rows = None
    begin = time.perf_counter()
    for index in range(args.eval_batches):
        ids, targets, mask, _ = make_batch(args, generator, dataset)
        positions = _query_positions(args, mask)
        truth = targets.gather(1, positions)
        wrong = None
        with _logit_stream(args, model, parallel, ids, positions, index == 0) as stream:
            for sl, logits in stream:
                target = truth[:, sl].to(logits.device)
                metrics.update(logits, target, positions[:, sl].to(logits.device))
                misses = (logits.argmax(-1) != target).sum(1)
                wrong = misses if wrong is None else wrong + misses
        solved = (wrong == 0).sum()
        exact_rows = solved if exact_rows is None else exact_rows + solved
    summary = metrics.finalize()
    summary["exact"] = int(exact_rows) / max(1, args.eval_batches * args.batch_size)
    result = {"event": "eval", **({"step": step} if step is not None else {}), "length": args.length,
              **{k: round(v, 6) if isinstance(v, float) else v for k, v in summary.items()},
              "seconds": round(time.perf_counter() - begin, 3),
              "peak_allocated_gib": round(torch.cuda.max_memory_allocated() / GiB, 3) if on_gpu else None}
    emit(result, args, parallel.rank)
    if args.output and parallel.rank == 0 and not during_training:
        Path(args.output).parent.mkdir(parents=True, exist_ok=True)
        Path(args.output).write_text(json.dumps(result, indent=2) + "\n")
    return result


# ---------------------------------------------------------------------------
# the commands
# ---------------------------------------------------------------------------

def _resolve_architecture(args, ck) -> dict:
    """Model options from the checkpoint (resume) or the flags, written back onto ``args``."""
    if args.task == "enwik8":
        args.vocab_size = 256                      # byte tokens
    options = dict(ckpt.model_config(ck)) if ck is not None else model_options(args)
    options.setdefault("model", "stack")
    if args.topk is not None and options["model"] == "stack":
        options["topk"] = args.topk                # inference-time override of the read width
    for key, value in options.items():
        setattr(args, key, value)
    args.topk = options.get("topk", 64)
    return options


def _execution(args) -> ExecutionConfig:
    return ExecutionConfig(backend=args.backend, checkpoint_chunks=args.checkpoint_chunks,
                           encoder_chunk=args.encoder_chunk, query_chunk=args.query_chunk,
                           loss_chunk=args.loss_chunk, flash_attention=args.flash_attention,
                           attention_q_chunk=args.attention_q_chunk, attention_kv_chunk=args.attention_kv_chunk)


def _plan_report(args, model, options) -> None:
    kv_element = 2 if args.precision == "bf16" else 4
    report = {"model": options,
              "training": [training_estimate(model, args.batch_size, args.length, c, args.checkpoint_chunks)
                           for c in (1, 2, 4, 8) if model.heads % c == 0],
              "inference_raw_kv_bytes": (2 * args.batch_size * args.length * model.dim * kv_element
                                         if isinstance(model, StackModel) else None)}
    print(json.dumps(report, indent=2))


def _this_rank_device(args):
    """``(device, HBM capacity)`` of this process (CPU runs get a nominal 64 GiB)."""
    if args.device != "cuda":
        return torch.device("cpu"), 64 * GiB
    if not torch.cuda.is_available():
        raise RuntimeError("NVIDIA CUDA is required; use --device cpu for the reference path")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    device = torch.device("cuda", torch.cuda.current_device())
    return device, torch.cuda.mem_get_info(device)[1]


def _datasets(args):
    """``(data, validation data)``; ``None`` for the synthetic tasks."""
    if args.task == "tokens":
        validation = TokenDataset(args.validation_tokens, args.token_dtype) if args.validation_tokens else None
        return TokenDataset(args.tokens, args.token_dtype), validation
    if args.task == "enwik8":
        path = args.tokens or "data/enwik8"
        training = args.command == "train"
        validation = enwik8_dataset(path, args.split) if training and args.eval_every else None
        return enwik8_dataset(path, "train" if training else args.split), validation
    return None, None


def run(args):
    """``plan``, ``train`` or ``eval`` for one process of a (torchrun) job of 1..8 ranks."""
    torch.manual_seed(args.seed)
    random.seed(args.seed)
    ck = ckpt.load(args.resume) if args.resume else None
    options = _resolve_architecture(args, ck)
    model = build_model(options, device="meta" if args.command == "plan" else "cpu", execution=_execution(args))
    if ck is not None:
        state = ck.pop("model")
        if args.command != "plan":
            model.load_state_dict(state, strict=True)
        if args.command != "train":
            ck.clear()                             # only training resumes optimizer and RNG state
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not 1 <= world <= 8:
        raise ValueError("supported process count is 1..8")
    if args.command == "plan":
        _plan_report(args, model, options)
        return None
    device, capacity = _this_rank_device(args)
    if world > 1:
        init_distributed(args.device)
        smallest = torch.tensor(capacity, device=device, dtype=torch.long)
        dist.all_reduce(smallest, op=dist.ReduceOp.MIN)     # plan for the smallest GPU of the job
        capacity = int(smallest)
    cp = choose_cp(args, model, world, capacity) if args.command == "train" else 1
    parallel = None
    try:
        parallel = ParallelContext.initialize(cp, args.device)
        estimate = training_estimate(model, args.batch_size, args.length, cp, args.checkpoint_chunks)
        estimate.pop("note")
        record = {"event": "configuration", "model": options, "world": world, "cp": cp, "dp": parallel.dp_size,
                  "effective_batch": args.batch_size * parallel.dp_size * args.grad_accum, **estimate}
        if world == 1 and args.device == "cuda" and torch.cuda.device_count() > 1:
            record["hint"] = (f"{torch.cuda.device_count()} GPUs are visible; launch with torchrun "
                              "--nproc_per_node=N to use them")
        emit(record, args, parallel.rank)
        over = estimate["estimated_total_bytes"] > capacity * args.memory_fraction
        if args.command == "train" and device.type == "cuda" and over and not args.allow_over_budget:
            raise MemoryError("training estimate exceeds the memory budget; reduce the micro-batch, "
                              "use CP/recompute, or pass --allow-over-budget")
        if args.task in ("passkey", "copying", "mqar") and args.vocab_size < data.VOCAB:
            raise ValueError("synthetic tasks require vocab_size >= 128")
        dataset, validation = _datasets(args)
        model.to(device)
        if device.type == "cuda" and isinstance(model, StackModel) and args.backend != "torch":
            # NVLink exchange: symmetric heap sized for the longest sequence this run sees.
            length = max(args.length, getattr(args, "eval_length", 0) or 0)
            parallel.attach_fused(device, max(512 << 20, parallel.fused_heap_bytes(model, args.batch_size, length)))
        if args.command == "train":
            return train(args, model, parallel, ck, dataset, validation)
        return evaluate(args, model, parallel, dataset)
    finally:
        if parallel is not None:
            parallel.close()
        if dist.is_initialized():
            dist.destroy_process_group()
