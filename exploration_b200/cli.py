"""Command line: ``python -m st {plan,train,eval,validate,benchmark}``.

Flags, JSON config files and their precedence match the reference
(st/cli.py:16-209): a JSON file holds only ``model`` and ``runtime`` objects
whose keys are flag destinations; explicit flags beat the JSON, which beats
the defaults; JSON values are re-checked for type and choice; legacy flags
are rejected. The option table below is the single definition: each entry
says which option group it belongs to, and the subcommands that hide it.
"""
from __future__ import annotations

import argparse
import json
import sys

COMMANDS = {
    "plan": "Estimate model size and memory without allocating weights",
    "train": "Train with dense attention; optionally evaluate and checkpoint",
    "eval": "Evaluate a checkpoint; StackModel uses paged sparse inference",
    "validate": "Run reference, CUDA parity or multi-GPU correctness checks",
    "benchmark": "Measure attention latency/memory on a CUDA GPU",
}

BOOL = argparse.BooleanOptionalAction
MODEL = "model"
DATA = "data"
EXEC = "execution"
TRAIN = "training"
EVAL = "evaluation"
FILES = "files"

# (flag, group, argparse keyword arguments)
OPTIONS = [
    ("--config", FILES, dict(help="JSON with model and runtime objects")),
    ("--model", MODEL, dict(choices=["stack", "baseline"], default="stack")),
    ("--layers", MODEL, dict(type=int, default=3, help="baseline depth")),
    ("--task", DATA, dict(choices=["passkey", "mqar", "copying", "tokens", "enwik8", "random"],
                          default="passkey")),
    ("--tokens", DATA, dict(default="", help="flat token corpus (required for task=tokens)")),
    ("--token-dtype", DATA, dict(default="uint16", choices=["uint8", "uint16", "int32", "int64"])),
    ("--validation-tokens", DATA, dict(default="", help="held-out token file for periodic evaluation")),
    ("--split", DATA, dict(choices=["train", "val", "test"], default="val", help="enwik8 eval split")),
    ("--vocab-size", MODEL, dict(type=int, default=128)),
    ("--dim", MODEL, dict(type=int, default=256)),
    ("--heads", MODEL, dict(type=int, default=4)),
    ("--block-size", MODEL, dict(type=int, default=16)),
    ("--arch", MODEL, dict(default="Lx2,G")),
    ("--ffn-ratio", MODEL, dict(type=float, default=4.0)),
    ("--topk", MODEL, dict(type=int, default=None, help="inference top-k; training is always dense")),
    ("--length", DATA, dict(type=int, default=512)),
    ("--batch-size", DATA, dict(type=int, default=1, help="micro-batch per data-parallel replica")),
    ("--grad-accum", TRAIN, dict(type=int, default=1)),
    ("--context-parallel", TRAIN, dict(default="auto", help="auto or a divisor of heads and WORLD_SIZE")),
    ("--precision", EXEC, dict(choices=["fp32", "bf16"], default="bf16")),
    ("--backend", EXEC, dict(choices=["auto", "torch", "cuda", "triton"], default="auto",
                             help="cuda: native sm_100a kernels (triton is a synonym); "
                                  "torch: bounded reference")),
    ("--flash-attention", EXEC, dict(dest="flash_attention", choices=["auto", "flash", "math"],
                                     default="auto", help="baseline SDPA kernel selection")),
    ("--checkpoint-chunks", EXEC, dict(action=BOOL, default=True)),
    ("--activation-offload", TRAIN, dict(action="store_true",
                                         help="offload autograd saved tensors to pinned host RAM")),
    ("--optimizer-shard", TRAIN, dict(action=BOOL, default=True)),
    ("--profile", TRAIN, dict(default="", help="directory for a torch.profiler trace of steps 2-4 "
                                                "(NVTX phase ranges included); empty disables")),
    ("--cuda-graph", TRAIN, dict(dest="cuda_graph", action=BOOL, default=False,
                                 help="capture each training step in a CUDA graph (flat AdamW, "
                                      "explicit gradient reduction; CUDA, one micro-step)")),
    ("--encoder-chunk", EXEC, dict(type=int, default=1024)),
    ("--query-chunk", EXEC, dict(type=int, default=0, help="queries per tile; 0 = automatic")),
    ("--loss-chunk", EXEC, dict(type=int, default=128)),
    ("--attention-q-chunk", EXEC, dict(type=int, default=128, help="torch-reference query tile")),
    ("--attention-kv-chunk", EXEC, dict(type=int, default=4096, help="torch-reference KV tile")),
    ("--steps", TRAIN, dict(type=int, default=1000)),
    ("--eval-every", TRAIN, dict(type=int, default=0, help="evaluation interval; 0 disables it")),
    ("--stop-exact", TRAIN, dict(type=float, default=None,
                                 help="save and stop once periodic exact accuracy reaches this")),
    ("--lr", TRAIN, dict(type=float, default=3e-4)),
    ("--weight-decay", TRAIN, dict(type=float, default=0.01)),
    ("--clip-grad", TRAIN, dict(type=float, default=1.0)),
    ("--seed", DATA, dict(type=int, default=0)),
    ("--log-every", TRAIN, dict(type=int, default=10)),
    ("--save-every", TRAIN, dict(type=int, default=0)),
    ("--save", TRAIN, dict(default="runs/stack.pt")),
    ("--resume", FILES, dict(default="")),
    ("--weights-only", TRAIN, dict(action="store_true", help="load weights, reset optimizer and RNG")),
    ("--log", FILES, dict(default="", help="rank-zero JSONL path")),
    ("--device", EXEC, dict(choices=["cuda", "cpu"], default="cuda")),
    ("--memory-fraction", EXEC, dict(type=float, default=0.8)),
    ("--allow-over-budget", TRAIN, dict(action="store_true",
                                        help="override the conservative training memory estimate")),
    ("--npairs", DATA, dict(type=int, default=16)),
    ("--npairs-density", DATA, dict(type=float, default=0.0, help="MQAR pairs per token")),
    ("--nqueries", DATA, dict(type=int, default=4)),
    ("--nkeytoks", DATA, dict(type=int, choices=[1, 2], default=1)),
    ("--supervision", DATA, dict(choices=["task", "all", "tail"], default="task")),
    ("--tail-tokens", DATA, dict(type=int, default=0, help="final tokens for --supervision tail")),
    ("--eval-batches", EVAL, dict(type=int, default=1)),
    ("--eval-positions", EVAL, dict(type=int, default=0,
                                    help="0 = task mask; otherwise evenly spaced query positions")),
    ("--cache", EVAL, dict(default="auto", choices=["auto", "cuda", "cpu", "disk"])),
    ("--cache-dir", EVAL, dict(default="")),
    ("--page-tokens", EVAL, dict(type=int, default=65536)),
    ("--inference-query-chunk", EVAL, dict(type=int, default=16)),
    ("--workspace-mb", EVAL, dict(type=int, default=256)),
    ("--max-query-states-mb", EVAL, dict(type=int, default=256)),
    ("--metric-buckets", EVAL, dict(default="auto", help="absolute position edges, e.g. 0,1024,4096")),
    ("--output", FILES, dict(default="", help="eval JSON output written by rank zero")),
]

# Options `plan` shows besides the model group.
PLAN_EXTRA = {"config", "task", "length", "batch_size", "precision", "checkpoint_chunks", "resume",
              "encoder_chunk", "query_chunk", "loss_chunk", "backend", "flash_attention",
              "attention_q_chunk", "attention_kv_chunk"}
POSITIVE = ("length", "batch_size", "grad_accum", "encoder_chunk", "loss_chunk", "attention_q_chunk",
            "attention_kv_chunk", "steps", "log_every", "eval_batches", "page_tokens",
            "inference_query_chunk", "workspace_mb", "max_query_states_mb")


def _dest(flag, kwargs):
    return kwargs.get("dest", flag[2:].replace("-", "_"))


def _visible(command, group, dest):
    if command == "plan":
        return group == MODEL or dest in PLAN_EXTRA
    if command == "eval":
        return group != TRAIN
    return True


def _add_experiment_options(parser, command):
    groups = {name: parser.add_argument_group(name) for name in (MODEL, DATA, EXEC, TRAIN, EVAL, FILES)}
    for flag, group, kwargs in OPTIONS:
        dest = _dest(flag, kwargs)
        if _visible(command, group, dest):
            groups[group].add_argument(flag, **kwargs)
        else:
            default = kwargs.get("default", False if kwargs.get("action") == "store_true" else None)
            parser.set_defaults(**{dest: default})


def parser():
    top = argparse.ArgumentParser(prog="python -m st",
                                  description="Stack experiments on B200: one command entry point.",
                                  epilog="Start: python -m st benchmark --help", allow_abbrev=False)
    sub = top.add_subparsers(dest="command", required=True, title="commands")
    top.experiments = {}
    for name in ("plan", "train", "eval"):
        child = sub.add_parser(name, help=COMMANDS[name], description=COMMANDS[name], allow_abbrev=False)
        _add_experiment_options(child, name)
        top.experiments[name] = child
    from .tools.benchmark import parser as benchmark_parser
    from .tools.validate import parser as validate_parser
    sub.add_parser("benchmark", help=COMMANDS["benchmark"], parents=[benchmark_parser()],
                   add_help=False, allow_abbrev=False)
    sub.add_parser("validate", help=COMMANDS["validate"], parents=[validate_parser()],
                   add_help=False, allow_abbrev=False)
    return top


def _check_json_types(top, experiment, args):
    """argparse does not validate defaults injected from JSON; do it here."""
    for action in experiment._actions:
        if action.dest == "help":
            continue
        value = getattr(args, action.dest, None)
        if value is None:
            continue
        if action.type is int and type(value) is not int:
            top.error(f"{action.dest} must be an integer")
        if action.type is float and (isinstance(value, bool) or not isinstance(value, (int, float))):
            top.error(f"{action.dest} must be a number")
        if isinstance(action, (BOOL, argparse._StoreTrueAction)) and type(value) is not bool:
            top.error(f"{action.dest} must be a boolean")
        if action.choices is not None and value not in action.choices:
            top.error(f"invalid {action.dest}: {value!r}; choose from {action.choices}")


def parse_args(argv=None):
    top = parser()
    first, _ = top.parse_known_args(argv)
    if first.command not in top.experiments:
        return top.parse_args(argv)
    experiment = top.experiments[first.command]
    if first.config:
        with open(first.config) as handle:
            config = json.load(handle)
        if not isinstance(config, dict) or any(not isinstance(config.get(k, {}), dict)
                                               for k in ("model", "runtime")):
            top.error("config must contain model/runtime JSON objects")
        if set(config) - {"model", "runtime"}:
            raise ValueError("config root accepts only model and runtime")
        defaults = dict(config.get("model", {}), **config.get("runtime", {}))
        known = ({a.dest for a in experiment._actions} | set(experiment._defaults)) \
            - {"command", "config", "help"}
        if set(defaults) - known:
            raise ValueError(f"unknown config keys: {sorted(set(defaults) - known)}")
        experiment.set_defaults(**defaults)
    args = top.parse_args(argv)
    _check_json_types(top, experiment, args)
    if args.query_chunk < 0:
        top.error("query_chunk must be nonnegative (0=auto)")
    if args.tail_tokens < 0:
        top.error("tail_tokens must be nonnegative")
    for name in POSITIVE:
        if getattr(args, name) < 1:
            top.error(f"{name} must be positive")
    if not 0 < args.memory_fraction < 1:
        top.error("memory_fraction must lie strictly between 0 and 1")
    if args.context_parallel != "auto":
        text = str(args.context_parallel)
        if not text.isdigit() or int(text) < 1:
            top.error("context_parallel must be auto or a positive integer")
        args.context_parallel = str(int(text))
    if args.command == "train" and args.length > 65536:
        top.error("dense training is limited to 65536 tokens; longer lengths are inference-only")
    if args.command == "eval" and not args.resume:
        top.error("eval requires --resume")
    if args.weights_only and not args.resume:
        top.error("weights-only requires --resume")
    if args.topk is not None and args.topk < 1:
        top.error("topk must be positive")
    if min(args.eval_every, args.save_every, args.eval_positions, args.npairs_density) < 0:
        top.error("intervals, eval_positions and npairs_density must be nonnegative")
    if args.stop_exact is not None and (not 0 <= args.stop_exact <= 1 or not args.eval_every):
        top.error("stop-exact requires a threshold in [0,1] and eval-every > 0")
    if args.command == "train" and args.task == "tokens" and args.eval_every and not args.validation_tokens:
        top.error("periodic token evaluation requires --validation-tokens (a held-out corpus)")
    return args


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv:
        parser().print_help()
        return None
    if argv[0] == "validate":
        from .tools.validate import main as validate
        return validate(argv[1:])
    if argv[0] == "benchmark":
        from .tools.benchmark import main as benchmark
        return benchmark(argv[1:])
    args = parse_args(argv)
    from .runtime.engine import run
    return run(args)


def entrypoint():
    """Console script: never use a result dictionary as the exit status."""
    main()
