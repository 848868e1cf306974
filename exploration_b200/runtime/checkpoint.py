"""Atomic, resumable checkpoints (format version 2).

Layout, shared with the reference so checkpoints move between frameworks
(st/runtime/checkpoint.py:39-93)::

    {"format_version": 2,
     "model": CPU state dict (tied/shared weights stay aliased),
     "opt": optimizer state (consolidated for ZeRO-1),
     "config": {"model": ModelConfig.to_dict(), "runtime": {...}},
     "step": last completed step,
     "rng_by_rank": [{"torch", "python", "data", "cuda"?}, ...],
     "topology": {"world_size", "cp_size"}}

Rank 0 writes to a temporary file in the target directory, fsyncs and
renames it over the target, so a crash never leaves a torn checkpoint. A
failure on rank 0 is broadcast, so every rank raises.
"""
from __future__ import annotations

import os
import random
import tempfile
from pathlib import Path

import torch
import torch.distributed as dist

FORMAT_VERSION = 2


def rng_state(generator: torch.Generator) -> dict:
    state = {"torch": torch.get_rng_state(), "python": random.getstate(),
             "data": generator.get_state()}
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        state["cuda"] = torch.cuda.get_rng_state()
    return state


def restore_rng(state: dict, generator: torch.Generator) -> None:
    torch.set_rng_state(state["torch"])
    random.setstate(state["python"])
    generator.set_state(state["data"])
    if "cuda" in state and torch.cuda.is_available():
        torch.cuda.set_rng_state(state["cuda"])


def cpu_state_dict(model) -> dict:
    """CPU copy of ``model.state_dict()`` that keeps aliased entries aliased."""
    copies, result = {}, {}
    for name, value in model.state_dict().items():
        key = (value.device, value.data_ptr(), tuple(value.shape), tuple(value.stride()), value.dtype)
        if key not in copies:
            copies[key] = value.detach().cpu()
        result[name] = copies[key]
    return result


def _optimizer_state(optimizer):
    if hasattr(optimizer, "consolidate_state_dict"):
        optimizer.consolidate_state_dict(to=0)
    return optimizer


def save(path, model, optimizer, config, step, generator, parallel) -> None:
    _optimizer_state(optimizer)
    local = rng_state(generator)
    if parallel.world_size > 1:
        states = [None] * parallel.world_size if parallel.rank == 0 else None
        dist.gather_object(local, states, dst=0)
    else:
        states = [local]
    error = None
    if parallel.rank == 0:
        temp = None
        try:
            target = Path(path)
            target.parent.mkdir(parents=True, exist_ok=True)
            payload = {"format_version": FORMAT_VERSION, "model": cpu_state_dict(model),
                       "opt": optimizer.state_dict(), "config": config, "step": step,
                       "rng_by_rank": states,
                       "topology": {"world_size": parallel.world_size, "cp_size": parallel.cp_size}}
            fault_point("checkpoint_write")
            with tempfile.NamedTemporaryFile(dir=target.parent, prefix=target.name + ".",
                                             suffix=".tmp", delete=False) as handle:
                temp = handle.name
                torch.save(payload, handle)
                handle.flush()
                os.fsync(handle.fileno())
            os.replace(temp, target)
        except Exception as exc:
            error = f"checkpoint save failed: {exc}"
            if temp and os.path.exists(temp):
                os.unlink(temp)
    if parallel.world_size > 1:
        box = [error]
        dist.broadcast_object_list(box, src=0)
        error = box[0]
    if error:
        raise RuntimeError(error)


def load(path):
    """Load a locally trusted checkpoint (it holds pickled optimizer/RNG state)."""
    return torch.load(path, map_location="cpu", weights_only=False, mmap=True)


def model_config(ck: dict) -> dict:
    """Architecture of a checkpoint, migrating legacy ``args``-style checkpoints."""
    if "config" in ck:
        return ck["config"]["model"]
    args = ck.get("args", {})
    vocab = 256 if args.get("task") == "lm" else 128
    if args.get("model", "stack") == "baseline":
        return dict(model="baseline", vocab_size=vocab, dim=args.get("d", 256),
                    heads=args.get("heads", 4), layers=args.get("layers", 3),
                    ffn_ratio=args.get("ffn_ratio", 4))
    return dict(vocab_size=vocab, dim=args.get("d", 256), heads=args.get("heads", 4),
                block_size=args.get("b", 16), topk=args.get("read_m") or 64,
                arch=args.get("arch") or "Lx2,G", ffn_ratio=args.get("ffn_ratio", 4))


def fault_point(name: str) -> None:
    """Host-side fault injection hook (see :mod:`exploration_b200.runtime.faults`)."""
    from .faults import maybe_fail
    maybe_fail(name)
