"""Resumable checkpoints in the reference's format version 2.

The file is a ``torch.save`` dictionary whose layout is the interchange
format of both frameworks (st/runtime/checkpoint.py:39-93 in the reference)::

    {"format_version": 2,
     "model": CPU state dict (tied / shared weights stored once, aliased),
     "opt": optimizer state (consolidated on rank 0 for ZeRO-1),
     "config": {"model": ModelConfig.to_dict(), "runtime": {...}},
     "step": last completed step,
     "rng_by_rank": [{"torch", "python", "data", "cuda"?}, ...],
     "topology": {"world_size", "cp_size"}}

How this framework writes it: the model's tensors are staged from the device
into one pinned host buffer with asynchronous copies on a side stream and a
single synchronisation (parameters of the flat-parameter step are views of one
device buffer, so aliases are found by storage and offset, not by name); the
per-rank RNG states travel to rank 0 in one ``gather_object``; rank 0 writes a
temporary file next to the target, flushes it to disk, renames it over the
target and syncs the directory, so a crash leaves either the old or the new
checkpoint. Every rank learns rank 0's outcome and raises on failure.
"""
from __future__ import annotations

import os
import random
import tempfile
from pathlib import Path

import torch
import torch.distributed as dist

FORMAT_VERSION = 2


# ---------------------------------------------------------------------------
# RNG state: host generators, the data generator, and the current CUDA device's
# ---------------------------------------------------------------------------

_HOST_RNGS = {"torch": (torch.get_rng_state, torch.set_rng_state),
              "python": (random.getstate, random.setstate)}


def rng_state(generator: torch.Generator) -> dict:
    state = {name: get() for name, (get, _) in _HOST_RNGS.items()}
    state["data"] = generator.get_state()
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        state["cuda"] = torch.cuda.get_rng_state()
    return state


def restore_rng(state: dict, generator: torch.Generator) -> None:
    for name, (_, put) in _HOST_RNGS.items():
        put(state[name])
    generator.set_state(state["data"])
    if "cuda" in state and torch.cuda.is_available():
        torch.cuda.set_rng_state(state["cuda"])


# ---------------------------------------------------------------------------
# model state on the host
# ---------------------------------------------------------------------------

def _alias_key(t: torch.Tensor):
    return (t.device, t.untyped_storage().data_ptr(), t.storage_offset(), tuple(t.shape), tuple(t.stride()), t.dtype)


def cpu_state_dict(model) -> dict:
    """Host copy of ``model.state_dict()``; entries that alias one tensor stay one tensor.

    Device tensors are copied into a single pinned buffer by asynchronous
    copies on a side stream, then synchronised once.
    """
    state = model.state_dict()
    unique = {}
    for value in state.values():
        unique.setdefault(_alias_key(value), value.detach())
    on_device = [(key, t) for key, t in unique.items() if t.is_cuda]
    host = {key: t.cpu() for key, t in unique.items() if not t.is_cuda}
    if on_device:
        device = on_device[0][1].device
        sizes = [t.numel() * t.element_size() for _, t in on_device]
        offsets = [0]
        for size in sizes:
            offsets.append(offsets[-1] + (size + 63) // 64 * 64)   # 64-byte aligned slots
        staging = torch.empty(offsets[-1], dtype=torch.uint8, pin_memory=True)
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for (key, t), start, size in zip(on_device, offsets, sizes):
                slot = staging[start:start + size].view(t.dtype).view(t.shape)
                slot.copy_(t.contiguous() if not t.is_contiguous() else t, non_blocking=True)
                host[key] = slot
        stream.synchronize()
    return {name: host[_alias_key(value)] for name, value in state.items()}


# ---------------------------------------------------------------------------
# writing
# ---------------------------------------------------------------------------

def _write_atomically(target: Path, payload: dict) -> None:
    target.parent.mkdir(parents=True, exist_ok=True)
    fd, temp = tempfile.mkstemp(dir=target.parent, prefix=f".{target.name}.", suffix=".partial")
    try:
        with os.fdopen(fd, "wb") as handle:
            torch.save(payload, handle)
            handle.flush()
            os.fsync(handle.fileno())
        os.replace(temp, target)
    except BaseException:
        if os.path.exists(temp):
            os.unlink(temp)
        raise
    try:                                   # make the rename itself durable
        directory = os.open(target.parent, os.O_RDONLY)
    except OSError:
        return
    try:
        os.fsync(directory)
    except OSError:
        pass
    finally:
        os.close(directory)


def _agree(parallel, error):
    """Rank 0's outcome on every rank (the same collective on all of them)."""
    if parallel.world_size == 1:
        return error
    box = [error]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def save(path, model, optimizer, config, step, generator, parallel) -> None:
    if hasattr(optimizer, "consolidate_state_dict"):
        optimizer.consolidate_state_dict(to=0)
    mine = rng_state(generator)
    states = [mine]
    if parallel.world_size > 1:
        states = [None] * parallel.world_size if parallel.rank == 0 else None
        dist.gather_object(mine, states, dst=0)
    error = None
    if parallel.rank == 0:
        try:
            payload = {"format_version": FORMAT_VERSION, "model": cpu_state_dict(model),
                       "opt": optimizer.state_dict(), "config": config, "step": step, "rng_by_rank": states,
                       "topology": {"world_size": parallel.world_size, "cp_size": parallel.cp_size}}
            fault_point("checkpoint_write")
            _write_atomically(Path(path), payload)
        except Exception as exc:              # reported on every rank below
            error = f"checkpoint save failed: {exc}"
    error = _agree(parallel, error)
    if error:
        raise RuntimeError(error)


def load(path):
    """Load a locally trusted checkpoint (it holds pickled optimizer and RNG state)."""
    return torch.load(path, map_location="cpu", weights_only=False, mmap=True)


# Checkpoints from before format 2 kept argparse-style keys under "args".
_LEGACY_KEYS = {"dim": ("d", 256), "heads": ("heads", 4), "ffn_ratio": ("ffn_ratio", 4)}


def model_config(ck: dict) -> dict:
    """Architecture of a checkpoint; legacy ``args`` checkpoints are migrated."""
    if "config" in ck:
        return ck["config"]["model"]
    args = ck.get("args", {})
    config = {"vocab_size": 256 if args.get("task") == "lm" else 128}
    config.update({key: args.get(old, default) for key, (old, default) in _LEGACY_KEYS.items()})
    if args.get("model", "stack") == "baseline":
        return {"model": "baseline", **config, "layers": args.get("layers", 3)}
    config.update(block_size=args.get("b", 16), topk=args.get("read_m") or 64, arch=args.get("arch") or "Lx2,G")
    return config


def fault_point(name: str) -> None:
    """Host-side fault injection hook (see :mod:`exploration_b200.runtime.faults`)."""
    from .faults import maybe_fail
    maybe_fail(name)
