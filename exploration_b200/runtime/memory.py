"""Capacity planning for training and paged inference.

Estimates are conservative and only used to choose a configuration or to
refuse an obviously over-budget run; they are not throughput promises
(reference: st/runtime/memory.py:43-112). Budgets assume a B200: 180 GB of
HBM3e per GPU, so the GPU tier of the KV cache is the default for far longer
contexts than on smaller parts.
"""
from __future__ import annotations

import os
import shutil
from dataclasses import asdict, dataclass

import torch

GiB = 1 << 30
MiB = 1 << 20


def available_host_memory() -> int | None:
    try:
        with open("/proc/meminfo") as handle:
            for line in handle:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    try:
        import psutil
        return psutil.virtual_memory().available
    except ImportError:
        return None


@dataclass
class InferencePlan:
    cache: str
    cache_bytes: int
    gpu_budget_bytes: int
    page_tokens: int
    encoder_chunk: int
    query_chunk: int
    score_tokens: int
    head_chunk: int
    host_available_bytes: int | None

    def to_dict(self) -> dict:
        return asdict(self)


def _local_processes() -> int:
    return max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1")))


def plan_inference(model, batch, local_length, *, cache="auto", memory_fraction=0.8,
                   page_tokens=65536, encoder_chunk=4096, query_chunk=16, workspace_mb=256,
                   cache_dir=None) -> InferencePlan:
    """Pick the KV tier (cuda -> cpu -> disk) and every streaming chunk size."""
    if not 0 < memory_fraction < 1 or min(batch, local_length, page_tokens, encoder_chunk,
                                          query_chunk, workspace_mb) < 1:
        raise ValueError("positive sizes and 0 < memory_fraction < 1 required")
    if cache not in ("auto", "cuda", "cpu", "disk"):
        raise ValueError("cache must be auto/cuda/cpu/disk")
    param = next(model.parameters())
    b, dim, heads = model.block_size, model.dim, model.heads
    element = param.element_size()
    total = 2 * batch * local_length * dim * element
    if param.is_cuda:
        free, capacity = torch.cuda.mem_get_info(param.device)
        # Free memory is measured after the weights; keep slack for kernel
        # workspaces, NCCL buffers and allocator fragmentation.
        budget = max(0, min(int(capacity * memory_fraction), free - 2 * GiB))
    else:
        budget = 0
    workspace = workspace_mb * MiB
    host = available_host_memory()
    host_budget = None if host is None else host / _local_processes()
    need = total + 4 * workspace
    if cache == "auto":
        if param.is_cuda and need < budget:
            cache = "cuda"
        elif host_budget is not None and need < host_budget * 0.7:
            cache = "cpu"
        elif host_budget is None and need <= 2 * GiB:
            cache = "cpu"
        elif cache_dir:
            cache = "disk"
        else:
            raise MemoryError(f"KV needs {total / GiB:.2f} GiB per rank; pass --cache-dir for disk "
                              "paging or use more inference ranks")
    if cache == "cuda" and (not param.is_cuda or need >= budget):
        raise MemoryError(f"GPU KV needs {total / GiB:.2f} GiB plus workspace; use --cache auto/cpu/disk")
    if cache == "cpu" and host_budget is not None and need > host_budget * 0.7:
        raise MemoryError(f"CPU KV needs {total / GiB:.2f} GiB; available RAM {host / GiB:.2f} GiB")
    if cache == "disk":
        if not cache_dir:
            raise ValueError("disk cache needs --cache-dir on a filesystem with room for the shard")
        os.makedirs(cache_dir, exist_ok=True)
        if (total + GiB) * _local_processes() > shutil.disk_usage(cache_dir).free:
            raise MemoryError("insufficient free disk space for the local KV shard")
    page = max(b, min(page_tokens, workspace // max(2 * batch * dim * element, 1)) // b * b)
    enc = max(b, min(encoder_chunk, workspace // max(24 * batch * dim * element, 1)) // b * b)
    qc = max(1, min(query_chunk, workspace // max(batch * heads * model.topk * b * 4, 1)))
    score = max(b, min(page, workspace // max(4 * batch * heads * qc * 4, 1)) // b * b)
    head_chunk = max(1, min(qc, workspace // max(batch * model.lm_head.out_features * 4, 1)))
    return InferencePlan(cache, total, budget, page, enc, qc, score, head_chunk, host)


def training_estimate(model, batch, length, cp_size=1, checkpoint_chunks=True) -> dict:
    """Parameter/optimizer bytes (16 B/param) plus an activation factor per layer."""
    params = sum(p.numel() for p in model.parameters())
    local = -(-length // (cp_size * model.block_size)) * model.block_size
    layers = len(model.local) if hasattr(model, "local") else len(model.blocks)
    reads = len(model.reads) if hasattr(model, "reads") else layers
    factor = (layers * 2 + reads * 8 + 12) if checkpoint_chunks else (layers * 16 + reads * 20 + 12)
    activations = batch * local * model.dim * 4 * factor
    return {"parameters": params, "parameter_optimizer_bytes": params * 16,
            "estimated_activation_bytes": activations,
            "estimated_total_bytes": params * 16 + activations + 2 * GiB,
            "local_tokens": local, "context_parallel": cp_size,
            "note": "Capacity estimate; measure peak memory on the target GPU."}
