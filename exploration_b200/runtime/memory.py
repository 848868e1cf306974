"""Memory planning for training and paged inference on a B200 node.

Training: :func:`training_estimate` adds up what one rank of this framework
holds for a step, item by item, from the buffers it actually allocates:

* the flat parameter state of the graph step (fp32 master weights, the fp32
  gradient in the symmetric heap, the bf16 GEMM shadow, and AdamW's two fp32
  moments, which ZeRO-1 divides over the data-parallel ranks);
* the activations kept for backward per token and per layer on the native
  path (bf16 GEMM inputs, the fp32 residual stream, the kept GELU derivative,
  the gated-attention row statistics), or only the layer inputs when blocks
  are recomputed;
* the Ulysses exchange buffers of the NVLink path when CP > 1;
* a fixed allowance for kernel workspaces, NCCL and allocator slack.

It is an estimate for choosing CP and refusing runs that cannot fit, not a
measurement (the reference's planner is st/runtime/memory.py:43-112; this one
is derived from this framework's own buffers).

Inference: :func:`plan_inference` places the raw K/V of the read rounds for
this rank's shard in the fastest tier that holds it: device HBM (180 GB per
B200), pinned host memory (page-locked memory is taken from a smaller share of
the node's free RAM, divided among the node's ranks), or preallocated files.
Every transient buffer of the streaming loops (prefill chunk, transfer page,
score tile, head slice) is bounded by one workspace size.
"""
from __future__ import annotations

import os
import shutil
from dataclasses import asdict, dataclass

import torch

GiB = 1 << 30
MiB = 1 << 20

B200_HBM_BYTES = 183_359 * MiB          # what nvidia-smi reports for one B200
RUNTIME_ALLOWANCE = 2 * GiB             # kernel workspaces, NCCL buffers, allocator slack
PINNED_SHARE = 0.7                      # page-locked fraction of a rank's share of free host RAM
CACHE_TIERS = ("auto", "cuda", "cpu", "disk")


def available_host_memory() -> int | None:
    """Free host RAM in bytes (``MemAvailable``), or ``None`` when it cannot be read."""
    try:
        with open("/proc/meminfo") as handle:
            for line in handle:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    try:
        import psutil
    except ImportError:
        return None
    return psutil.virtual_memory().available


def ranks_on_this_node() -> int:
    return max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1")))


# ---------------------------------------------------------------------------
# training
# ---------------------------------------------------------------------------

def _layer_counts(model):
    if hasattr(model, "local"):
        return len(model.local), len(model.reads)
    return len(model.blocks), 0


def _ffn_hidden(model) -> int:
    layers = model.local if hasattr(model, "local") else model.blocks
    for layer in layers:
        return layer.ffn[0].out_features
    return 4 * model.dim


def activation_bytes_per_token(model, recompute: bool) -> int:
    """Bytes kept for backward per local token, summed over all layers."""
    d = model.dim
    hidden = _ffn_hidden(model)
    local_layers, read_rounds = _layer_counts(model)
    if recompute:
        # Only each layer's fp32 input survives; one layer is rebuilt at a time.
        live = 2 * d + 6 * d + 2 * d + 4 * d + 4 * hidden
        return 4 * d * (local_layers + read_rounds) + live
    # LayerNorm outputs (bf16), QKV or q (bf16), attention output (bf16), fp32
    # residual after attention, FFN input (bf16), GELU output and derivative
    # (bf16, hidden wide), fp32 residual after the FFN.
    block = 2 * d + 6 * d + 2 * d + 4 * d + 2 * d + 4 * hidden + 4 * d
    read = block - 4 * d + 4 * d + 8 * model.heads      # q instead of QKV, fp32 row statistics per head
    raw_kv = 4 * d if read_rounds else 0                # bf16 K and V shared by every read round
    return local_layers * block + read_rounds * read + raw_kv


def training_estimate(model, batch, length, cp_size=1, checkpoint_chunks=True, dp_size=1) -> dict:
    """One rank's training footprint in bytes (see the module docstring for the items)."""
    params = sum(p.numel() for p in model.parameters())
    local = -(-length // (cp_size * model.block_size)) * model.block_size
    flat_state = params * (4 + 4 + 2) + params * 8 // max(1, dp_size)
    tokens = batch * local
    activations = tokens * activation_bytes_per_token(model, checkpoint_chunks)
    activations += tokens * 4 * model.lm_head.out_features                # fp32 logits of the loss slices
    exchange = 0
    if cp_size > 1:
        # Head-layout q/k/v (and their gradients) over the whole sequence for
        # this rank's heads, plus the landed sequence-layout copies.
        exchange = tokens * model.dim * 2 * 3 * 2 + tokens * model.dim * 2 * 2
    total = flat_state + activations + exchange + RUNTIME_ALLOWANCE
    return {"parameters": params, "parameter_optimizer_bytes": flat_state,
            "estimated_activation_bytes": activations, "exchange_bytes": exchange,
            "estimated_total_bytes": total, "local_tokens": local, "context_parallel": cp_size,
            "device_capacity_bytes": B200_HBM_BYTES,
            "note": "Capacity estimate from this framework's buffers; measure peak memory on the target GPU."}


# ---------------------------------------------------------------------------
# paged inference
# ---------------------------------------------------------------------------

@dataclass
class InferencePlan:
    cache: str                         # tier of the K/V: cuda, cpu (pinned) or disk
    cache_bytes: int                   # K/V bytes of this rank's shard
    gpu_budget_bytes: int              # device bytes the K/V may take
    page_tokens: int                   # tokens per host/disk -> device transfer page
    encoder_chunk: int                 # prefill tokens per encoder pass
    query_chunk: int                   # queries per read pass
    score_tokens: int                  # keys per block-score tile
    head_chunk: int                    # queries per LM-head slice
    host_available_bytes: int | None

    def to_dict(self) -> dict:
        return asdict(self)


def _device_budget(param, memory_fraction) -> int:
    if not param.is_cuda:
        return 0
    free, capacity = torch.cuda.mem_get_info(param.device)
    # ``free`` is measured with the weights resident; the runtime allowance
    # stays free for the kernels' own buffers.
    return max(0, min(int(capacity * memory_fraction), free - RUNTIME_ALLOWANCE))


def _choose_tier(cache, need, device_budget, pinned_budget, cache_dir, on_cuda) -> str:
    if cache != "auto":
        return cache
    if on_cuda and need < device_budget:
        return "cuda"
    if pinned_budget is None:
        # Free RAM unknown: a small cache still goes to host memory.
        if need <= 2 * GiB:
            return "cpu"
    elif need < pinned_budget:
        return "cpu"
    if cache_dir:
        return "disk"
    raise MemoryError(f"the K/V shard needs {need / GiB:.2f} GiB per rank; pass --cache-dir for disk "
                      "paging or run on more inference ranks")


def _fit(limit_bytes, bytes_per_item, cap, multiple=1) -> int:
    """Largest multiple of ``multiple`` (at least one) not above ``cap`` whose items fit in ``limit_bytes``."""
    count = min(cap, limit_bytes // max(1, bytes_per_item))
    return max(multiple, count // multiple * multiple)


def plan_inference(model, batch, local_length, *, cache="auto", memory_fraction=0.8, page_tokens=65536,
                   encoder_chunk=4096, query_chunk=16, workspace_mb=256, cache_dir=None) -> InferencePlan:
    """Tier of the K/V cache and the chunk sizes of prefill and the read passes."""
    if not 0 < memory_fraction < 1:
        raise ValueError("positive sizes and 0 < memory_fraction < 1 required")
    if min(batch, local_length, page_tokens, encoder_chunk, query_chunk, workspace_mb) < 1:
        raise ValueError("positive sizes and 0 < memory_fraction < 1 required")
    if cache not in CACHE_TIERS:
        raise ValueError("cache must be auto/cuda/cpu/disk")
    param = next(model.parameters())
    elem = param.element_size()
    block, dim = model.block_size, model.dim
    kv_bytes = 2 * batch * local_length * dim * elem
    workspace = workspace_mb * MiB
    need = kv_bytes + 4 * workspace                  # transfer pages and score tiles in flight
    device_budget = _device_budget(param, memory_fraction)
    host = available_host_memory()
    pinned_budget = None if host is None else int(host / ranks_on_this_node() * PINNED_SHARE)
    tier = _choose_tier(cache, need, device_budget, pinned_budget, cache_dir, param.is_cuda)
    if tier == "cuda" and (not param.is_cuda or need >= device_budget):
        raise MemoryError(f"GPU K/V needs {kv_bytes / GiB:.2f} GiB plus workspace; use --cache auto/cpu/disk")
    if tier == "cpu" and pinned_budget is not None and need > pinned_budget:
        raise MemoryError(f"pinned K/V needs {kv_bytes / GiB:.2f} GiB; free host RAM is "
                          f"{(host or 0) / GiB:.2f} GiB; use --cache disk")
    if tier == "disk":
        if not cache_dir:
            raise ValueError("disk cache needs --cache-dir on a filesystem with room for the shard")
        os.makedirs(cache_dir, exist_ok=True)
        if (kv_bytes + GiB) * ranks_on_this_node() > shutil.disk_usage(cache_dir).free:
            raise MemoryError("insufficient free disk space for the local K/V shard")
    heads, topk = model.heads, model.topk
    # A transfer page holds K and V of `page` tokens; two pages are in flight.
    page = _fit(workspace // 2, 2 * batch * dim * elem, page_tokens, block)
    # A prefill chunk keeps about 24 activations of width `dim` per token alive.
    enc = _fit(workspace, 24 * batch * dim * elem, encoder_chunk, block)
    # A query gathers `topk` selected blocks of `block` keys per head (fp32 scores).
    queries = _fit(workspace, 4 * batch * heads * topk * block, query_chunk)
    # A score tile is fp32 logits of every query of the chunk against `score` keys.
    score = min(page, _fit(workspace // 4, 4 * batch * heads * queries, page, block))
    vocab = model.lm_head.out_features
    head = _fit(workspace, 4 * batch * vocab, queries)
    return InferencePlan(tier, kv_bytes, device_budget, page, enc, queries, score, head, host)
