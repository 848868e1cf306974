"""Paged exact top-k sparse attention: the inference-time read operator.

For each query row (position ``p``), head and visible remote block ``j``
(``j < p // b - 1`` and fully inside the KV shard), the exact block score
``s_j = logsumexp_{i in j} q . k_i / sqrt(D)`` is computed from the raw keys
(reference: st/ops/sparse.py:99-174). The ``topk`` best blocks per head are
popped into one softmax together with the local window (blocks ``p//b - 1``
and ``p//b``, tokens ``<= p``); a popped block carries the gate bias
``s_j - log Z_R`` where ``Z_R`` sums the masses of *all* visible remote
blocks, selected or not. With ``topk >= blocks`` this equals the dense gated
operator.

Work is bounded: scoring streams key tiles of ``score_page_tokens`` and
keeps a running top-k plus a running ``log Z_R``; the pop reads only the
pages that hold a selected block or a local window. With a process group the
KV cache is a sequence shard per rank: top-k candidates, ``Z_R`` and the
per-rank partial outputs are merged globally, so ``topk`` stays global.
CUDA tensors run the sm_100a kernels (``csrc/sparse``); CPU tensors run the
torch reference below.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..config import canonical_backend
from . import _native
from .gated_reference import NEG_INF, work_dtype
from .launch import record


def _finite_or_zero(x):
    return torch.where(torch.isfinite(x), x, torch.zeros_like(x))


class TensorPages:
    """An in-memory KV shard exposed as block-aligned pages.

    ``k, v [B, N, H, D]`` hold tokens ``[offset, offset + N)`` of the prompt.
    The same protocol (``pages``/``touched_pages``) is served by the tiered
    cache of :mod:`exploration_b200.runtime.inference`.
    """

    def __init__(self, k, v, page_tokens: int = 65536, offset: int = 0):
        self.k, self.v = k, v
        self.page_tokens, self.offset = page_tokens, offset
        self.length = k.shape[1]

    @property
    def page_count(self) -> int:
        return -(-self.length // self.page_tokens)

    def page(self, index: int, device, keys_only: bool = False):
        lo = index * self.page_tokens
        hi = min(lo + self.page_tokens, self.length)
        key = self.k[:, lo:hi].to(device, non_blocking=True)
        value = None if keys_only else self.v[:, lo:hi].to(device, non_blocking=True)
        return self.offset + lo, key, value

    def pages(self, device, indices=None, keys_only: bool = False):
        for index in (range(self.page_count) if indices is None else indices):
            if index * self.page_tokens < self.length:
                yield self.page(index, device, keys_only)

    def touched_pages(self, ids, positions, b: int) -> list:
        """Pages holding a selected block or a local-window block of any row."""
        local = torch.div(positions, b, rounding_mode="floor")
        blocks = torch.cat((ids.reshape(-1), (local - 1).reshape(-1), local.reshape(-1)))
        tokens = blocks.to(torch.int64) * b
        inside = (tokens >= self.offset) & (tokens < self.offset + self.length)
        pages = torch.div(tokens[inside] - self.offset, self.page_tokens, rounding_mode="floor")
        return pages.unique().cpu().tolist()


# ----------------------------------------------------------------------------
# torch reference pieces
# ----------------------------------------------------------------------------

def block_scores_reference(q, k, positions, b, offset):
    """Visible block scores ``[B, Q, H, G]`` of one key tile starting at ``offset``."""
    dtype = work_dtype(q)
    n = k.shape[1]
    pad = (-n) % b
    kh = k.transpose(1, 2).to(dtype)
    if pad:
        kh = torch.nn.functional.pad(kh, (0, 0, 0, pad))
    a = (q.transpose(1, 2).to(dtype) @ kh.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    a[..., n:] = NEG_INF
    scores = a.unflatten(-1, (-1, b)).logsumexp(-1).transpose(1, 2)   # [B,Q,H,G]
    first = offset // b
    block = torch.arange(scores.shape[-1], device=q.device) + first
    pos = positions[:, :, None, None]
    visible = ((block < torch.div(pos, b, rounding_mode="floor") - 1)
               & ((block + 1) * b <= offset + n) & (pos >= 0))
    return scores.masked_fill(~visible, NEG_INF)


def pop_reference(q, k, v, positions, ids, scores, log_zr, b, offset):
    """Softmax over local window + selected blocks restricted to one page.

    Returns the page's normalised output ``[B,Q,H,D]`` and its log mass
    ``[B,Q,H]`` (``-inf`` when the page holds none of the row's keys).
    """
    dtype = work_dtype(q)
    batch, queries, heads, dim = q.shape
    n = k.shape[1]
    local_base = torch.div(positions, b, rounding_mode="floor") - 1        # [B,Q]
    local_blocks = torch.stack((local_base, local_base + 1), -1)           # [B,Q,2]
    local_blocks = local_blocks[:, :, None, :].expand(-1, -1, heads, -1)
    blocks = torch.cat((local_blocks, ids), -1)                            # [B,Q,H,2+K]
    zr = _finite_or_zero(log_zr)
    window_shape = (*scores.shape[:-1], 2)
    bias = torch.cat((scores.new_zeros(window_shape), scores - zr[..., None]), -1)
    selected_ok = (ids >= 0) & torch.isfinite(scores)
    block_ok = torch.cat((selected_ok.new_ones(window_shape), selected_ok), -1)
    token = blocks[..., None] * b + torch.arange(b, device=q.device)       # [B,Q,H,S,b]
    pos = positions[:, :, None, None, None]
    ok = (block_ok[..., None] & (pos >= 0) & (token >= 0) & (token <= pos)
          & (token >= offset) & (token < offset + n))
    token = token.flatten(-2)
    ok = ok.flatten(-2)
    bias = bias[..., None].expand(-1, -1, -1, -1, b).flatten(-2)
    rel = (token - offset).clamp(0, n - 1)
    rows = torch.arange(batch, device=q.device)[:, None, None, None]
    hs = torch.arange(heads, device=q.device)[None, None, :, None]
    kr = k[rows, rel, hs].to(dtype)                                        # [B,Q,H,S*b,D]
    vr = v[rows, rel, hs].to(dtype)
    logits = (kr @ q.to(dtype)[..., None]).squeeze(-1) / math.sqrt(dim) + bias
    logits = logits.masked_fill(~ok, NEG_INF)
    lse = logits.logsumexp(-1)
    weights = torch.exp(logits - _finite_or_zero(lse)[..., None])
    out = (weights[..., None, :] @ vr).squeeze(-2)
    return out, lse


def lse_merge(out, lse, part, part_lse):
    """Combine two normalised partial softmax reads by their log masses."""
    total = torch.logaddexp(lse, part_lse)
    ref = _finite_or_zero(total)
    merged = out * torch.exp(lse - ref)[..., None] + part * torch.exp(part_lse - ref)[..., None]
    return merged, total


def _topk_merge(scores, ids, new_scores, new_ids, topk):
    candidates = torch.cat((scores, new_scores), -1)
    candidate_ids = torch.cat((ids, new_ids), -1)
    best, take = candidates.topk(topk, -1)
    return best, candidate_ids.gather(-1, take)


def _global_logsumexp(x, group):
    peak = x.clone()
    dist.all_reduce(peak, op=dist.ReduceOp.MAX, group=group)
    ref = _finite_or_zero(peak)
    mass = torch.exp(x - ref)
    dist.all_reduce(mass, group=group)
    return ref + mass.log()


# ----------------------------------------------------------------------------
# public operator
# ----------------------------------------------------------------------------

@torch.inference_mode()
def _score_chunks(cache, device, tile, native):
    """``(first token, keys)`` pieces to score: a cache resident on the device in
    one pass (the native scorer streams any length), otherwise page by page in
    tiles of ``tile`` tokens."""
    if native and isinstance(cache, TensorPages) and cache.k.device == device and cache.k.is_contiguous():
        yield cache.offset, cache.k
        return
    for start, keys, _ in cache.pages(device, keys_only=True):
        for lo in range(0, keys.shape[1], tile):
            yield start + lo, keys[:, lo:lo + tile]


def sparse_attention(q, cache, positions, block_size, topk, backend="auto", group=None,
                     score_page_tokens=65536, return_selection=False):
    """Exact scoring, global top-k, gate and sparse pop over a paged KV cache.

    ``q [B,Q,H,D]`` and ``positions [B,Q]`` are replicated over ``group``.
    Returns ``[B,Q,H,D]`` in q's dtype (and the selection when asked).
    """
    b = block_size
    if topk < 1 or score_page_tokens < b or cache.page_tokens % b or cache.offset % b:
        raise ValueError("topk must be positive and cache pages/offset block aligned")
    path = canonical_backend(backend)
    native = path != "torch" and q.is_cuda
    if path == "cuda" and not q.is_cuda:
        raise ValueError("the native backend runs on CUDA tensors")
    ext = _native.native(q) if native else None
    dtype = work_dtype(q)
    shape = q.shape[:3]
    tile = max(b, score_page_tokens // b * b)
    pos32 = positions.to(torch.int32).contiguous() if native else None
    qc = q.contiguous()
    scores = ids = log_zr = None
    for first, chunk in _score_chunks(cache, q.device, tile, native):
        if native and ext.block_scores_tc_supported(qc, chunk, b, topk):
            part_scores, part_ids, part_zr = ext.block_scores_topk_tc(
                qc, chunk.contiguous(), pos32, b, first, topk)
            record("block_scores_topk", dtype=str(q.dtype), head_dim=q.shape[-1], block=b, path="tcgen05")
        elif native:
            part_scores, part_ids, part_zr = ext.block_scores_topk(
                qc, chunk.contiguous(), pos32, b, first, topk)
            record("block_scores_topk", dtype=str(q.dtype), head_dim=q.shape[-1], block=b)
        else:
            s = block_scores_reference(q, chunk, positions, b, first)
            part_zr = s.logsumexp(-1)
            count = min(topk, s.shape[-1])
            part_scores, part_ids = s.topk(count, -1)
            part_ids = part_ids + first // b
        part_scores, part_zr, part_ids = part_scores.to(dtype), part_zr.to(dtype), part_ids.to(torch.int64)
        if scores is None and part_scores.shape[-1] == topk:
            # The first piece already holds k candidates per row: no merge needed.
            scores, ids, log_zr = part_scores, part_ids, part_zr
            continue
        if scores is None:
            scores = torch.full((*shape, topk), NEG_INF, dtype=dtype, device=q.device)
            ids = torch.full(scores.shape, -1, dtype=torch.int64, device=q.device)
            log_zr = torch.full(shape, NEG_INF, dtype=dtype, device=q.device)
        log_zr = torch.logaddexp(log_zr, part_zr)
        scores, ids = _topk_merge(scores, ids, part_scores, part_ids, topk)
    if scores is None:                                   # an empty cache
        scores = torch.full((*shape, topk), NEG_INF, dtype=dtype, device=q.device)
        ids = torch.full(scores.shape, -1, dtype=torch.int64, device=q.device)
        log_zr = torch.full(shape, NEG_INF, dtype=dtype, device=q.device)
    distributed = group is not None and dist.is_initialized() and dist.get_world_size(group) > 1
    if distributed:
        world = dist.get_world_size(group)
        gathered_s = [torch.empty_like(scores) for _ in range(world)]
        gathered_i = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(gathered_s, scores.contiguous(), group=group)
        dist.all_gather(gathered_i, ids.contiguous(), group=group)
        scores, take = torch.cat(gathered_s, -1).topk(topk, -1)
        ids = torch.cat(gathered_i, -1).gather(-1, take)
        log_zr = _global_logsumexp(log_zr, group)
    if distributed or return_selection or not native:
        ids = ids.masked_fill(~torch.isfinite(scores), -1)   # the native pop skips -inf scores itself
    out = lse = None
    resident = native and isinstance(cache, TensorPages) and cache.k.device == q.device
    pieces = [(cache.offset, cache.k, cache.v)] if resident else \
        cache.pages(q.device, cache.touched_pages(ids, positions, b))
    for start, keys, values in pieces:
        if native:
            part, part_lse = ext.sparse_pop(qc, keys.contiguous(), values.contiguous(), pos32,
                                            ids.contiguous(), scores.float().contiguous(),
                                            log_zr.float().contiguous(), b, start)
            record("sparse_pop", dtype=str(q.dtype), head_dim=q.shape[-1], block=b)
            part, part_lse = part.to(dtype), part_lse.to(dtype)
        else:
            part, part_lse = pop_reference(q, keys, values, positions, ids, scores, log_zr, b, start)
        if out is None:
            out, lse = part, part_lse
        else:
            out, lse = lse_merge(out, lse, part, part_lse)
    if out is None:
        out = torch.zeros(q.shape, dtype=dtype, device=q.device)
        lse = torch.full(shape, NEG_INF, dtype=dtype, device=q.device)
    if distributed:
        weight = torch.exp(lse - _finite_or_zero(_global_peak(lse, group)))
        out = out * weight[..., None]
        dist.all_reduce(out, group=group)
        dist.all_reduce(weight, group=group)
        out = out / weight.clamp_min(torch.finfo(dtype).tiny)[..., None]
    result = out.to(q.dtype)
    if return_selection:
        return result, {"indices": ids, "scores": scores, "log_zr": log_zr}
    return result


def _global_peak(x, group):
    peak = x.clone()
    dist.all_reduce(peak, op=dist.ReduceOp.MAX, group=group)
    return peak
