"""Streaming prefill and paged (optionally multi-GPU) sparse inference.

``InferenceSession.prefill`` encodes one prompt in block-aligned encoder
chunks, writes the raw K/V of this rank's sequence shard into a tiered cache
and keeps the encoded state only at the requested query positions.
``iter_logits`` then runs the G rounds with paged exact top-k attention and
yields logits one query chunk at a time (reference: st/runtime/inference.py).

Cache tiers (chosen by :func:`.memory.plan_inference`):

* ``cuda``: K/V resident in HBM (180 GB per B200 holds 1M tokens of a 1B
  model many times over); pages are views, nothing is copied.
* ``cpu``: K/V in *pinned* host memory. Pages are copied to the GPU on a
  side stream one page ahead of use, so PCIe transfer overlaps scoring.
* ``disk``: K/V in preallocated files (``posix_fallocate`` fails early
  instead of a SIGBUS mid-prefill) mapped with ``torch.from_file``. Pages
  are staged into pinned buffers and copied ahead on the side stream.

All tiers compute identical values; tests compare them with the in-core
forward.
"""
from __future__ import annotations

import os
import shutil
import tempfile
from pathlib import Path

import torch
import torch.distributed as dist

from ..ops.sparse import TensorPages, sparse_attention
from .faults import maybe_fail
from .memory import plan_inference

NATIVE_PREFILL_CHUNK = 16384   # prefill chunk (tokens) on the native CUDA path


def _allocate_file(path: Path, size: int) -> None:
    with open(path, "xb") as handle:
        if hasattr(os, "posix_fallocate"):
            os.posix_fallocate(handle.fileno(), 0, size)
        else:
            handle.truncate(size)


class KVCache(TensorPages):
    """Write-once raw K/V storage for one rank's shard ``[offset, offset + length)``."""

    def __init__(self, batch, length, heads, dim, dtype, device, plan, offset=0, cache_dir=None):
        self.directory = None
        self.tier = plan.cache
        self._copy_stream = None
        shape = (batch, length, heads, dim)
        device = torch.device(device)
        if self.tier == "disk":
            self.directory = tempfile.TemporaryDirectory(prefix="eb200-kv-", dir=cache_dir)
            count = batch * length * heads * dim
            size = count * torch.empty((), dtype=dtype).element_size()
            tensors = []
            for name in ("keys", "values"):
                path = Path(self.directory.name) / f"{name}.bin"
                _allocate_file(path, size)
                tensors.append(torch.from_file(str(path), shared=True, size=count,
                                               dtype=dtype).view(shape))
            k, v = tensors
        elif self.tier == "cpu":
            pin = device.type == "cuda" and torch.cuda.is_available()
            k = torch.empty(shape, dtype=dtype, pin_memory=pin)
            v = torch.empty(shape, dtype=dtype, pin_memory=pin)
        else:
            k = torch.empty(shape, dtype=dtype, device=device)
            v = torch.empty(shape, dtype=dtype, device=device)
        super().__init__(k, v, plan.page_tokens, offset)

    def write(self, start, k, v):
        lo = start - self.offset
        if lo < 0 or lo + k.shape[1] > self.length:
            raise ValueError("KV write outside the owned shard")
        self.k[:, lo:lo + k.shape[1]].copy_(k, non_blocking=self.tier == "cpu")
        self.v[:, lo:lo + v.shape[1]].copy_(v, non_blocking=self.tier == "cpu")

    # -- paged reads with one-page-ahead transfer ---------------------------

    def _stage(self, source, lo, hi, device):
        piece = source[:, lo:hi]
        if self.tier == "disk":
            pinned = torch.empty(piece.shape, dtype=piece.dtype, pin_memory=True)
            pinned.copy_(piece)
            piece = pinned
        return piece.to(device, non_blocking=True)

    def pages(self, device, indices=None, keys_only=False):
        device = torch.device(device)
        if self.tier == "cuda" or device.type != "cuda":
            yield from super().pages(device, indices, keys_only)
            return
        order = [i for i in (range(self.page_count) if indices is None else indices)
                 if i * self.page_tokens < self.length]
        if not order:
            return
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device)
        consumer = torch.cuda.current_stream(device)

        def issue(index):
            lo = index * self.page_tokens
            hi = min(lo + self.page_tokens, self.length)
            # The copy must not overwrite memory the consumer still reads.
            self._copy_stream.wait_stream(consumer)
            with torch.cuda.stream(self._copy_stream):
                key = self._stage(self.k, lo, hi, device)
                value = None if keys_only else self._stage(self.v, lo, hi, device)
                done = torch.cuda.Event()
                done.record(self._copy_stream)
            return self.offset + lo, key, value, done

        ahead = issue(order[0])
        for position in range(len(order)):
            start, key, value, done = ahead
            ahead = issue(order[position + 1]) if position + 1 < len(order) else None
            consumer.wait_event(done)
            key.record_stream(consumer)
            if value is not None:
                value.record_stream(consumer)
            yield start, key, value

    def close(self):
        self.k = self.v = None
        if self.directory is not None:
            self.directory.cleanup()
            self.directory = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class InferenceSession:
    """A write-once raw-KV cache plus bounded query states for one prompt.

    ``prefill(ids_cpu, positions_cpu)`` then ``iter_logits()``. Every rank of
    ``group`` passes the same ids and positions. Use as a context manager so
    caches (and their files) are released deterministically.
    """

    def __init__(self, model, *, group=None, cache="auto", cache_dir=None, memory_fraction=0.8,
                 page_tokens=65536, encoder_chunk=4096, query_chunk=16, workspace_mb=256,
                 max_query_states_mb=256):
        if model.training:
            raise ValueError("call model.eval() before creating an inference session")
        self.model, self.group = model, group
        first = next(model.parameters())
        self.device, self.dtype = first.device, first.dtype
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if not 1 <= self.world <= 8:
            raise ValueError("inference supports 1..8 ranks")
        self.options = dict(cache=cache, cache_dir=cache_dir, memory_fraction=memory_fraction,
                            page_tokens=page_tokens, encoder_chunk=encoder_chunk,
                            query_chunk=query_chunk, workspace_mb=workspace_mb)
        self.max_query_bytes = max_query_states_mb * (1 << 20)
        self.cache = None
        self.query_states = None
        self.query_directory = None
        self.ready = False

    def _query_storage(self, batch, count, query_bytes):
        """Zero-initialised ``[B, Q, dim]`` query states (GPU, host or a mapped file)."""
        if query_bytes > self.max_query_bytes:
            directory = self.options["cache_dir"]
            if not directory:
                raise MemoryError("query states exceed --max-query-states-mb; pass --cache-dir or "
                                  "evaluate fewer positions")
            local = max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
            if query_bytes * local + (1 << 30) > shutil.disk_usage(directory).free:
                raise MemoryError("insufficient disk space for the query-state cache")
            self.query_directory = tempfile.TemporaryDirectory(prefix="eb200-queries-", dir=directory)
            path = Path(self.query_directory.name) / "queries.bin"
            _allocate_file(path, query_bytes)
            # A fresh file reads as zeros: rows owned by other ranks stay zero.
            return torch.from_file(str(path), shared=True, size=batch * count * self.model.dim,
                                   dtype=self.dtype).view(batch, count, self.model.dim)
        place = self.device if self.plan.cache == "cuda" else "cpu"
        return torch.zeros(batch, count, self.model.dim, dtype=self.dtype, device=place)

    @torch.inference_mode()
    def prefill(self, input_ids, positions):
        if self.cache is not None or self.ready:
            raise RuntimeError("use a new session for each prompt")
        if input_ids.ndim != 2 or min(input_ids.shape) < 1 or input_ids.device.type != "cpu":
            raise ValueError("input_ids must be a nonempty CPU [B,N] tensor")
        batch, n = input_ids.shape
        positions = positions.to("cpu", dtype=torch.long)
        if positions.ndim != 2 or positions.shape[0] != batch or positions.shape[1] < 1:
            raise ValueError("positions must be nonempty [B,Q]")
        if (positions < 0).any() or (positions >= n).any():
            raise ValueError("query positions must lie within the prompt")
        m = self.model
        b = m.block_size
        shard = -(-n // (self.world * b)) * b
        start, end = self.rank * shard, min((self.rank + 1) * shard, n)
        if start >= end:
            raise ValueError("each inference rank must own at least one token block")
        self.plan = plan_inference(m, batch, end - start, **self.options)
        element = torch.empty((), dtype=self.dtype).element_size()
        self.positions = positions
        sorted_pos, sorted_index = positions.sort(1)
        # L layers of receptive field: recompute L blocks before the shard.
        warm = max(0, start - len(m.local) * b)
        halos = [None] * len(m.local)
        try:
            self.cache = KVCache(batch, end - start, m.heads, m.hd, self.dtype, self.device,
                                 self.plan, start, self.options["cache_dir"])
            self.query_states = self._query_storage(batch, positions.shape[1],
                                                    positions.numel() * m.dim * element)
            step = self.plan.encoder_chunk
            if self.device.type == "cuda" and getattr(m, "backend", "auto") != "torch":
                # Values do not depend on the chunk; on the native path bigger
                # chunks mean far fewer launches (the workspace holds them).
                step = max(step, NATIVE_PREFILL_CHUNK // b * b)
            for lo in range(warm, end, step):
                hi = min(end, lo + step)
                maybe_fail("prefill_chunk")
                x = m.embedding(input_ids[:, lo:hi].to(self.device, non_blocking=True))
                for i, layer in enumerate(m.local):
                    previous = halos[i]
                    halos[i] = x[:, -b:].clone()
                    x = layer(x, previous=previous, start=lo)
                k, v = m.raw_kv(x, None)
                keep = max(start, lo)
                if hi <= keep:
                    continue
                self.cache.write(keep, k[:, keep - lo:], v[:, keep - lo:])
                bounds = torch.tensor([keep, hi])
                for row in range(batch):
                    left, right = torch.searchsorted(sorted_pos[row], bounds).tolist()
                    if right <= left:
                        continue
                    cols = sorted_index[row, left:right]
                    rows_needed = (positions[row, cols] - lo).to(self.device)
                    gathered = x[row, rows_needed]
                    if self.query_states.device.type == "cpu":
                        self.query_states[row, cols] = gathered.cpu()
                    else:
                        self.query_states[row, cols.to(self.query_states.device)] = gathered
            self.ready = True
        except BaseException:
            self.close()
            raise
        return self

    @torch.inference_mode()
    def iter_logits(self, return_selection=False):
        if not self.ready:
            raise RuntimeError("prefill must complete before inference")
        m = self.model
        for lo in range(0, self.positions.shape[1], self.plan.query_chunk):
            hi = min(lo + self.plan.query_chunk, self.positions.shape[1])
            # A private contiguous copy: the all-reduce below works in place.
            z = self.query_states[:, lo:hi].to(self.device, non_blocking=True, copy=True)
            z = z.contiguous()
            if self.world > 1:
                dist.all_reduce(z, group=self.group)
            pos = self.positions[:, lo:hi].to(self.device)
            selection = None
            for rd in m.reads:
                q = m._query(rd, z).reshape(*z.shape[:2], m.heads, m.hd)
                result = sparse_attention(q, self.cache, pos, m.block_size, m.topk, backend=m.backend,
                                          group=self.group, score_page_tokens=self.plan.score_tokens,
                                          return_selection=return_selection)
                ctx, selection = result if return_selection else (result, None)
                z = m._finish(rd, z, ctx.reshape(*z.shape[:2], m.dim))
            for j in range(0, hi - lo, self.plan.head_chunk):
                stop = min(j + self.plan.head_chunk, hi - lo)
                from ..ops import fused
                hidden = fused.layer_norm(z[:, j:stop], m.final_norm, m.backend)
                logits = fused.linear(hidden, m.lm_head, m.backend)
                yield slice(lo + j, lo + stop), logits, selection

    def close(self):
        if self.cache is not None:
            self.cache.close()
            self.cache = None
        self.query_states = None
        if self.query_directory is not None:
            self.query_directory.cleanup()
            self.query_directory = None
        self.ready = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
