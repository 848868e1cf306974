"""Stack: a decoder-only LM that trains dense and infers sparse.

Layers (reference: st/models/stack.py:1-59, 130-188):

* ``L`` layers (:class:`HaloMemoryBlock`) encode tokens with causal
  attention over a two-block window;
* one raw K/V projection (no RoPE) after the last ``L`` is written once and
  shared by every ``G`` round;
* ``G`` rounds (:class:`GlobalReadBlock`) turn the state ``z`` of each
  supervised position into a query and read the whole causal prefix through
  block-gated attention, then apply ``read_out``, a residual and an FFN;
* the LM head is a final LayerNorm and a projection tied to the embedding.

A block's gate score is its exact attention partition function
``s_j = logsumexp_{i in j} q . k_i / sqrt(D)``, written from the query at read
time and never stored. Training evaluates the gate densely over every block
(:meth:`forward_loss`, exact gated attention). Inference keeps the per-head
top-k blocks by ``s_j`` and pops their tokens (:mod:`..ops.sparse`); with
``topk >= blocks`` both are the same function.

``arch`` is a comma list of ``L``/``G`` items; ``XxN`` repeats with
independent weights and ``(X)xN`` cycles one shared module N times. All L
precede all G.
"""
from __future__ import annotations

import math
import re
from numbers import Integral

import torch
from torch import nn
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

from ..config import canonical_backend
from ..ops import fused
from ..ops.attention import dense_attention
from ..parallel.context import ParallelContext
from ..runtime import trace
from ..data.synthetic import KEY
from ..ops.gated_reference import block_log_mass, eager_gated
from ..ops.sparse import TensorPages, sparse_attention
from .blocks import FeedForward, HaloMemoryBlock, KVProjection, RotaryEmbedding

# On the native path one query tile covers this many supervised positions:
# the gated-attention kernel never materialises Q x N, so the only memory the
# tile bounds is a few [tile, dim] activations.
NATIVE_QUERY_TILE = 65536
NATIVE_LOSS_TILE = 65536


_ARCH_ITEM = re.compile(r"(?P<shared>\((?P<skind>[A-Za-z]+)\)x(?P<scount>\S*))|(?P<kind>[A-Za-z]+)(?:x(?P<count>\S*))?")


def parse_arch(arch):
    """``'Lx2,(G)x4'`` -> ``[(kind, count, shared), ...]`` in application order.

    ``L`` is a local halo encoder block, ``G`` a global read round; ``XxN``
    repeats ``X`` N times with independent weights, ``(X)xN`` applies one
    shared module N times, a bare ``X`` means ``Xx1``; every ``L`` precedes
    every ``G``.
    """
    if not isinstance(arch, str) or not arch.strip():
        raise ValueError("arch must be a nonempty spec like 'Lx2,G'")
    spec = []
    for item in (part.strip() for part in arch.split(",")):
        match = _ARCH_ITEM.fullmatch(item)
        if match is None:
            if item.startswith("("):
                raise ValueError(f"shared layers must look like '(X)xN': {item!r}")
            raise ValueError(f"unknown layer kind in arch item {item!r} (want L or G)")
        shared = match["shared"] is not None
        kind = match["skind"] if shared else match["kind"]
        count = match["scount"] if shared else (match["count"] if match["count"] is not None else "1")
        if kind not in ("L", "G"):
            raise ValueError(f"unknown layer kind in arch item {item!r} (want L or G)")
        if not count.isdigit() or int(count) < 1:
            raise ValueError(f"repeat count must be a positive integer in {item!r}")
        spec.append((kind, int(count), shared))
    if "GL" in "".join(kind for kind, _, _ in spec):      # some G before some L
        raise ValueError("all L layers must precede all G layers (encode -> read)")
    return spec


class GlobalReadBlock(nn.Module):
    """Query-side weights of one G round: query norm/projection, read-out, FFN."""

    def __init__(self, dim, ffn_ratio):
        super().__init__()
        self.q_norm = nn.LayerNorm(dim)
        self.wq = nn.Linear(dim, dim, bias=False)
        self.read_out = nn.Linear(dim, dim, bias=False)
        self.ffn_norm = nn.LayerNorm(dim)
        self.ffn = FeedForward(dim, ffn_ratio)


def _check_positive(**values):
    for name, value in values.items():
        if isinstance(value, bool) or not isinstance(value, Integral) or value < 1:
            raise ValueError(f"{name} must be a positive integer")


class StackModel(nn.Module):
    """``forward([B,N], sup=None) -> [B,N,vocab]``; ``forward(..., targets=)`` -> loss sums."""

    def __init__(self, vocab_size, dim=256, heads=4, block_size=16, topk=64, arch="Lx2,G",
                 ffn_ratio=4, pos_chunk=0, backend="auto", checkpoint_chunks=False,
                 encoder_chunk=1024, loss_chunk=128, attention_q_chunk=128,
                 attention_kv_chunk=4096):
        super().__init__()
        _check_positive(vocab_size=vocab_size, dim=dim, heads=heads, block_size=block_size, topk=topk)
        if isinstance(pos_chunk, bool) or not isinstance(pos_chunk, Integral) or pos_chunk < 0:
            raise ValueError("pos_chunk must be a non-negative integer (0 = auto)")
        if block_size < 2:
            raise ValueError("block_size must be at least 2")
        if dim % heads or (dim // heads) % 2:
            raise ValueError("dim / heads must be an even integer for RoPE")
        if not math.isfinite(ffn_ratio) or ffn_ratio <= 0:
            raise ValueError("ffn_ratio must be finite and positive")
        canonical_backend(backend)
        chunks = (encoder_chunk, loss_chunk, attention_q_chunk, attention_kv_chunk)
        if any(isinstance(c, bool) or not isinstance(c, Integral) or c < 1 for c in chunks) \
                or encoder_chunk < block_size:
            raise ValueError("encoder_chunk >= block_size and attention/loss chunks > 0 required")
        self.dim, self.heads, self.hd = dim, heads, dim // heads
        self.block_size, self.topk, self.pos_chunk = block_size, topk, pos_chunk
        self.arch, self.backend = arch, backend
        self.checkpoint_chunks, self.loss_chunk = checkpoint_chunks, loss_chunk
        self.attention_q_chunk, self.attention_kv_chunk = attention_q_chunk, attention_kv_chunk
        self.embedding = nn.Embedding(vocab_size, dim)
        nn.init.normal_(self.embedding.weight, std=0.02)
        self.rope = RotaryEmbedding(self.hd)
        shared, local, reads = {}, [], []
        for kind, count, is_shared in parse_arch(arch):
            for _ in range(count):
                if is_shared and kind in shared:
                    module = shared[kind]
                elif kind == "L":
                    module = HaloMemoryBlock(dim, heads, block_size, self.rope, ffn_ratio,
                                             query_chunk_size=max(1, encoder_chunk // block_size),
                                             checkpoint_chunks=checkpoint_chunks, backend=backend)
                else:
                    module = GlobalReadBlock(dim, ffn_ratio)
                if is_shared:
                    shared[kind] = module
                (local if kind == "L" else reads).append(module)
        self.local = nn.ModuleList(local)
        self.reads = nn.ModuleList(reads)
        self.raw_kv = KVProjection(dim, heads, self.rope, use_rope=False, backend=backend)
        self.final_norm = nn.LayerNorm(dim)
        self.lm_head = nn.Linear(dim, vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight

    # -- execution settings --------------------------------------------------

    def set_backend(self, backend: str) -> None:
        """Switch every sub-module between the native kernels and the torch reference."""
        canonical_backend(backend)
        self.backend = backend
        for module in self.modules():
            if hasattr(module, "backend") and module is not self:
                module.backend = backend

    def _native(self, x) -> bool:
        return x.is_cuda and canonical_backend(self.backend) != "torch"

    # -- encoder ---------------------------------------------------------------

    def encode_shard(self, input_ids, parallel, offset):
        """Embedding -> L layers (with CP halos) -> raw K/V in head layout."""
        x = fused.embedding(input_ids, self.embedding, self.backend)
        for layer in self.local:
            halo = parallel.halo(x, self.block_size)
            x = layer(x, previous=halo, start=offset)
        fused_exchange = None
        if parallel.ulysses is not None and self._native(x):
            h = fused.layer_norm(x, self.raw_kv.norm, self.backend)
            fused_exchange = parallel.fused(h, self.heads, self.hd)
        if fused_exchange is not None:
            # K/V projection whose epilogue stores head shards to their owners.
            kv = fused_exchange.project_to_heads(h, self.raw_kv.proj.weight, 2, self.heads, self.hd)
            return x, kv[0], kv[1]
        raw_k, raw_v = self.raw_kv(x, None)
        return x, parallel.to_heads(raw_k), parallel.to_heads(raw_v)

    def encode(self, input_ids):
        """Tokens -> ``(x, raw_k, raw_v)`` for one unsharded sequence."""
        if input_ids.ndim != 2 or min(input_ids.shape) < 1:
            raise ValueError("input_ids must have nonempty shape [batch, sequence]")
        x = self.embedding(input_ids)
        positions = torch.arange(input_ids.shape[1], device=x.device)
        for block in self.local:
            x = block(x, positions)
        raw_k, raw_v = self.raw_kv(x, positions)
        return x, raw_k, raw_v

    # -- dense read round ----------------------------------------------------

    def _query(self, rd, z, link=None):
        return fused.linear(fused.layer_norm(z, rd.q_norm, self.backend, link), rd.wq, self.backend)

    def _finish(self, rd, z, context, link=None):
        z = fused.linear_residual(context, rd.read_out, z, self.backend, link)
        return self._ffn(rd, z)

    def _ffn(self, rd, z):
        link = fused.ResidualLink()       # z feeds ffn_norm and the FFN residual
        return fused.ffn_residual(fused.layer_norm(z, rd.ffn_norm, self.backend, link), z, rd.ffn,
                                  self.backend, link)

    def _dense_round(self, rd, z, k, v, positions, parallel):
        recompute = self.checkpoint_chunks and torch.is_grad_enabled()
        if not recompute and parallel.ulysses is not None and self._native(z):
            link = fused.ResidualLink()   # z feeds q_norm and the read_out residual
            h = fused.layer_norm(z, rd.q_norm, self.backend, link)
            fused_exchange = parallel.fused(h, self.heads, self.hd)
            if fused_exchange is None:
                link.armed = False        # h is dropped: the residual op keeps its gradient
            else:
                # Query projection -> head owners, attention, then the output
                # projection reading the context straight from its owners.
                q = fused_exchange.project_to_heads(h, rd.wq.weight, 1, self.heads, self.hd)[0]
                if k.dtype != q.dtype:
                    k, v = k.to(q.dtype), v.to(q.dtype)
                ctx = dense_attention(q, k, v, positions, self.block_size, self.backend,
                                      q_chunk=self.attention_q_chunk, kv_chunk=self.attention_kv_chunk)
                z = fused_exchange.heads_to_linear_residual(ctx, rd.read_out, z, link)
                return self._ffn(rd, z)
        link = fused.ResidualLink()       # z feeds q_norm and the read_out residual
        if recompute:
            q = checkpoint(self._query, rd, z, link, use_reentrant=False, preserve_rng_state=False)
        else:
            q = self._query(rd, z, link)
        q = parallel.to_heads(q.reshape(*z.shape[:2], self.heads, self.hd))
        if k.dtype != q.dtype:
            k, v = k.to(q.dtype), v.to(q.dtype)
        ctx = dense_attention(q, k, v, positions, self.block_size, self.backend,
                              q_chunk=self.attention_q_chunk, kv_chunk=self.attention_kv_chunk)
        ctx = parallel.to_sequence(ctx).reshape(*z.shape[:2], self.dim)
        if recompute:
            return checkpoint(self._finish, rd, z, ctx, link, use_reentrant=False, preserve_rng_state=False)
        return self._finish(rd, z, ctx, link)

    def _head_loss(self, hidden, labels):
        h = fused.layer_norm(hidden, self.final_norm, self.backend)
        logits = fused.linear(h, self.lm_head, self.backend, out_f32=True)
        return fused.cross_entropy_sum(logits, labels, self.backend)

    def forward_loss(self, input_ids, targets, sup=None, parallel=None, offset=0, static_width=False):
        """Dense training loss: returns sums and counts, never ``[B,N,V]``.

        Inputs are the local sequence shard under context parallelism. Every
        CP rank runs the same collectives, also when it owns no supervised
        token; the caller normalises by the global count
        (reference: st/models/stack.py:215-279).

        ``static_width``: read every position of the shard (unsupervised ones
        get position -1 and no loss) instead of compacting the supervised ones
        first. The work no longer depends on the data and there is no host
        synchronisation, which a captured CUDA graph needs; values are the same.
        """
        parallel = parallel or ParallelContext()
        if input_ids.ndim != 2 or input_ids.shape != targets.shape or min(input_ids.shape) < 1:
            raise ValueError("ids and targets must have identical nonempty [B,N] shape")
        if self.heads % parallel.cp_size:
            raise ValueError("heads must be divisible by context_parallel")
        if sup is None:
            sup = targets != -100
        if sup.shape != targets.shape or sup.dtype != torch.bool:
            raise ValueError("sup must be bool [B,N]")
        sup = sup & (targets != -100)
        parallel.begin_step()
        batch, n = input_ids.shape
        device = input_ids.device
        if static_width:
            width = n
            safe = torch.arange(n, device=device)[None].expand(batch, -1)
            valid = sup
            pos = torch.where(valid, safe + offset, -1)
            picked = targets.masked_fill(~valid, -100)
        else:
            width = parallel.max_query_count(int(sup.sum(1).max()), device)
            # Sort integer positions (supervised first, in order), never features.
            order = torch.arange(n, device=device)[None].expand(batch, -1)
            order = torch.where(sup, order, n).sort(1).values
            if width > n:
                order = F.pad(order, (0, width - n), value=n)
            order = order[:, :width]
            valid = order < n
            safe = order.clamp_max(n - 1)
            pos = torch.where(valid, order + offset, -1)
            picked = targets.gather(1, safe).masked_fill(~valid, -100)
        with trace.phase("encode"):
            x, k, v = self.encode_shard(input_ids, parallel, offset)
        rows = torch.arange(batch, device=device)[:, None]
        native = self._native(x)
        step = self.pos_chunk or (NATIVE_QUERY_TILE if native else self._reference_chunk(n))
        loss_step = max(self.loss_chunk, NATIVE_LOSS_TILE) if native else self.loss_chunk
        losses, hits = [], []
        for lo in range(0, width, step):
            hi = min(lo + step, width)
            if static_width:
                all_rows = lo == 0 and hi == n
            else:
                all_rows = lo == 0 and hi == n and not bool((~valid).any()) if native else False
            z = x if all_rows else x[rows, safe[:, lo:hi]]
            positions = parallel.gather_positions(pos[:, lo:hi])
            for rd in self.reads:
                # Collectives are never inside a checkpoint: every rank must
                # issue the same sequence even when it supervises nothing.
                with trace.phase("read_round"):
                    z = self._dense_round(rd, z, k, v, positions, parallel)
            for j in range(0, hi - lo, loss_step):
                labels = picked[:, lo + j:min(lo + j + loss_step, hi)]
                hidden = z[:, j:j + loss_step]
                if self.checkpoint_chunks and torch.is_grad_enabled():
                    loss, hit = checkpoint(self._head_loss, hidden, labels, use_reentrant=False,
                                           preserve_rng_state=False)
                else:
                    loss, hit = self._head_loss(hidden, labels)
                losses.append(loss)
                hits.append(hit.detach())
        hit = torch.cat(hits, 1)
        loss_sum = losses[0] if len(losses) == 1 else torch.stack(losses).sum()
        return {"loss_sum": loss_sum, "count": valid.sum(), "correct": (hit & valid).sum(),
                "row_errors": ((~hit) & valid).sum(1), "positions": pos, "hits": hit}

    # -- inference helpers ---------------------------------------------------

    @staticmethod
    def supervised_positions(sup, n):
        """``[B,S]`` supervised positions (equal count per row); ``sup=None`` -> all."""
        if sup is None:
            return None, n
        counts = sup.sum(1)
        s = int(counts[0])
        if s < 1 or not bool((counts == s).all()):
            raise ValueError("sup must mark the same positive count per row")
        return sup.nonzero()[:, 1].reshape(sup.shape[0], s), s

    # -- whole-sequence forward (inference, validation and the sparse reference) --

    def _reference_chunk(self, n: int) -> int:
        """Queries per chunk of the materialising top-k read ([chunk, heads, n] logits near 2^27 elements)."""
        if self.pos_chunk > 0:
            return self.pos_chunk
        return max(16, min(4096, (1 << 27) // max(1, 3 * self.heads * n)))

    def _read(self, rd, z, raw_k, raw_v, positions, blocks):
        """One G round for the states ``z`` of ``positions`` over an unsharded sequence.

        With ``topk`` at least the number of blocks every block is read: the
        dense gated operator (native kernels on CUDA). Otherwise the top-k rule
        applies: without autograd through the paged sparse operator, with
        autograd through the materialising reference (its gate is
        differentiable, unselected blocks included).
        """
        if self.topk >= blocks:
            return self._dense_round(rd, z, raw_k, raw_v, positions, ParallelContext())
        q = self._query(rd, z).view(*z.shape[:2], self.heads, self.hd)
        if torch.is_grad_enabled():
            ctx = eager_gated(q, raw_k, raw_v, positions, self.block_size, topk=self.topk)
        else:
            pages = TensorPages(raw_k, raw_v, page_tokens=max(self.block_size, 65536 // self.block_size * self.block_size))
            ctx = sparse_attention(q, pages, positions, self.block_size, self.topk, self.backend)
        return self._finish(rd, z, ctx.reshape(*z.shape[:2], self.dim))

    def _positions(self, sup, batch, n, device):
        pos, count = self.supervised_positions(sup, n)
        if pos is None:
            pos = torch.arange(n, device=device)[None].expand(batch, n)
        return pos.to(device), count

    @staticmethod
    def _rows(x, positions):
        return torch.gather(x, 1, positions[..., None].expand(-1, -1, x.shape[-1]))

    def forward(self, input_ids, sup=None, *, targets=None, parallel=None, offset=0, compact=False):
        """Logits ``[B, N, V]`` (zero off ``sup``), or ``[B, S, V]`` at the supervised positions
        with ``compact``; with ``targets`` the training loss sums of :meth:`forward_loss`."""
        if targets is not None:
            return self.forward_loss(input_ids, targets, sup, parallel, offset)
        batch, n = input_ids.shape if input_ids.ndim == 2 else (0, 0)
        with trace.phase("encode"):
            x, raw_k, raw_v = self.encode(input_ids)
        pos, count = self._positions(sup, batch, n, x.device)
        blocks = -(-n // self.block_size)
        step = self._reference_chunk(n)
        states = []
        with trace.phase("read_rounds"):
            for lo in range(0, count, step):
                part = pos[:, lo:lo + step]
                z = self._rows(x, part)
                for rd in self.reads:
                    z = self._read(rd, z, raw_k, raw_v, part, blocks)
                states.append(z)
        z = states[0] if len(states) == 1 else torch.cat(states, 1)
        picked = fused.linear(fused.layer_norm(z, self.final_norm, self.backend), self.lm_head, self.backend)
        if compact:
            return picked
        logits = picked.new_zeros(batch, n, picked.shape[-1])
        return logits.scatter(1, pos[..., None].expand(-1, -1, picked.shape[-1]), picked)

    @torch.no_grad()
    def diagnose(self, idx, sup=None, needle_pos=None):
        """How well the first G round's top-k captures its gate, from block scores alone.

        * ``sel_cov``: softmax mass (over remote block scores) of the kept blocks;
        * ``gate_margin``: weakest kept minus strongest dropped remote block score;
        * ``needle_block_hit`` (passkey, ``needle_pos [B]``): at each row's first
          supervised position, the fraction of heads that keep a block of the
          needle, over rows whose needle lies before the local window.
        """
        if not self.reads:
            return {}
        self.eval()
        batch, n = idx.shape
        b = self.block_size
        x, raw_k, _ = self.encode(idx)
        pos, count = self._positions(sup, batch, n, x.device)
        rd = self.reads[0]
        sums = torch.zeros(6, dtype=torch.float64, device=x.device)   # coverage, margin, needle: (sum, count)
        step = self._reference_chunk(n)
        for lo in range(0, count, step):
            part = pos[:, lo:lo + step]
            q = self._query(rd, self._rows(x, part)).view(batch, part.shape[1], self.heads, self.hd)
            scores = block_log_mass(q, raw_k, part, b)                # [B,c,H,G]
            remote = torch.isfinite(scores)
            top, chosen = scores.topk(min(self.topk, scores.shape[-1]), -1)
            kept = torch.zeros_like(remote).scatter(-1, chosen, torch.isfinite(top))
            dropped = remote & ~kept
            any_remote = remote.any(-1)
            share = torch.where(kept, scores.softmax(-1), torch.zeros_like(scores)).sum(-1)
            sums[0] += share[any_remote].sum()
            sums[1] += any_remote.sum()
            both = kept.any(-1) & dropped.any(-1)
            gap = scores.masked_fill(~kept, math.inf).amin(-1) - scores.masked_fill(~dropped, -math.inf).amax(-1)
            sums[2] += gap[both].sum()
            sums[3] += both.sum()
            if needle_pos is not None and lo == 0:
                width = KEY + 1                                        # the needle: marker and key digits
                needle_blocks = (needle_pos.to(x.device)[:, None] + torch.arange(width, device=x.device)) // b
                before_window = needle_blocks.amax(-1) <= part[:, 0] // b - 2
                hit = kept[:, 0].gather(-1, needle_blocks[:, None, :].expand(-1, self.heads, -1)).any(-1)
                sums[4] += hit.double().mean(-1)[before_window].sum()
                sums[5] += before_window.sum()
        totals = sums.tolist()
        report = {}
        for name, (total, n_items) in zip(("sel_cov", "gate_margin", "needle_block_hit"),
                                          zip(totals[0::2], totals[1::2])):
            if n_items:
                report[name] = round(total / n_items, 4)
        return report
