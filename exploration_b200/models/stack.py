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
import time
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
from .blocks import FeedForward, HaloMemoryBlock, KVProjection, RotaryEmbedding, _gather_heads

# On the native path one query tile covers this many supervised positions:
# the gated-attention kernel never materialises Q x N, so the only memory the
# tile bounds is a few [tile, dim] activations.
NATIVE_QUERY_TILE = 65536
NATIVE_LOSS_TILE = 65536


def parse_arch(arch):
    """``'Lx2,(G)x4'`` -> ``[(kind, count, shared), ...]`` in application order."""
    if not isinstance(arch, str) or not arch.strip():
        raise ValueError("arch must be a nonempty spec like 'Lx2,G'")
    spec = []
    for raw in arch.split(","):
        item = raw.strip()
        shared = item.startswith("(")
        if shared:
            kind, sep, count = item[1:].partition(")x")
            if not sep:
                raise ValueError(f"shared layers must look like '(X)xN': {item!r}")
        else:
            kind, _, count = item.partition("x")
            count = count or "1"
        if kind not in ("L", "G"):
            raise ValueError(f"unknown layer kind in arch item {item!r} (want L or G)")
        if not count.isdigit() or int(count) < 1:
            raise ValueError(f"repeat count must be a positive integer in {item!r}")
        spec.append((kind, int(count), shared))
    kinds = [k for k, _, _ in spec]
    if "G" in kinds and "L" in kinds:
        last_l = len(kinds) - 1 - kinds[::-1].index("L")
        if kinds.index("G") < last_l:
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
        x = self.embedding(input_ids)
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
        step = self.pos_chunk or (NATIVE_QUERY_TILE if native else self._chunk_size(n))
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

    def push_scores(self, q, kb, visible):
        """Exact block partition functions ``[B,c,H,G]`` (invisible blocks: -inf).

        ``q [B,c,H,D]``, ``kb [B,G,b,H,D]``, ``visible [B,c,G]``.
        """
        logits = torch.einsum("bchd,bgwhd->bchgw", q, kb) / math.sqrt(self.hd)
        return logits.logsumexp(-1).masked_fill(~visible[:, :, None, :], float("-inf"))

    def _chunk_size(self, n):
        """Queries per chunk bounding the sparse-reference temporaries (~2^29-2^31 elements)."""
        if self.pos_chunk > 0:
            return self.pos_chunk
        groups = -(-n // self.block_size)
        m = min(self.topk, groups)
        per_query = self.heads * (n + 2 * m * self.block_size * self.hd)
        small = self.dim <= 512
        cap, budget = (2048, 1 << 31) if small else (512, 1 << 29)
        return min(cap, max(16, budget // max(per_query, 1)))

    def _read_round_sparse(self, rd, z, sl, env):
        """Differentiable top-k read round (mathematical reference, any grad mode)."""
        batch, count, _ = z.shape
        n, b, groups = env["n"], env["b"], env["groups"]
        pos = env["pos"][:, sl]
        window = env["src"][:, sl]                                   # [B,c,2b]
        rows3 = env["rows3"]
        k_local = env["raw_k"][rows3, window.clamp(0, n - 1)]        # [B,c,2b,H,D]
        v_local = env["raw_v"][rows3, window.clamp(0, n - 1)]
        q = rd.wq(rd.q_norm(z)).reshape(batch, count, self.heads, self.hd)
        s = self.push_scores(q, env["kb"], env["visible"][:, sl])    # [B,c,H,G]
        with torch.no_grad():
            top, sel = s.topk(min(self.topk, groups), dim=-1)
            sel_ok = torch.isfinite(top)
        gate = torch.nan_to_num(s - s.logsumexp(-1, keepdim=True), nan=0.0, neginf=0.0)
        gate_sel = torch.where(sel_ok, gate.gather(3, sel), torch.zeros((), dtype=gate.dtype,
                                                                       device=gate.device))
        tokens = (sel[..., None] * b + torch.arange(b, device=z.device)).reshape(
            batch, count, self.heads, -1)                            # [B,c,H,m*b]
        tok_ok = (sel_ok[..., None].expand(-1, -1, -1, -1, b).reshape(batch, count, self.heads, -1)
                  & (tokens < n) & (tokens <= pos[:, :, None, None]))
        idx = tokens.clamp(0, n - 1).permute(0, 2, 1, 3)
        k_remote = _gather_heads(env["raw_k"].transpose(1, 2), idx).permute(0, 2, 1, 3, 4)
        v_remote = _gather_heads(env["raw_v"].transpose(1, 2), idx).permute(0, 2, 1, 3, 4)
        bias = gate_sel[..., None].expand(-1, -1, -1, -1, b).reshape(batch, count, self.heads, -1)
        s_local = torch.einsum("bchd,bcwhd->bchw", q, k_local) / math.sqrt(self.hd)
        s_remote = torch.einsum("bchd,bchkd->bchk", q, k_remote) / math.sqrt(self.hd) + bias
        mask = torch.cat([env["src_valid"][:, sl, None].expand(-1, -1, self.heads, -1), tok_ok], -1)
        probs = torch.cat([s_local, s_remote], -1).masked_fill(~mask, float("-inf")).softmax(-1)
        width = s_local.shape[-1]
        ctx = (torch.einsum("bchw,bcwhd->bchd", probs[..., :width], v_local)
               + torch.einsum("bchk,bchkd->bchd", probs[..., width:], v_remote))
        z = z + rd.read_out(ctx.reshape(batch, count, self.dim))
        return z + rd.ffn(rd.ffn_norm(z))

    def _prof_tick(self, device):
        """Phase timer (enable with ``model._prof = True``); synchronises the device."""
        if not getattr(self, "_prof", False):
            return None
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        return time.perf_counter()

    def forward(self, input_ids, sup=None, *, targets=None, parallel=None, offset=0, compact=False):
        if targets is not None:
            return self.forward_loss(input_ids, targets, sup, parallel, offset)
        if input_ids.ndim != 2 or min(input_ids.shape) < 1:
            raise ValueError("input_ids must have nonempty shape [batch, sequence]")
        batch, n = input_ids.shape
        b = self.block_size
        groups = -(-n // b)
        t0 = self._prof_tick(input_ids.device)
        x, raw_k, raw_v = self.encode(input_ids)
        t1 = self._prof_tick(input_ids.device)
        pos, s_n = self.supervised_positions(sup, n)
        if pos is None:
            pos = torch.arange(n, device=x.device)[None].expand(batch, n)
        dense = self.topk >= groups
        sparse_grad = not dense and torch.is_grad_enabled()
        env = None
        if sparse_grad:
            kb = F.pad(raw_k, (0, 0, 0, 0, 0, groups * b - n)).reshape(batch, groups, b, self.heads,
                                                                       self.hd)
            block_end = (torch.arange(groups, device=x.device) + 1) * b
            env = dict(n=n, b=b, groups=groups, kb=kb, raw_k=raw_k, raw_v=raw_v,
                       rows3=torch.arange(batch, device=x.device)[:, None, None])
        rows = torch.arange(batch, device=x.device)[:, None]
        window = torch.arange(2 * b, device=x.device)
        outs = []
        chunk = self._chunk_size(n)
        for start in range(0, s_n, chunk):
            sl = slice(start, min(s_n, start + chunk))
            pc = pos[:, sl]
            z = x[rows, pc]
            if sparse_grad:
                block_of = torch.div(pc, b, rounding_mode="floor")
                first_valid = ((block_of - 1) * b).clamp_min(0)
                src = pc[:, :, None] - (2 * b - 1) + window
                env.update(pos=pc, src=src,
                           src_valid=(src >= first_valid[:, :, None]) & (src >= 0),
                           visible=block_end[None, None, :] <= ((block_of - 1) * b)[:, :, None])
            for rd in self.reads:
                if dense:
                    z = self._dense_round(rd, z, raw_k, raw_v, pc, ParallelContext())
                elif not torch.is_grad_enabled():
                    from ..ops.sparse import TensorPages, sparse_attention
                    q = self._query(rd, z).reshape(batch, z.shape[1], self.heads, self.hd)
                    pages = TensorPages(raw_k, raw_v, page_tokens=max(b, 65536 // b * b))
                    ctx = sparse_attention(q, pages, pc, b, min(self.topk, groups), self.backend)
                    z = self._finish(rd, z, ctx.reshape(batch, z.shape[1], self.dim))
                else:
                    z = self._read_round_sparse(rd, z, slice(None), env)
            outs.append(z)
        t2 = self._prof_tick(input_ids.device)
        z = outs[0] if len(outs) == 1 else torch.cat(outs, dim=1)
        sup_logits = fused.linear(fused.layer_norm(z, self.final_norm, self.backend), self.lm_head,
                                  self.backend)
        if compact:
            return sup_logits
        logits = sup_logits.new_zeros(batch, n, sup_logits.shape[-1])
        logits[rows, pos] = sup_logits
        t3 = self._prof_tick(input_ids.device)
        if t0 is not None:
            self._prof_stats = {"enc_s": round(t1 - t0, 3), "read_s": round(t2 - t1, 3),
                                "head_s": round(t3 - t2, 3)}
        return logits

    @torch.no_grad()
    def diagnose(self, idx, sup=None, needle_pos=None):
        """Selection quality of the first G round (push only, no pop).

        ``sel_cov``: attention mass covered by the selected blocks;
        ``gate_margin``: lowest selected minus highest unselected visible score;
        ``needle_block_hit`` (passkey): fraction of heads whose top-k holds a
        needle block at the first supervised position, over rows whose needle
        lies outside the local window (reference: st/models/stack.py:463-534).
        """
        if not self.reads:
            return {}
        self.eval()
        batch, n = idx.shape
        b = self.block_size
        groups = -(-n // b)
        x, raw_k, _ = self.encode(idx)
        pos, s_n = self.supervised_positions(sup, n)
        if pos is None:
            pos = torch.arange(n, device=x.device)[None].expand(batch, n)
        block_of = torch.div(pos, b, rounding_mode="floor")
        kb = F.pad(raw_k, (0, 0, 0, 0, 0, groups * b - n)).reshape(batch, groups, b, self.heads,
                                                                   self.hd)
        block_end = (torch.arange(groups, device=x.device) + 1) * b
        rd = self.reads[0]
        rows = torch.arange(batch, device=x.device)[:, None]
        keep = min(self.topk, groups)
        cov = [0.0, 0.0]
        margin = [0.0, 0.0]
        needle = [0.0, 0.0]
        step = self._chunk_size(n)
        for start in range(0, s_n, step):
            stop = min(s_n, start + step)
            count = stop - start
            visible = block_end[None, None, :] <= ((block_of[:, start:stop] - 1) * b)[:, :, None]
            z = x[rows, pos[:, start:stop]]
            q = rd.wq(rd.q_norm(z)).reshape(batch, count, self.heads, self.hd)
            s = self.push_scores(q, kb, visible)
            top, sel = s.topk(keep, dim=-1)
            sel_ok = torch.isfinite(top)
            p = s.softmax(-1)
            p_sel = torch.where(sel_ok, p.gather(3, sel), torch.zeros((), dtype=p.dtype,
                                                                      device=p.device))
            coverage = p_sel.sum(-1)
            has_visible = visible.any(-1, keepdim=True).expand_as(coverage)
            cov[0] += coverage[has_visible].sum().item()
            cov[1] += has_visible.sum().item()
            chosen = torch.zeros_like(s, dtype=torch.bool).scatter(3, sel, sel_ok)
            unchosen = visible[:, :, None, :] & ~chosen
            lowest = s.masked_fill(~chosen, float("inf")).min(-1).values
            highest = s.masked_fill(~unchosen, float("-inf")).max(-1).values
            both = chosen.any(-1) & unchosen.any(-1)
            margin[0] += (lowest - highest)[both].sum().item()
            margin[1] += both.sum().item()
            if needle_pos is not None and start == 0:
                needle_blocks = torch.div(needle_pos.to(x.device)[:, None]
                                          + torch.arange(6, device=x.device), b,
                                          rounding_mode="floor")
                first_block = int(pos[0, 0]) // b
                outside = needle_blocks.max(-1).values <= first_block - 2
                if outside.any():
                    at_first = chosen[:, 0]
                    hit = at_first.gather(2, needle_blocks[:, None, :].expand(-1, self.heads, -1)).any(-1)
                    needle[0] += hit[outside].float().mean(-1).sum().item()
                    needle[1] += int(outside.sum().item())
        out = {}
        if cov[1]:
            out["sel_cov"] = round(cov[0] / cov[1], 4)
        if margin[1]:
            out["gate_margin"] = round(margin[0] / margin[1], 4)
        if needle[1]:
            out["needle_block_hit"] = round(needle[0] / needle[1], 4)
        return out
