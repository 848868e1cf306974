"""Bounded-memory torch reference of exact block-gated dense attention.

Definition (reference: docs/ARCHITECTURE.md:20-26, st/ops/attention.py:1-6).
For a query at position ``p`` in block ``P = p // b`` and key ``i`` with
logit ``a_i = q . k_i / sqrt(D)``:

* block ``j`` has mass ``M_j = sum_{i in j} exp(a_i)`` and score ``s_j = log M_j``;
* keys in blocks ``>= P - 1`` and ``<= p`` are *local* and keep logit ``a_i``;
* blocks ``j < P - 1`` are *remote*; ``Z_R = sum_remote M_j``; a remote key's
  logit is ``a_i + s_j - log Z_R``;
* one softmax runs over the local and remote keys together.

The forward streams key tiles with two online-softmax accumulators (local,
and remote on ``a_i + s_j``) plus a running ``log Z_R``; ``-log Z_R`` is a
per-row constant, so it is applied once at the end. The backward recomputes
each tile and carries the exact derivative through ``log M_j`` (a segmented
block sum) and through ``log Z_R`` (one per-row scalar ``rho``). No
``Q x N`` tensor is kept. This module is the CPU path, the numerical oracle
for the sm_100a kernels and the timed CPU baseline.
"""
from __future__ import annotations

import math

import torch

NEG_INF = float("-inf")


def work_dtype(t: torch.Tensor) -> torch.dtype:
    return torch.float64 if t.dtype == torch.float64 else torch.float32


def _finite_or_zero(x: torch.Tensor) -> torch.Tensor:
    return torch.where(torch.isfinite(x), x, torch.zeros_like(x))


class _OnlineSoftmax:
    """Running (max, denominator, numerator) of a softmax-weighted value sum."""

    def __init__(self, shape, dim, dtype, device):
        self.m = torch.full(shape, NEG_INF, dtype=dtype, device=device)
        self.den = torch.zeros(shape, dtype=dtype, device=device)
        self.num = torch.zeros((*shape, dim), dtype=dtype, device=device)

    def absorb(self, logits: torch.Tensor, values: torch.Tensor):
        new_m = torch.maximum(self.m, logits.amax(-1))
        ref = _finite_or_zero(new_m)
        keep = torch.exp(self.m - ref)
        weights = torch.exp(logits - ref[..., None])
        self.den = self.den * keep + weights.sum(-1)
        self.num = self.num * keep[..., None] + weights @ values
        self.m = new_m

    def log_mass(self) -> torch.Tensor:
        return self.m + self.den.log()

    def mean(self) -> torch.Tensor:
        tiny = torch.finfo(self.den.dtype).tiny
        return self.num / self.den.clamp_min(tiny)[..., None]


def _key_tile(k, v, lo, hi, b, dtype):
    """Keys/values ``[lo, hi)`` as ``[B, H, T, D]`` padded to a whole block."""
    kt = k[:, lo:hi].transpose(1, 2).to(dtype)
    vt = v[:, lo:hi].transpose(1, 2).to(dtype)
    pad = (-(hi - lo)) % b
    if pad:
        kt = torch.nn.functional.pad(kt, (0, 0, 0, pad))
        vt = torch.nn.functional.pad(vt, (0, 0, 0, pad))
    return kt, vt


def _tile_logits(qt, kt, pos, lo, hi, b):
    """Scaled logits, per-key block score and the remote/local masks of one tile.

    ``qt`` [B,H,Q,D], ``kt`` [B,H,T,D] (T a multiple of b), ``pos`` [B,Q].
    Keys at or beyond ``hi`` (tile padding) get ``-inf`` logits, so they are
    never remote and never local.
    """
    scale = 1.0 / math.sqrt(qt.shape[-1])
    a = (qt @ kt.transpose(-1, -2)) * scale
    span = kt.shape[-2]
    key = torch.arange(lo, lo + span, device=qt.device)
    a = a.masked_fill((key >= hi)[None, None, None, :], NEG_INF)
    block_score = a.unflatten(-1, (span // b, b)).logsumexp(-1).repeat_interleave(b, -1)
    p = pos[:, None, :, None]
    live = p >= 0
    key_block = (key // b)[None, None, None, :]
    query_block = torch.div(p, b, rounding_mode="floor")
    remote = live & (key_block < query_block - 1)
    local = live & (key_block >= query_block - 1) & (key[None, None, None, :] <= p) \
        & (key < hi)[None, None, None, :]
    return a, block_score, remote, local


def gated_forward(q, k, v, positions, block_size, q_chunk=128, kv_chunk=4096):
    """Return ``(out, remote_context, remote_prob, log_zr, lse)``.

    ``out`` has q's dtype; the statistics are in the working dtype:
    ``remote_context`` is the remote part of ``out`` (already weighted by the
    remote probability mass ``remote_prob``), ``log_zr`` is ``log Z_R`` and
    ``lse`` the log normaliser of the joint softmax. Empty sets give ``-inf``.
    """
    b = block_size
    dtype = work_dtype(q)
    batch, queries, heads, dim = q.shape
    nk = k.shape[1]
    kv_chunk = max(b, kv_chunk // b * b)
    out = torch.empty_like(q)
    remote_ctx = torch.empty(q.shape, dtype=dtype, device=q.device)
    remote_prob = torch.empty(q.shape[:3], dtype=dtype, device=q.device)
    log_zr = torch.empty_like(remote_prob)
    lse = torch.empty_like(remote_prob)
    resident = _key_tile(k, v, 0, nk, b, dtype) if nk <= kv_chunk else None
    for q0 in range(0, queries, q_chunk):
        q1 = min(q0 + q_chunk, queries)
        qt = q[:, q0:q1].transpose(1, 2).to(dtype)
        pos = positions[:, q0:q1]
        rows = qt.shape[:-1]
        local = _OnlineSoftmax(rows, dim, dtype, q.device)
        remote = _OnlineSoftmax(rows, dim, dtype, q.device)
        zr = torch.full(rows, NEG_INF, dtype=dtype, device=q.device)
        for lo in range(0, nk, kv_chunk):
            hi = min(lo + kv_chunk, nk)
            kt, vt = resident if resident is not None else _key_tile(k, v, lo, hi, b, dtype)
            a, sb, is_remote, is_local = _tile_logits(qt, kt, pos, lo, hi, b)
            zr = torch.logaddexp(zr, a.masked_fill(~is_remote, NEG_INF).logsumexp(-1))
            remote.absorb((a + sb).masked_fill(~is_remote, NEG_INF), vt)
            local.absorb(a.masked_fill(~is_local, NEG_INF), vt)
        log_remote = remote.log_mass() - _finite_or_zero(zr)
        log_local = local.log_mass()
        total = torch.logaddexp(log_remote, log_local)
        ref = _finite_or_zero(total)
        p_remote = torch.exp(log_remote - ref)
        rc = remote.mean() * p_remote[..., None]
        lc = local.mean() * torch.exp(log_local - ref)[..., None]
        out[:, q0:q1] = (lc + rc).transpose(1, 2).to(q.dtype)
        remote_ctx[:, q0:q1] = rc.transpose(1, 2)
        remote_prob[:, q0:q1] = p_remote.transpose(1, 2)
        log_zr[:, q0:q1] = zr.transpose(1, 2)
        lse[:, q0:q1] = total.transpose(1, 2)
    return out, remote_ctx, remote_prob, log_zr, lse


def gated_backward(grad, q, k, v, positions, out, remote_ctx, remote_prob, log_zr, lse,
                   block_size, q_chunk=128, kv_chunk=4096):
    """Exact first derivatives ``(dq, dk, dv)`` of :func:`gated_forward`."""
    b = block_size
    dtype = work_dtype(q)
    scale = 1.0 / math.sqrt(q.shape[-1])
    nk = k.shape[1]
    kv_chunk = max(b, kv_chunk // b * b)
    dq = torch.zeros(q.shape, dtype=dtype, device=q.device)
    dk = torch.zeros(k.shape, dtype=dtype, device=q.device)
    dv = torch.zeros(v.shape, dtype=dtype, device=q.device)
    resident = _key_tile(k, v, 0, nk, b, dtype) if nk <= kv_chunk else None
    for q0 in range(0, q.shape[1], q_chunk):
        q1 = min(q0 + q_chunk, q.shape[1])
        qt = q[:, q0:q1].transpose(1, 2).to(dtype)
        gt = grad[:, q0:q1].transpose(1, 2).to(dtype)
        ot = out[:, q0:q1].transpose(1, 2).to(dtype)
        pos = positions[:, q0:q1]
        delta = (gt * ot).sum(-1)
        rho = (gt * remote_ctx[:, q0:q1].transpose(1, 2)).sum(-1) \
            - delta * remote_prob[:, q0:q1].transpose(1, 2)
        zr = _finite_or_zero(log_zr[:, q0:q1].transpose(1, 2))
        total = _finite_or_zero(lse[:, q0:q1].transpose(1, 2))
        for lo in range(0, nk, kv_chunk):
            hi = min(lo + kv_chunk, nk)
            kt, vt = resident if resident is not None else _key_tile(k, v, lo, hi, b, dtype)
            a, sb, is_remote, is_local = _tile_logits(qt, kt, pos, lo, hi, b)
            logit = torch.where(is_remote, a + sb - zr[..., None], a)
            prob = torch.where(is_remote | is_local, torch.exp(logit - total[..., None]),
                               torch.zeros_like(a))
            direct = prob * (gt @ vt.transpose(-1, -2) - delta[..., None])
            span = kt.shape[-2]
            block_sum = direct.unflatten(-1, (span // b, b)).sum(-1).repeat_interleave(b, -1)
            # d log M_j / d a_i = exp(a_i - s_j); d log Z_R / d a_i = exp(a_i - log Z_R).
            gate = torch.exp(a - sb) * block_sum - torch.exp(a - zr[..., None]) * rho[..., None]
            da = (direct + torch.where(is_remote, gate, torch.zeros_like(gate))) * scale
            width = hi - lo
            dq[:, q0:q1] += (da @ kt).transpose(1, 2)
            dk[:, lo:hi] += (da.transpose(-1, -2) @ qt).transpose(1, 2)[:, :width]
            dv[:, lo:hi] += (prob.transpose(-1, -2) @ gt).transpose(1, 2)[:, :width]
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def _logits(q, k):
    """``a = q . k / sqrt(D)`` as ``[B, H, Q, N]`` in the work dtype."""
    dtype = work_dtype(q)
    return (q.transpose(1, 2).to(dtype) @ k.transpose(1, 2).to(dtype).transpose(-1, -2)) / math.sqrt(q.shape[-1])


def _visible_block_scores(a, positions, b):
    """Block scores ``s_j = logsumexp_{i in j} a_i`` ``[B, H, Q, G]``, ``-inf`` off the remote blocks
    (blocks ``j < P - 1`` of a query in block ``P``), and the visibility mask."""
    n = a.shape[-1]
    s = torch.nn.functional.pad(a, (0, (-n) % b), value=NEG_INF).unflatten(-1, (-1, b)).logsumexp(-1)
    blocks = torch.arange(s.shape[-1], device=a.device)
    visible = blocks < torch.div(positions[:, None, :, None], b, rounding_mode="floor") - 1
    return s.masked_fill(~visible, NEG_INF), visible


def block_log_mass(q, k, positions, block_size):
    """Remote block scores ``[B, Q, H, G]`` of queries ``q [B, Q, H, D]`` at ``positions [B, Q]``
    over keys ``k [B, N, H, D]`` (``-inf`` for blocks that are not remote to the query)."""
    s, _ = _visible_block_scores(_logits(q, k), positions, block_size)
    return s.transpose(1, 2)


def eager_gated(q, k, v, positions, block_size, topk=None):
    """Materialising ``Q x N`` form of the operator (small checks and the differentiable top-k read).

    With ``topk``, a query reads remote keys only from its ``topk`` highest
    scoring remote blocks per head (the inference rule); the gate still
    normalises over every remote block, so unselected blocks receive gradient
    through ``log Z_R``. ``topk=None`` (or at least the number of blocks) is
    the dense training operator.
    """
    b = block_size
    n = k.shape[1]
    a = _logits(q, k)                                                  # [B,H,Q,N]
    s, visible = _visible_block_scores(a, positions, b)
    any_remote = visible.any(-1, keepdim=True)
    safe = torch.where(any_remote, s, torch.zeros_like(s))
    gate = (safe - safe.logsumexp(-1, keepdim=True)).masked_fill(~visible, 0.0)
    read = visible
    if topk is not None and topk < s.shape[-1]:
        with torch.no_grad():
            top, chosen = s.topk(topk, -1)
            read = torch.zeros_like(s, dtype=torch.bool).scatter(-1, chosen, torch.isfinite(top))
    key_block = torch.arange(n, device=q.device) // b
    pos = positions[:, None, :, None]
    local = key_block >= torch.div(pos, b, rounding_mode="floor") - 1
    allowed = (torch.arange(n, device=q.device) <= pos) & (local | read[..., key_block])
    bias = gate[..., key_block]
    probs = torch.nan_to_num((a + bias).masked_fill(~allowed, NEG_INF).softmax(-1), nan=0.0)
    return (probs @ v.transpose(1, 2).to(a.dtype)).transpose(1, 2).to(q.dtype)
