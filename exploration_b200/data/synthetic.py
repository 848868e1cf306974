"""Synthetic retrieval tasks: passkey, copying and MQAR.

Every generator returns ``(input_ids, targets, mask, extra)`` on CPU (or the
requested device): ``input_ids``/``targets`` are the next-token pair of a
sampled length ``n + 1`` sequence, ``mask`` marks supervised target columns
and ``extra`` is the passkey needle position (``None`` for other tasks).

Token alphabet (a contract shared with the reference, st/data/synthetic.py:29-34):
digits 0-9, filler 18-29 (MQAR filler 26-29), 30 = P, 31 = Q, 32 = SEP,
MQAR keys 34-97. The draws below are made from the caller's
``torch.Generator`` in the same order as the reference generators
(st/data/synthetic.py:44-113), so one seed yields the same batch in both
frameworks; tests pin this by value.
"""
from __future__ import annotations

import torch

FILL0, FILL1 = 18, 30
P, Q, SEP = 30, 31, 32
VOCAB = 128
KEY = 5
MQAR_KEYS = list(range(34, 98))
MQAR_FILL0, MQAR_FILL1 = 26, 30


def _shift(seq: torch.Tensor, supervised_tail: int):
    """Split an ``[B, n+1]`` sequence into inputs/targets with a tail mask."""
    inputs, targets = seq[:, :-1], seq[:, 1:]
    mask = torch.zeros(inputs.shape, dtype=torch.bool)
    mask[:, -supervised_tail:] = True
    return inputs, targets, mask


def _place(device, *tensors):
    return tuple(t.to(device) if t is not None else None for t in tensors)


def passkey_batch(bs: int, n: int, g: torch.Generator, device):
    """Filler with a ``[P, d1..d5]`` needle and ``[P, Q, d1..d5]`` at the end."""
    seq = torch.randint(FILL0, FILL1, (bs, n + 1), generator=g)
    digits = torch.randint(0, 10, (bs, KEY), generator=g)
    tail = KEY + 2
    last_start = n + 1 - tail - (KEY + 1)
    needle = torch.randint(0, last_start + 1, (bs,), generator=g)
    rows = torch.arange(bs)
    seq[rows, needle] = P
    seq[rows[:, None], needle[:, None] + torch.arange(1, KEY + 1)] = digits
    seq[:, -tail] = P
    seq[:, -tail + 1] = Q
    seq[:, -KEY:] = digits
    inputs, targets, mask = _shift(seq, KEY)
    return _place(device, inputs, targets, mask, needle)


def copying_batch(bs: int, n: int, g: torch.Generator, device, c: int | None = None):
    """``[pattern][SEP][filler][SEP][pattern]``; the final copy is supervised."""
    c = c or n // 8
    assert 2 * c + 2 <= n + 1, "sequence too short for the copy pattern"
    seq = torch.randint(FILL0, FILL1, (bs, n + 1), generator=g)
    pattern = torch.randint(FILL0, FILL1, (bs, c), generator=g)
    seq[:, :c] = pattern
    seq[:, c] = SEP
    seq[:, -c - 1] = SEP
    seq[:, -c:] = pattern
    inputs, targets, mask = _shift(seq, c)
    return _place(device, inputs, targets, mask, None)


def resolve_npairs(n: int, n_pairs: int, density: float) -> int:
    """A fixed pair count, or ``round(n * density)`` (at least 1) when density > 0."""
    if density and density > 0:
        return max(1, round(n * density))
    return n_pairs


def mqar_batch(bs: int, n: int, g: torch.Generator, device, n_pairs: int = 16,
               n_queries: int = 4, key_tokens: int = 1):
    """Multi-query associative recall.

    ``n_pairs`` key/value pairs are spread one per segment through MQAR
    filler; the tail holds ``n_queries`` records ``[Q, key..., value]`` and the
    value of each record is supervised. Keys are distinct within a sequence
    (a per-row permutation of the key alphabet, or of its ``key_tokens``-fold
    product) and values are digits.
    """
    alphabet = len(MQAR_KEYS)
    n_keys = alphabet ** key_tokens
    assert n_pairs <= n_keys, f"n_pairs={n_pairs} > {n_keys} distinct keys"
    record = key_tokens + 2
    tail = record * n_queries
    seq = torch.randint(MQAR_FILL0, MQAR_FILL1, (bs, n + 1), generator=g)
    segment = (n + 1 - tail) // n_pairs
    assert segment >= key_tokens + 1, "sequence too short for n_pairs"
    key_ids = torch.argsort(torch.rand(bs, n_keys, generator=g), dim=1)[:, :n_pairs]
    digits = [MQAR_KEYS[0] + key_ids // (alphabet ** (key_tokens - 1 - j)) % alphabet
              for j in range(key_tokens)]
    keys = torch.stack(digits, -1)                       # [bs, pairs, key_tokens]
    values = torch.randint(0, 10, (bs, n_pairs), generator=g)
    jitter = torch.randint(0, segment - key_tokens, (bs, n_pairs), generator=g)
    where = torch.arange(n_pairs)[None] * segment + jitter
    rows = torch.arange(bs)[:, None]
    for j in range(key_tokens):
        seq[rows, where + j] = keys[..., j]
    seq[rows, where + key_tokens] = values
    asked = torch.randint(0, n_pairs, (bs, n_queries), generator=g)
    start = n + 1 - tail
    seq[:, start::record] = Q
    for j in range(key_tokens):
        seq[:, start + 1 + j::record] = keys[..., j].gather(1, asked)
    seq[:, start + 1 + key_tokens::record] = values.gather(1, asked)
    inputs, targets = seq[:, :-1], seq[:, 1:]
    mask = torch.zeros(bs, n, dtype=torch.bool)
    mask[:, start + key_tokens::record] = True
    return _place(device, inputs, targets, mask, None)


def random_batch(bs: int, n: int, g: torch.Generator, vocab_size: int):
    """Uniform token ids with full next-token supervision (throughput task)."""
    seq = torch.randint(vocab_size, (bs, n + 1), generator=g)
    return seq[:, :-1], seq[:, 1:], torch.ones(bs, n, dtype=torch.bool), None
