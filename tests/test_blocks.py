"""Streaming invariance: chunk sizes never change values."""
import torch

from exploration_b200.models.blocks import HaloMemoryBlock, KVProjection, RotaryEmbedding
from exploration_b200.ops.fused import local_attention_reference


def test_halo_chunk_invariance():
    torch.manual_seed(123)
    dim, heads, b = 16, 2, 8
    rope = RotaryEmbedding(dim // heads)
    ref = HaloMemoryBlock(dim, heads, b, rope, 4, query_chunk_size=64)
    fine = HaloMemoryBlock(dim, heads, b, rope, 4, query_chunk_size=1)
    fine.load_state_dict(ref.state_dict())
    ref, fine = ref.double().eval(), fine.double().eval()
    for n in (1, 3, 7, 8, 9, 37, 64):
        x = torch.randn(2, n, dim, dtype=torch.double)
        pos = torch.arange(n)
        with torch.no_grad():
            torch.testing.assert_close(fine(x, pos), ref(x, pos), rtol=1e-8, atol=1e-10)


def test_kv_projection_chunk_invariance():
    torch.manual_seed(123)
    dim, heads = 16, 2
    rope = RotaryEmbedding(dim // heads)
    ref = KVProjection(dim, heads, rope, use_rope=True)
    fine = KVProjection(dim, heads, rope, use_rope=True, chunk_tokens=4)
    fine.load_state_dict(ref.state_dict())
    ref, fine = ref.double().eval(), fine.double().eval()
    x = torch.randn(2, 37, dim, dtype=torch.double)
    pos = torch.arange(37)
    with torch.no_grad():
        k1, v1 = ref(x, pos)
        k2, v2 = fine(x, pos)
    torch.testing.assert_close(k2, k1, rtol=1e-8, atol=1e-10)
    torch.testing.assert_close(v2, v1, rtol=1e-8, atol=1e-10)


def _window_oracle(qkv, prev, start, valid_start, b):
    """Per-query loop: absolute-position windows, RoPE at (row, column - b)."""
    batch, n, _, heads, dim = qkv.shape
    rope = RotaryEmbedding(dim)
    out = torch.zeros(batch, n, heads, dim, dtype=qkv.dtype)
    keys = qkv if prev is None else torch.cat((prev, qkv), 1)
    key_base = start if prev is None else start - b
    for t in range(n):
        g, r = divmod(t, b)
        cols, weights_k, weights_v = [], [], []
        for c in range(2 * b):
            if c > b + r:
                continue
            key_abs = start + (g - 1) * b + c
            if not (valid_start <= key_abs < start + n):
                continue
            cols.append(c)
            weights_k.append(keys[:, key_abs - key_base, 1])
            weights_v.append(keys[:, key_abs - key_base, 2])
        kk = torch.stack(weights_k, 1)                       # [B,W,H,D]
        vv = torch.stack(weights_v, 1)
        q = rope(qkv[:, t, 0], torch.tensor(r))
        kk = rope(kk, torch.tensor(cols) - b)
        logits = torch.einsum("bhd,bwhd->bhw", q, kk) / dim ** 0.5
        out[:, t] = torch.einsum("bhw,bwhd->bhd", logits.softmax(-1), vv)
    return out.reshape(batch, n, heads * dim)


def test_local_attention_reference_matches_loop_oracle():
    torch.manual_seed(8)
    b, heads, dim = 4, 2, 6
    for n, with_prev in ((1, False), (5, True), (13, False), (16, True)):
        qkv = torch.randn(2, n, 3, heads, dim, dtype=torch.float64)
        prev = torch.randn(2, b, 3, heads, dim, dtype=torch.float64) if with_prev else None
        start = 8
        valid = start - b if with_prev else start
        got = local_attention_reference(qkv, prev, start, valid, n, b, heads)
        torch.testing.assert_close(got, _window_oracle(qkv, prev, start, valid, b), rtol=1e-10,
                                   atol=1e-12)
